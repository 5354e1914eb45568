"""Programmatic dependent launch needs every grid launched with programmatic
stream serialisation to wait for its predecessor before it touches memory:
such a grid may start while the previous grid in the stream is still running.
This reads the kernel sources and checks that each kernel named in a
``launch_pdl(...)`` call, and each kernel that ``launch_pairs`` launches, begins
with ``pdl_wait();`` (``griddepcontrol.wait``)."""
import pathlib
import re

CSRC = pathlib.Path(__file__).resolve().parents[1] / "vc-attention_b200" / "csrc"


def _sources():
    return {p.name: p.read_text() for p in sorted(CSRC.glob("*.cu"))}


def _first_statement(src, name):
    """The first statement in the body of every __global__ function called `name`."""
    out = []
    for m in re.finditer(r"__global__[^;{]*?\b" + re.escape(name) + r"\s*\(", src):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        body = src[src.index("{", i) + 1:]
        body = re.sub(r"//[^\n]*", "", body)
        out.append(body.strip().split(";", 1)[0].strip())
    return out


def _launched_with_pdl(srcs):
    names = set()
    for src in srcs.values():
        for m in re.finditer(r"launch_pdl\(\s*([A-Za-z_]\w*)", src):
            names.add(m.group(1))
    return names


def test_every_pdl_launched_kernel_waits_first():
    srcs = _sources()
    names = _launched_with_pdl(srcs)
    # the staged quantiser is launched through a local alias
    if "kernel" in names:
        names.discard("kernel")
        names.add("qk_quant_staged_kernel")
    names.add("attn_kernel")          # launch_pairs sets the attribute for the attention kernels
    assert {"cluster_assign128_kernel", "k_colsum_kernel", "vprep_kernel", "qk_quant_kernel"} <= names
    seen = {}
    for name in sorted(names):
        firsts = [s for src in srcs.values() for s in _first_statement(src, name)]
        assert firsts, f"no __global__ definition found for {name}"
        seen[name] = firsts
        assert all(s == "pdl_wait()" for s in firsts), (name, firsts)
    assert len(seen["attn_kernel"]) == 2          # the ExpCast and the exp-mode kernels


def test_launch_pairs_sets_programmatic_serialisation():
    src = (CSRC / "vcb_attn_pair.cuh").read_text()
    body = src[src.index("int launch_pairs("):]
    assert "cudaLaunchAttributeProgrammaticStreamSerialization" in body
