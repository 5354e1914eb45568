"""Deterministic inputs shared by make_golden.py and the tests.

Every input is regenerated from a seeded CPU ``torch.Generator`` so the
committed fixtures only hold the reference's outputs.
"""
import math
import struct

import torch

# Known-answer ExpCast inputs from the reference's own tests.
KNOWN_U = [0.0, -1.0, -1.6, -8.0, -14.0, -100.0, -float("inf")]      # test_core.py:19
KNOWN_CODES = [120, 112, 107, 56, 8, 0, 0]                             # test_core.py:21
KNOWN_DECODED = [256, 128, 88, 1, 2 ** -6, 0, 0]                       # test_core.py:22
FMA_BITS = [0xc1226786, 0xc12104a2, 0xc11cdbf5, 0xc118b349, 0xc1148a9c, 0xc11327b8,
            0xc10ad65f, 0xc106adb2, 0xc1028506, 0xc0ff7e7b, 0xc0fcb8b2, 0xc0f72d21]  # test_paper_alignment.py:233-234
FMA_CODES = [3, 3, 7, 9, 13, 13, 19, 23, 25, 27, 29, 31]               # test_paper_alignment.py:236


def expcast_inputs():
    """Known answers, the 12 single-FMA regressions, every code boundary +-1 ulp,
    specials and a dense random sweep over [-24, 1]."""
    known = torch.tensor(KNOWN_U) / math.log2(math.e)
    fma = torch.tensor([struct.unpack("<f", struct.pack("<I", v))[0] for v in FMA_BITS])
    boundary = (torch.arange(120, dtype=torch.float32) + 0.5 - 119.65) / (8 * math.log2(math.e))
    edges = torch.cat([boundary, torch.nextafter(boundary, torch.full_like(boundary, -math.inf)),
                       torch.nextafter(boundary, torch.full_like(boundary, math.inf))])
    special = torch.tensor([0.0, -0.0, -1e6, -math.inf, 1e-30, -1e-30, 0.01, 0.05])
    g = torch.Generator().manual_seed(7)
    sweep = torch.rand(200_000, generator=g) * 25.0 - 24.0
    return torch.cat([known, fma, edges, special, sweep]).float()


def hadamard_input(dim):
    g = torch.Generator().manual_seed(31 + dim)
    return torch.randn(2, 3, 7, dim, generator=g)


def quant_input(block):
    g = torch.Generator().manual_seed(100 + block)
    x = torch.randn(1, 2, 300, 128, generator=g)
    x[:, :, :40] *= 1e-3          # a block with a tiny scale
    x[:, 1, 128:256] *= 50.0      # and one with a large scale
    x[:, 0, 256:] = 0.0           # an all-zero tail block (scale 0 -> 1)
    return x


def exact_value_tile():
    """Values on a 1/64 grid with |v| < 8: every partial sum is exact in FP32,
    so the block mean does not depend on the summation order."""
    g = torch.Generator().manual_seed(13)
    return (torch.randint(-128, 128, (1, 2, 128, 21), generator=g).float() / 64.0 + 3.0)


def random_value_tile():
    g = torch.Generator().manual_seed(13)                  # test_paper_alignment.py:207-208
    return torch.randn(1, 2, 35, 21, generator=g) * 0.17 + 3.14159


def clustered_values(tokens=1000, heads=2, dim=16, seed=5):
    g = torch.Generator().manual_seed(seed)
    centers = torch.randn(1, heads, 8, dim, generator=g) * 8
    ids = torch.randint(0, 8, (1, heads, tokens, 1), generator=g).expand(1, heads, tokens, dim)
    return centers.gather(-2, ids) + 0.1 * torch.randn(1, heads, tokens, dim, generator=g)


def separated_values(tokens=1000, heads=2, dim=16, seed=6):
    """Tokens grouped by cluster, so the equispaced initialisation hits every
    cluster once and no token sits near a decision boundary."""
    g = torch.Generator().manual_seed(seed)
    centers = torch.randn(1, heads, 8, dim, generator=g) * 2
    ids = (torch.arange(tokens) * 8 // tokens).view(1, 1, tokens, 1).expand(1, heads, tokens, dim)
    return centers.gather(-2, ids) + 0.05 * torch.randn(1, heads, tokens, dim, generator=g)


def reference_test_inputs(shape, seed=1234):
    """test_cuda.py:62-69: Q, K ~ N(0,1); V ~ 0.2 N(0,1) + 3 (observable mean)."""
    batch, heads, nq, nk, d, dv = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, heads, nq, d, generator=g)
    k = torch.randn(batch, heads, nk, d, generator=g)
    v = torch.randn(batch, heads, nk, dv, generator=g) * 0.2 + 3.0
    return q, k, v


# Attention cases: name -> (shape or "c1", config kwargs, call kwargs).
ARMS = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False),
        "combined": (True, True)}                                     # replay.py:17

ATTENTION_CASES = {}
for _arm, (_smooth, _cast) in ARMS.items():
    ATTENTION_CASES[f"small_{_arm}"] = ((1, 1, 19, 35, 16, 16), dict(v_smooth=_smooth, expcast=_cast, clusters=1), {})
    ATTENTION_CASES[f"tile_{_arm}"] = ((1, 2, 129, 257, 128, 128), dict(v_smooth=_smooth, expcast=_cast), {})
    ATTENTION_CASES[f"odd_{_arm}"] = ((2, 2, 33, 145, 37, 21), dict(v_smooth=_smooth, expcast=_cast, clusters=1), {})
    ATTENTION_CASES[f"c1_{_arm}"] = ("c1", dict(v_smooth=_smooth, expcast=_cast), dict(step=0, total_steps=4))
ATTENTION_CASES["meanbf16_kq512"] = ((1, 1, 300, 700, 64, 48),
                                     dict(v_smooth=True, expcast=True, mean_dtype="bfloat16", k_quant_block=512), {})
ATTENTION_CASES["meanfp32_q64"] = ((1, 1, 200, 300, 64, 64),
                                   dict(v_smooth=True, expcast=False, mean_dtype="float32", q_block=64), {})
ATTENTION_CASES["scale007_nosmooth"] = ((1, 2, 130, 260, 37, 21),
                                        dict(v_smooth=True, expcast=True, k_smooth=False, qk_hadamard=False),
                                        dict(scale=0.07))
ATTENTION_CASES["kq128_rot_only"] = ((1, 1, 140, 390, 128, 128),
                                     dict(v_smooth=False, expcast=True, k_smooth=False, k_quant_block=128), {})


def attention_inputs(name):
    shape, _, _ = ATTENTION_CASES[name]
    if shape == "c1":
        import sys
        import pathlib
        sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[2] / "vc-attention_b200"))
        from vc_attention_b200.synthetic import make_qkv
        return make_qkv("c1", 20261201)
    return reference_test_inputs(shape)


C1_ROW_STRIDE = 16    # c1 fixtures keep every 16th query row


def schedule_script():
    """Steps fed to one LayoutCache: (request, step, total_steps, shape_trim)."""
    seq = [("a", s, 50, 0) for s in range(0, 20)]
    seq += [("a", 3, 50, 0)]                  # reversed step -> state reset
    seq += [("b", 0, 20, 0), ("b", 1, 20, 1), ("b", 2, 20, 1), ("b", 5, 20, 1)]
    return seq
