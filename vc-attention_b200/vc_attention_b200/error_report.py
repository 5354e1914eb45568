"""Error report for the b200_fp8 backend on the synthetic benchmark inputs.

The reference's CUDA benchmark compares a native output with an FP32 golden
and with its own quantised Python algorithm on the same inputs
(scripts/benchmark_cuda.py:152-183).  This CLI does the same for B200:

* ``native``: ``attention`` with ``Config(backend="b200_fp8")`` on the GPU,
  over all query rows (sampling Q first would change the per-block Q scales);
* ``fp32``: exact softmax attention in FP64 for a sample of query rows,
  spread evenly over the sequence;
* ``reference`` (when the upstream ``vc_attention`` package is importable):
  its ``reference`` backend on the same inputs and step.

It prints one JSON object with relative RMSE, max abs error and cosine for
native vs fp32, reference vs fp32 and native vs reference, per mode:

    python -m vc_attention_b200.error_report --config c2 --heads 2 --seq 4096
"""
from __future__ import annotations

import argparse
import json

import torch

MODES = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False),
         "combined": (True, True)}


def query_rows(length, count):
    """``count`` query rows spread evenly over [0, length), first and last included."""
    if count >= length:
        return list(range(length))
    if count == 1:
        return [0]
    return sorted({round(i * (length - 1) / (count - 1)) for i in range(count)})


@torch.no_grad()
def fp32_golden(q, k, v, rows, scale):
    """softmax(q[rows] k^T * scale) v in FP64 for BNSD tensors; returns
    [B, H, len(rows), Dv] FP64 on the inputs' device."""
    ids = torch.tensor(rows, device=q.device)
    qs = q.index_select(2, ids).double()
    s = torch.matmul(qs, k.double().transpose(-1, -2)) * scale
    return torch.matmul(torch.softmax(s, dim=-1), v.double())


def metrics(sample, golden):
    """Relative RMSE, max abs error and cosine of ``sample`` against ``golden``
    (the definitions of replay.py:20-32)."""
    x, g = sample.double().flatten(), golden.double().flatten()
    if not bool(torch.isfinite(x).all()):
        raise ValueError("non-finite attention output")
    delta = x - g
    rmse = delta.square().mean().sqrt()
    return {
        "relative_rmse": (rmse / g.square().mean().sqrt().clamp_min(1e-12)).item(),
        "max_abs": delta.abs().max().item(),
        "cosine": (torch.dot(x, g) / (x.norm() * g.norm()).clamp_min(1e-300)).item(),
    }


def _upstream_reference():
    try:
        from vc_attention import Config as RefConfig, attention as ref_attention
    except ImportError:
        return None
    return RefConfig, ref_attention


def report(*, config="c2", heads=2, seq=4096, seed=0, modes=tuple(MODES), rows=64, step=0, total_steps=4,
           device="cuda", reference_device="cpu"):
    from . import Config, attention
    from .synthetic import make_qkv

    q, k, v = (x.to(device) for x in make_qkv(config, seed, heads=heads, seq=seq, step=step))
    scale = q.shape[-1] ** -0.5
    ids = query_rows(q.shape[2], rows)
    golden = fp32_golden(q, k, v, ids, scale).cpu()
    upstream = _upstream_reference()
    out = {"config": config, "heads": heads, "seq": seq, "seed": seed, "step": step, "total_steps": total_steps,
           "dtype": str(q.dtype), "rows": len(ids), "reference": "vc_attention" if upstream else "not importable",
           "modes": {}}
    pick = torch.tensor(ids)
    for mode in modes:
        smooth, cast = MODES[mode]
        native, stats = attention(q, k, v, Config(v_smooth=smooth, expcast=cast), step=step,
                                  total_steps=total_steps, scale=scale)
        native = native.float().cpu().index_select(2, pick)
        entry = {"native_vs_fp32": metrics(native, golden), "smoothing_active": stats["smoothing_active"]}
        if upstream:
            ref_config, ref_attention = upstream
            rq, rk, rv = (x.to(reference_device) for x in (q, k, v))
            ref, _ = ref_attention(rq, rk, rv, ref_config(v_smooth=smooth, expcast=cast, backend="reference"),
                                   step=step, total_steps=total_steps, scale=scale)
            ref = ref.float().cpu().index_select(2, pick)
            entry["reference_vs_fp32"] = metrics(ref, golden)
            entry["native_vs_reference"] = metrics(native, ref)
        out["modes"][mode] = entry
    return out


def load_capture(path):
    """Q/K/V and metadata of a capture written by ``lightx2v.capture`` (or by
    the reference adapter, lightx2v.py:92-125), with the file's identity as
    the reference's replay records it (replay.py:80-89)."""
    import hashlib
    from pathlib import Path

    path = Path(path)
    record = torch.load(path, map_location="cpu", weights_only=True)
    q, k, v = (record[name] for name in ("q", "k", "v"))
    source = {"kind": "captured_qkv", "file": str(path.resolve()),
              "sha256": hashlib.sha256(path.read_bytes()).hexdigest(), "metadata": record["metadata"]}
    return q, k, v, source


def query_slice(q, q_start, q_limit):
    """Rows [q_start, q_start + q_limit) of Q (all rows from q_start when
    q_limit is 0); q_start must be a 128-row block boundary inside Q, so the
    slice's Q blocks quantise exactly as in the full call (replay.py:92-96).
    K and V are never cropped."""
    if q_start % 128 or not 0 <= q_start < q.shape[-2]:
        raise ValueError("q-start must be a valid 128-token block boundary")
    end = q.shape[-2] if q_limit == 0 else min(q.shape[-2], q_start + q_limit)
    return q[..., q_start:end, :]


def replay(path, *, modes=tuple(MODES), rows=64, q_start=0, q_limit=0, device="cuda", reference_device="cpu"):
    """The error report on a captured post-RoPE Q/K/V (replay.py:80-96): the
    capture's softmax scale and step, a 128-aligned query slice against the
    full K/V, each mode's native output against the FP64 softmax of the same
    rows (and against the upstream reference backend when importable)."""
    from . import Config, attention

    q, k, v, source = load_capture(path)
    meta = source["metadata"]
    scale, step, total = float(meta["scale"]), int(meta.get("step", 0)), int(meta.get("total_steps", 1))
    q = query_slice(q, q_start, q_limit)
    q, k, v = (x.to(device) for x in (q, k, v))
    ids = query_rows(q.shape[2], rows)
    golden = fp32_golden(q, k, v, ids, scale).cpu()
    upstream = _upstream_reference()
    pick = torch.tensor(ids)
    out = {"source": source, "q_start": q_start, "q_rows": q.shape[2], "kv_tokens": k.shape[2],
           "rows": len(ids), "step": step, "total_steps": total,
           "reference": "vc_attention" if upstream else "not importable", "modes": {}}
    for mode in modes:
        smooth, cast = MODES[mode]
        native, stats = attention(q, k, v, Config(v_smooth=smooth, expcast=cast), step=step, total_steps=total,
                                  scale=scale)
        native = native.float().cpu().index_select(2, pick)
        entry = {"native_vs_fp32": metrics(native, golden), "smoothing_active": stats["smoothing_active"]}
        if upstream:
            ref_config, ref_attention = upstream
            rq, rk, rv = (x.to(reference_device) for x in (q, k, v))
            ref, _ = ref_attention(rq, rk, rv, ref_config(v_smooth=smooth, expcast=cast, backend="reference"),
                                   step=step, total_steps=total, scale=scale)
            ref = ref.float().cpu().index_select(2, pick)
            entry["reference_vs_fp32"] = metrics(ref, golden)
            entry["native_vs_reference"] = metrics(native, ref)
        out["modes"][mode] = entry
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--capture", help="replay a captured Q/K/V file instead of the synthetic inputs")
    ap.add_argument("--q-start", type=int, default=0, help="with --capture: first query row (multiple of 128)")
    ap.add_argument("--q-limit", type=int, default=0, help="with --capture: query rows (0 = to the end)")
    ap.add_argument("--config", default="c2", choices=("c1", "c2", "c3", "c4", "c5"))
    ap.add_argument("--heads", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--mode", action="append", choices=sorted(MODES), help="repeatable; default: all four")
    ap.add_argument("--rows", type=int, default=64, help="query rows compared against the FP32 golden")
    ap.add_argument("--step", type=int, default=0)
    ap.add_argument("--total-steps", type=int, default=4)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--reference-device", default="cpu")
    a = ap.parse_args(argv)
    if a.rows < 1 or a.heads < 1 or a.seq < 1 or not 0 <= a.step < a.total_steps:
        ap.error("rows, heads and seq must be positive and 0 <= step < total-steps")
    if a.capture:
        if a.q_start % 128 or a.q_start < 0 or a.q_limit < 0:
            ap.error("q-start must be a non-negative multiple of 128 and q-limit non-negative")
        res = replay(a.capture, modes=tuple(a.mode or MODES), rows=a.rows, q_start=a.q_start, q_limit=a.q_limit,
                     device=a.device, reference_device=a.reference_device)
        print(json.dumps(res, indent=2))
        return 0
    res = report(config=a.config, heads=a.heads, seq=a.seq, seed=a.seed, modes=tuple(a.mode or MODES),
                 rows=a.rows, step=a.step, total_steps=a.total_steps, device=a.device,
                 reference_device=a.reference_device)
    print(json.dumps(res, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
