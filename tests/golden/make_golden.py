"""Generate the golden fixtures by running the reference implementation.

Run in a checkout that has the reference's Python sources available:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

It imports czfsdg/vc-attention's ``vc_attention.core`` (the pure PyTorch
``reference`` backend) and records its outputs on the deterministic inputs of
tests/golden/cases.py into tests/golden/golden.npz and schedule.json.  The
GPU test box never runs this script; it only reads the committed fixtures.
"""
import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

from vc_attention import core  # noqa: E402  (the reference package)


def main():
    torch.set_num_threads(8)
    out = {}
    x = cases.expcast_inputs()
    out["expcast_codes"] = core.expcast_codes(x).numpy()

    for dim in (1, 16, 37, 64, 128):
        out[f"hadamard_{dim}"] = core.hadamard(cases.hadamard_input(dim)).numpy()

    for block in (64, 128, 256):
        xq = cases.quant_input(block)
        out[f"quant_{block}"] = core._quantize_qk(xq, block).numpy()
        payloads = []
        for s in range(0, xq.shape[-2], block):
            payload, _ = core._encode(xq[..., s:s + block, :], (-2, -1))
            payloads.append(payload.view(torch.uint8))
        out[f"quant_payload_{block}"] = torch.cat(payloads, dim=-2).numpy()

    for mean_dtype in ("float16", "bfloat16", "float32"):
        cfg = core.Config(mean_dtype=mean_dtype)
        for kind, tile in (("exact", cases.exact_value_tile()), ("random", cases.random_value_tile())):
            payload, scale, stored = core.prepare_value_tile(tile, True, cfg)
            out[f"vtile_{kind}_{mean_dtype}_payload"] = payload.view(torch.uint8).numpy()
            out[f"vtile_{kind}_{mean_dtype}_scale"] = scale.numpy()
            out[f"vtile_{kind}_{mean_dtype}_stored"] = stored.numpy()
        payload, scale, stored = core.prepare_value_tile(cases.exact_value_tile(), False, cfg)
        out[f"vtile_inactive_{mean_dtype}_payload"] = payload.view(torch.uint8).numpy()
        out[f"vtile_inactive_{mean_dtype}_scale"] = scale.numpy()

    sv = cases.separated_values()
    spi, scenters = core.group_values(sv, clusters=8, iterations=2)
    out["group_sep_pi"] = spi.numpy().astype(np.int32)
    out["group_sep_centers"] = scenters.numpy()
    v = cases.clustered_values()
    pi, centers = core.group_values(v, clusters=8, iterations=2)
    out["group_pi"] = pi.numpy().astype(np.int32)
    out["group_centers"] = centers.numpy()
    pi3, centers3 = core.group_values(v, clusters=3, iterations=3, centers=centers[..., :3, :].clone())
    out["group_warm_pi"] = pi3.numpy().astype(np.int32)
    out["group_warm_centers"] = centers3.numpy()

    for name, (shape, cfg_kw, call_kw) in cases.ATTENTION_CASES.items():
        q, k, v = cases.attention_inputs(name)
        cfg = core.Config(**cfg_kw)
        result, stats = core.attention(q, k, v, cfg, **call_kw)
        if shape == "c1":
            result = result[:, :, ::cases.C1_ROW_STRIDE]
        out[f"attn_{name}"] = result.float().numpy()
        out[f"attn_{name}_tiles"] = np.array(stats["tiles"])

    np.savez_compressed(HERE / "golden.npz", **out)

    cfg = core.Config(v_smooth=True)
    cache = core.LayoutCache(cfg)
    records = []
    base_v = cases.clustered_values(tokens=64, heads=1, dim=8)
    last_pi = None
    for request, step, total, trim in cases.schedule_script():
        vv = base_v[:, :, : base_v.shape[2] - trim]
        pi, active, refreshed = cache.layout(vv, step=step, total_steps=total, request_id=request, layer_id=0)
        records.append({"request": request, "step": step, "total_steps": total, "trim": trim,
                        "active": bool(active), "refreshed": bool(refreshed), "has_pi": pi is not None,
                        "same_pi_as_previous": bool(pi is not None and pi is last_pi),
                        "entries": cache.entries})
        last_pi = pi
    (HERE / "schedule.json").write_text(json.dumps(records, indent=1) + "\n")
    print("wrote", HERE / "golden.npz", sum(a.nbytes for a in out.values()) / 1e6, "MB raw")


if __name__ == "__main__":
    main()
