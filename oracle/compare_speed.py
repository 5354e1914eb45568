"""Times the CPU restatement (oracle/) against the reference's own ``reference``
backend on the same configuration-1 inputs and the same thread count, so the
``port`` CPU baseline that bench.py reports can be set beside the reference's
speed.  Runs only where the reference is importable (the build container):

    PYTHONPATH=<reference>/src python oracle/compare_speed.py [--threads 8] [--reps 3]

Test infrastructure: nothing in the product imports this file."""
from __future__ import annotations

import argparse
import json
import pathlib
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "vc-attention_b200"))
sys.path.insert(0, str(ROOT))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=8)
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    import numpy as np
    import torch
    from threadpoolctl import threadpool_limits

    from oracle import oracle as O
    from vc_attention_b200.synthetic import make_qkv

    import vc_attention.core as ref

    torch.set_num_threads(a.threads)
    q, k, v = make_qkv("c1", 20260917)         # B1 H2 S2048 D128 fp32
    res = {"config": "c1: B1 H2 S2048 D128 fp32, step 0 of 4", "threads": a.threads, "modes": {}}
    for mode, (smooth, cast) in {"fp8_control": (False, False), "expcast": (False, True),
                                 "v_smooth": (True, False), "combined": (True, True)}.items():
        cfg = ref.Config(v_smooth=smooth, expcast=cast)
        t_ref, t_port = [], []
        for _ in range(a.reps):
            t0 = time.perf_counter()
            out_ref, _ = ref.attention(q, k, v, cfg, step=0, total_steps=4)
            t_ref.append(time.perf_counter() - t0)
            flat = [x[0].numpy() for x in (q, k, v)]
            t0 = time.perf_counter()
            with threadpool_limits(limits=1):
                pi = O.group_values(flat[2], clusters=8, iterations=2)[0] if smooth else None
                out_port = O.attention(*flat, expcast=cast, active=smooth, pi=pi, threads=a.threads, row_chunk=128)
            t_port.append(time.perf_counter() - t0)
        m = O.metrics(out_port, out_ref[0].numpy())
        res["modes"][mode] = {"reference_ms": 1e3 * min(t_ref), "port_ms": 1e3 * min(t_port),
                              "port_over_reference": min(t_port) / min(t_ref),
                              "outputs_relative_rmse": m["relative_rmse"]}
    print(json.dumps(res, indent=2))


if __name__ == "__main__":
    main()
