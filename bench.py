"""Benchmark of the b200_fp8 VC-Attention forward (configuration 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one full forward of the hot path over one batch on each GPU:
Lloyd clustering of V (a refresh step), Q/K demean + Hadamard + E4M3 block
quantisation, V tiles, and the fused tcgen05 attention; B=1, H=40, S=32768,
D=128, bf16 inputs, combined mode (ExpCast + V-Smooth), step 0 of 50.  With
N GPUs (torchrun) the 40 heads are split into contiguous ranges, 40/N per
rank (strong scaling: configuration 3 shards 5 heads per GPU at N=8); heads
are independent, so no collective touches the data path.

value     FP8 attention TFLOPS of the whole job, 4*B*H*S^2*D per step over
          the CUDA-event time of the step with inputs resident in HBM (max
          over ranks).  Q/K/V (1 GB) exceed the 126 MB L2, so no flush is needed.
e2e       the same metric through the public API for host-resident tensors
          (vc_attention_b200.attention_streamed): pinned Q/K/V in, pinned
          output back, every byte of both copies inside every timed step
          (overlapped with the forward chunk by chunk over the heads).
roofline  the fused attention kernel alone, timed with CUDA events on its
          stream, against the FP8 dense tensor peak measured in the same run
          (torch._scaled_mm, 8192^3, E4M3 -> BF16).
cpu_baseline / --impl reference
          the CPU restatement of the reference backend (oracle/) on the host
          cores, on a bounded sample (one head: all 256 query tiles over all
          keys for the baseline leg, 128 per step for --impl reference, with
          that head's full preprocessing), scaled to TFLOPS.

Other cases (not the bench line):
    --case attn|prep --heads H    small single-GPU cases for ncu
    --case ulysses                configuration 4 sequence-sharded (torchrun)
    --case schedule [--heads H --seq S]
                                  configuration 5's 50-step denoising loop in
                                  every mode, step times per schedule phase
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vc-attention_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

B, H, S, D = 1, 40, 32768, 128
METRIC = "FP8 attn fwd TFLOPS/GPU (4*B*H*S^2*D/t) at S=32k; % of FP8 MMA peak"
UNIT = "TFLOPS"
LAUNCHES_PER_STEP = 13   # clustering 7 (init, 2 x (assign, update), offsets, scatter), Q/K 4, V 1, attention 1
CONFIG = {"workload": "c3: B1 H40 S32768 D128 bf16 combined (ExpCast + V-Smooth), refresh step 0/50",
          "global_batch": None, "seq_len": S, "heads": H, "head_dim": D, "parallelism": None,
          "l2": "inputs (1 GB Q/K/V per GPU) larger than L2; no flush"}


def flops(b=B, h=H, sq=S, sk=S, d=D):
    return 4.0 * b * h * sq * sk * d


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during a region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def fp8_peak_tflops(device):
    """Dense E4M3 GEMM throughput of this GPU (cuBLAS via torch._scaled_mm)."""
    n = 8192
    a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=device)
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    best = float("inf")
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(10):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e) / 10)
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def cpu_reference(threads, heads=1, q_tiles=256):
    """Times the CPU restatement of the reference backend on one head: the
    full O(S) preprocessing (Lloyd, Q/K quantisation, V tiles) plus the
    streaming attention of `q_tiles` 128-row query tiles over all S keys."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import oracle as O
    from vc_attention_b200.synthetic import make_qkv

    q, k, v = make_qkv("c3", 1234, heads=heads)
    flat = [x.float().reshape(heads, S, D).numpy() for x in (q, k, v)]
    rows = q_tiles * 128
    t0 = time.perf_counter()
    with threadpool_limits(limits=1):
        pi, _, _ = O.group_values(flat[2], clusters=8, iterations=2)
        prep = O.Prepared(flat[0][:, :rows], flat[1], flat[2], pi=pi, active=True, q_block=128,
                          k_quant_block=256, kv_block=128, mean_dtype="float16", k_smooth=True, qk_hadamard=True)
        from concurrent.futures import ThreadPoolExecutor
        chunks = [slice(r, r + 128) for r in range(0, rows, 128)]
        with ThreadPoolExecutor(max_workers=threads) as pool:
            outs = list(pool.map(lambda sl: O.stream(prep, sl, expcast=True, scale=D ** -0.5), chunks))
    dt = time.perf_counter() - t0
    assert all(np.isfinite(o).all() for o in outs)
    sample_flops = flops(1, heads, rows, S, D)
    return {"value": sample_flops / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{heads} head(s), {q_tiles} query tiles x {S} keys, with the head's full clustering, "
                      f"Q/K and V preprocessing; {dt:.2f} s"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    times = []
    q_tiles = 128          # half a head per step: a whole --steps 10 --warmup 3 run stays near a minute
    for i in range(args.warmup + args.steps):
        r = cpu_reference(threads, q_tiles=q_tiles)
        if i >= args.warmup:
            times.append(r)
    value = statistics.median(x["value"] for x in times)
    cpu = dict(times[0])
    cpu["value"] = value
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": flops(1, 1, q_tiles * 128, S, D) / value / 1e9,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(CONFIG, global_batch=1, parallelism="cpu"), "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def _e4m3(b):
    return b.view(torch.float8_e4m3fn).float()


@torch.no_grad()
def rows_check(q, k, v, out, cfg, *, head, r0, pi, active, scale=D ** -0.5):
    """Checks 128 rows of one head of a GPU forward on the GPU that ran it.

    The reference's streaming loop (core.py:307-340) is evaluated with torch
    in FP32 (no TF32) over the library's own prepared operands of that head
    (E4M3 Q/K blocks and V tiles, whose bytes the GPU tests pin to the CPU
    checker), with the reference's FP64-intermediate ExpCast encode
    (core.py:60-68).  This needs no host-side checker, so it runs on every
    rank of a multi-GPU job.  Returns relative RMSE and cosine against the
    fused kernel's output rows."""
    from vc_attention_b200 import stages

    hs = slice(head, head + 1)
    qh, kh, vh = (x[:, hs].contiguous() for x in (q, k, v))
    ph = None if pi is None else pi[:, hs].contiguous()
    q8, qs, k8, ks = stages.quantize_qk(qh, kh, pi=ph, q_block=cfg.q_block, k_quant_block=cfg.k_quant_block,
                                        k_smooth=cfg.k_smooth, hadamard=cfg.qk_hadamard)
    v8, meta, _ = stages.prepare_v(vh, pi=ph, active=active, mean_dtype=cfg.mean_dtype)
    sk, dv = k.shape[2], v.shape[3]
    rows = torch.arange(r0, r0 + 128, device=q.device)
    keys = torch.arange(sk, device=q.device)
    qd = _e4m3(q8[0, rows]) * qs[0, rows // cfg.q_block][:, None]
    kd = _e4m3(k8[0, :sk]) * ks[0, keys // cfg.k_quant_block][:, None]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        m = torch.full((128, 1), -float("inf"), device=q.device)
        den = torch.zeros((128, 1), device=q.device)
        acc = torch.zeros((128, dv), device=q.device)
        for j, s0 in enumerate(range(0, sk, 128)):
            kt = kd[s0:s0 + 128]
            s = (qd @ kt.T) * scale
            newmax = torch.maximum(m, s.amax(-1, keepdim=True))
            alpha = torch.exp(m - newmax)
            shifted = s - newmax
            if cfg.expcast:
                code = (shifted.double() * 11.541560173034668 + 119.6500015258789).float()
                p8 = torch.round(code).clamp(0, 120).to(torch.uint8).view(torch.float8_e4m3fn).float()
                prob = p8 / 256.0
            else:
                prob = torch.exp(shifted)
                p8 = (prob * 256.0).to(torch.float8_e4m3fn).float()
            mass = prob.sum(-1, keepdim=True)
            resid = _e4m3(v8[0, j, :dv, :kt.shape[0]]).T
            contrib = (p8 @ resid / 256.0 + mass * meta[0, j, 1, :dv]) * meta[0, j, 0, :dv]
            acc = alpha * acc + contrib
            den = alpha * den + mass
            m = newmax
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    ref = (acc / den).to(out.dtype).double().flatten()
    got = out[0, head, r0:r0 + 128].double().flatten()
    rel = float(((got - ref).square().mean() / ref.square().mean().clamp_min(1e-30)).sqrt())
    cos = float(torch.dot(got, ref) / (got.norm() * ref.norm()).clamp_min(1e-8))
    return {"relative_rmse": rel, "cosine": cos}


def copy_ceiling_ms(hq, hk, hv, hout, device, reps=3):
    """H2D of the step's inputs and D2H of its output alone (pinned host
    memory, one stream per direction, both directions at once): the time
    the e2e step could not beat even with the compute fully hidden."""
    dq, dk, dv = (torch.empty(x.shape, dtype=x.dtype, device=device) for x in (hq, hk, hv))
    do = torch.empty(hout.shape, dtype=hout.dtype, device=device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    best = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(device)
        s.record(cur)
        up.wait_stream(cur)
        down.wait_stream(cur)
        with torch.cuda.stream(up):
            for d, h in ((dq, hq), (dk, hk), (dv, hv)):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(down):
            hout.copy_(do, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)
        e.record(cur)
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return best


def chunked_copy_ceiling_ms(hq, hk, hv, hout, device, reps=3, nbuf=8):
    """The e2e pipeline's copy traffic alone: per chunk of heads (the
    default of attention_streamed, a twentieth of them) three H2D copies
    into a ring of `nbuf` device slots on one stream, and one D2H copy of a
    chunk-sized slot on another once that chunk has landed, a slot reused
    once its D2H is done.  Both directions then carry many mid-sized copies
    at once, as in the pipeline, which the link serves more slowly than one
    copy per direction."""
    bh = hq.shape[0] * hq.shape[1]
    size = max(1, math.ceil(bh / 20))
    parts = [(a, min(a + size, bh)) for a in range(0, bh, size)]
    nbuf = min(nbuf, len(parts))
    flat = [x.reshape(bh, x.shape[2], x.shape[3]) for x in (hq, hk, hv)]
    of = hout.reshape(bh, hout.shape[2], hout.shape[3])
    ring = [torch.empty((nbuf, size) + tuple(x.shape[1:]), dtype=x.dtype, device=device) for x in flat]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    best = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize(device)
        ready = [torch.cuda.Event() for _ in parts]
        free = [torch.cuda.Event() for _ in parts]
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(device)
        s.record(cur)
        up.wait_stream(cur)
        down.wait_stream(cur)
        for i, (a, b_) in enumerate(parts):
            slot, m = i % nbuf, b_ - a
            with torch.cuda.stream(up):
                if i >= nbuf:
                    up.wait_event(free[i - nbuf])
                for r, x in zip(ring, flat):
                    r[slot, :m].copy_(x[a:b_], non_blocking=True)
                ready[i].record(up)
            with torch.cuda.stream(down):
                down.wait_event(ready[i])
                of[a:b_].copy_(ring[0][slot, :m], non_blocking=True)
                free[i].record(down)
        cur.wait_stream(up)
        cur.wait_stream(down)
        e.record(cur)
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return best


def config4_object(args, world, rank, local):
    """Configuration 4 inside the multi-GPU bench line: B1 H24 S131072 D128
    bf16, combined mode at a refresh step, inputs sequence-sharded (S/N tokens
    of all 24 heads per rank); one step is the seq->head all-to-all of Q/K/V
    (NCCL), the forward on 24/N heads over all tokens, and the head->seq
    all-to-all of the output (lightx2v.py:119, :138-139).  Times are CUDA
    events, max over ranks; the check compares 128 rows of this rank's first
    head with rows_check."""
    from vc_attention_b200 import Config, LayoutCache, sharding
    from vc_attention_b200.synthetic import make_qkv

    heads, seq = 24, 131072
    device = torch.device("cuda", local)
    group = torch.distributed.group.WORLD
    s = seq // world
    q, k, v = (x[:, :, rank * s:(rank + 1) * s].contiguous() for x in make_qkv("c4", 2000, device=device))
    cfg = Config(v_smooth=True, expcast=True)

    def step(i):
        cache = LayoutCache(cfg)
        out, _ = sharding.attention_seq_sharded(q, k, v, cfg, group=group, cache=cache, step=0, total_steps=50,
                                                request_id=i)
        return out, cache

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(args.steps):
        out, cache = step(i)
    e0.record()
    e0.synchronize()
    ms = sharding.max_over_ranks(s0.elapsed_time(e0) / args.steps)
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s1.record()
    for _ in range(args.steps):
        hs = [sharding.seq_to_heads(x, group) for x in (q, k, v)]
        sharding.heads_to_seq(hs[0], group)
    e1.record()
    e1.synchronize()
    a2a_ms = sharding.max_over_ranks(s1.elapsed_time(e1) / args.steps)
    # check: this rank's heads over all tokens, taken back from the sequence-sharded output
    qh, kh, vh = (sharding.seq_to_heads(x, group) for x in (q, k, v))
    oh = sharding.seq_to_heads(out, group)
    pi = cache._states[0]["pi"]
    chk = rows_check(qh, kh, vh, oh, cfg, head=0, r0=4096 + 128 * rank, pi=pi, active=True)
    worst_rmse = sharding.max_over_ranks(chk["relative_rmse"])
    worst_cos = -sharding.max_over_ranks(-chk["cosine"])
    total = 4.0 * heads * seq * seq * 128
    return {"workload": "c4: B1 H24 S131072 D128 bf16 combined, refresh step, sequence-sharded inputs",
            "parallelism": f"Ulysses: seq->head all-to-all, {heads // world} heads per rank, head->seq all-to-all",
            "ms_per_step": ms, "tflops_total": total / (ms * 1e-3) / 1e12,
            "tflops_per_gpu": total / (ms * 1e-3) / 1e12 / world, "all_to_all_ms": a2a_ms,
            "parity": {"rows": "128 rows of each rank's first head", "relative_rmse_max": worst_rmse,
                       "cosine_min": worst_cos, "tolerance": {"relative_rmse": 1e-3, "cosine": 0.9999},
                       "ok": worst_rmse <= 1e-3 and worst_cos >= 0.9999}}


def run_ours(args, world, rank, local):
    from vc_attention_b200 import Config, LayoutCache, attention_streamed, check_streamed, sharding, stages
    from vc_attention_b200.b200_backend import forward, group_values
    from vc_attention_b200.synthetic import make_qkv

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = Config(v_smooth=True, expcast=True)
    q, k, v = (sharding.shard_heads(x, world, rank) for x in make_qkv("c3", 1000, device=device))
    h_loc = q.shape[1]
    torch.cuda.empty_cache()
    scale = D ** -0.5
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    workspace = None

    pi_step = None

    def step():
        nonlocal workspace, pi_step
        pi, _ = group_values(v, clusters=cfg.clusters, iterations=cfg.iterations)
        pi_step = pi
        if workspace is None:
            import ctypes
            from vc_attention_b200 import _abi
            from vc_attention_b200.b200_backend import forward_args, _extension
            need = _extension().vcb_forward_workspace(ctypes.byref(forward_args(q, k, v, cfg, pi, True, scale, out)))
            workspace = torch.empty(need, dtype=torch.uint8, device=device)
        forward(q, k, v, cfg, pi=pi, active=True, scale=scale, out=out, workspace=workspace, status=status,
                check_status=False)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        for s, e in ev:
            s.record()
            step()
            e.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = sum(s.elapsed_time(e) for s, e in ev) / args.steps
    if int(status.item()) != 0:
        raise RuntimeError(f"device status flags {int(status.item())}")
    ms_max = sharding.max_over_ranks(ms)
    value = flops() / (ms_max * 1e-3) / 1e12

    # dominant kernel alone: the fused attention on prepared operands
    pi, _ = group_values(v, clusters=8, iterations=2)
    q8, qs, k8, ks = stages.quantize_qk(q, k, pi=pi)
    v8, meta, _ = stages.prepare_v(v, pi=pi, active=True, mean_op=False)
    attn_out = torch.empty((h_loc, S, D), dtype=torch.bfloat16, device=device)

    def attn():
        stages.attention_fp8(q8, qs, k8, ks, v8, meta, heads=h_loc, sq=S, sk=S, dv=D, expcast=True,
                             has_mean=True,
                             scale=scale, out=attn_out)

    for _ in range(3):
        attn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, args.steps)
    s.record()
    for _ in range(reps):
        attn()
    e.record()
    e.synchronize()
    attn_ms = s.elapsed_time(e) / reps
    attn_ms = sharding.max_over_ranks(attn_ms)
    achieved = flops(h=h_loc) / (attn_ms * 1e-3) / 1e12
    peak = fp8_peak_tflops(device)
    traffic, traffic_note = None, None
    tfile = ROOT / "profiles" / "attn_kernel_traffic.json"
    if tfile.exists():
        rec = json.loads(tfile.read_text())
        traffic = rec["bytes_per_launch_full_c3"] * h_loc / H
        traffic_note = (f"not measured in this run: DRAM bytes of one ncu capture ({rec['captured_case']}), "
                        f"scaled per head to this rank's {h_loc} heads ({tfile.relative_to(ROOT)})")

    # 128 rows of one head of the timed forward, checked on this GPU (max over ranks)
    chk = rows_check(q, k, v, out, cfg, head=h_loc - 1, r0=128 * (37 + 11 * rank), pi=pi_step, active=True)
    parity = {"rows": "128 query rows of each rank's last head, full K/V (replay semantics)",
              "relative_rmse_max": sharding.max_over_ranks(chk["relative_rmse"]),
              "cosine_min": -sharding.max_over_ranks(-chk["cosine"]),
              "tolerance": {"relative_rmse": 1e-3, "cosine": 0.9999},
              "reference": "core.py:307-340 in torch FP32 (FP64-intermediate ExpCast) over this library's "
                           "prepared operands"}
    parity["ok"] = parity["relative_rmse_max"] <= 1e-3 and parity["cosine_min"] >= 0.9999

    # end to end through the public API, host buffers in and out
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    barrier(world)
    e2e_ms, e2e_stats = [], []
    # the host issues every chunk's copies and launches inside the timed
    # region, so a garbage-collector pause there would stall the GPU
    gc.collect()
    gc.disable()
    # at least 20 timed steps (about 0.5 s), so that a few steps stretched by
    # other load on a shared host cannot move the median
    e2e_steps = max(args.steps, 20)
    for i in range(args.warmup + e2e_steps):
        torch.cuda.synchronize()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        # host in, host out: per-chunk H2D, forwards on rotating compute streams, D2H
        _, st = attention_streamed(hq, hk, hv, cfg, cache=LayoutCache(cfg), step=0, total_steps=50,
                                   request_id=i, device=device, out=hout, synchronize=False)
        e.record()
        e.synchronize()
        e2e_stats.append(st)
        if i >= args.warmup:
            e2e_ms.append(s.elapsed_time(e))
    gc.enable()
    # every e2e step's device status is read after the timed loop: a step
    # whose kernels flagged non-finite input, an expired wait or a failed
    # layout check invalidates the e2e figure (check_streamed raises)
    for st in e2e_stats:
        check_streamed(st)
    # The e2e figure is the median step (max over ranks of each rank's
    # median): the host issues every chunk's copies and launches inside the
    # step, so a few steps can be stretched by other load on a shared host
    # (one box showed single steps of 56-306 ms among 22 ms ones); the mean
    # and every step stay in the line.
    e2e_mean = sharding.max_over_ranks(sum(e2e_ms) / len(e2e_ms))
    e2e = sharding.max_over_ranks(statistics.median(e2e_ms))
    ceiling = sharding.max_over_ranks(copy_ceiling_ms(hq, hk, hv, hout, device))
    ceiling_chunked = sharding.max_over_ranks(chunked_copy_ceiling_ms(hq, hk, hv, hout, device))
    c4 = config4_object(args, world, rank, local) if world > 1 and not args.no_config4 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(len(os.sched_getaffinity(0)))
    if rank == 0:
        nbytes = q.numel() * q.element_size()
        line = {
            "metric": METRIC, "value": value, "value_per_gpu": value / world, "unit": UNIT, "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e4m3 (bf16 in/out, fp32 accumulate)", "data": "synthetic",
            "config": dict(CONFIG, global_batch=1,
                           parallelism=f"{world} rank(s), {h_loc} heads each (contiguous head ranges), "
                                       "no collective"),
            "e2e": {"value": flops() / (e2e * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e,
                    "estimator": "median step time, max over ranks of each rank's median",
                    "ms_per_step_mean": e2e_mean,
                    "value_from_mean": flops() / (e2e_mean * 1e-3) / 1e12,
                    "steps_ms": [round(t, 3) for t in e2e_ms], "timed_steps": e2e_steps,
                    "h2d_bytes_per_step": 3 * nbytes, "d2h_bytes_per_step": nbytes,
                    "status_checked": True,
                    "copy_ceiling_ms": ceiling,
                    "frac_of_copy_ceiling": ceiling / e2e,
                    "copy_ceiling": "the same H2D and D2H bytes alone, pinned, one stream per direction, "
                                    "max over ranks",
                    "copy_ceiling_chunked_ms": ceiling_chunked,
                    "frac_of_chunked_copy_ceiling": ceiling_chunked / e2e,
                    "copy_ceiling_chunked": "the pipeline's own copies alone: per chunk of heads three H2D "
                                            "copies into a ring of 8 device slots and one chunk-sized D2H, "
                                            "the two directions at once, max over ranks"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_note,
                         "kernel": "attn_kernel",
                         "kernel_ms": attn_ms,
                         "peak_source": "measured in this run: torch._scaled_mm E4M3 8192^3 burst",
                         "frac_of_spec_4500": achieved / 4500.0},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "parity": parity,
            "config4": c4,
        }
        print(json.dumps(line))


def run_ulysses(args, world, rank, local):
    """Configuration 4 on N GPUs: B1 H24 S131072 D128 bf16, combined mode,
    inputs sequence-sharded (S/N tokens of all heads per rank).  A step is the
    seq->head all-to-all of Q/K/V, the forward on 24/N heads over all tokens,
    and the head->seq all-to-all of the output.  Prints one JSON line (rank 0)
    with the step time (max over ranks) and the share of the all-to-alls."""
    from vc_attention_b200 import Config, sharding
    from vc_attention_b200.synthetic import make_qkv

    heads, seq = 24, 131072
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    q, k, v = make_qkv("c4", 2000, device=device)
    s = seq // world
    q, k, v = (x[:, :, rank * s:(rank + 1) * s].contiguous() for x in (q, k, v))
    torch.cuda.empty_cache()
    cfg = Config(v_smooth=True, expcast=True)
    group = torch.distributed.group.WORLD if world > 1 else None

    def step():
        if world == 1:
            from vc_attention_b200 import attention
            return attention(q, k, v, cfg)[0]
        return sharding.attention_seq_sharded(q, k, v, cfg, group=group)[0]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(args.steps):
        step()
    e0.record()
    e0.synchronize()
    ms = sharding.max_over_ranks(s0.elapsed_time(e0) / args.steps)
    a2a_ms = 0.0
    if world > 1:   # the two all-to-alls alone
        s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s1.record()
        for _ in range(args.steps):
            hs = [sharding.seq_to_heads(x, group) for x in (q, k, v)]
            sharding.heads_to_seq(hs[0], group)
        e1.record()
        e1.synchronize()
        a2a_ms = sharding.max_over_ranks(s1.elapsed_time(e1) / args.steps)
    if rank == 0:
        total = 4.0 * heads * seq * seq * 128
        print(json.dumps({"case": "ulysses", "workload": "c4: B1 H24 S131072 D128 bf16 combined, sequence-sharded",
                          "n_gpus": world, "steps": args.steps, "ms_per_step": ms,
                          "tflops_total": total / (ms * 1e-3) / 1e12, "all_to_all_ms": a2a_ms}))


def run_case(args):
    """Small single-GPU cases for profilers (ncu): `--case attn` runs the
    fused attention on prepared operands, `--case prep` the clustering, Q/K
    and V preparation, each `--steps` times at `--heads` heads of config 3."""
    from vc_attention_b200 import stages
    from vc_attention_b200.b200_backend import group_values
    from vc_attention_b200.synthetic import make_qkv

    q, k, v = make_qkv("c3", 1, device="cuda", heads=args.heads)
    if args.case == "prep":
        for _ in range(args.steps):
            pi, _ = group_values(v, clusters=8, iterations=2)
            stages.quantize_qk(q, k, pi=pi)
            stages.prepare_v(v, pi=pi, active=True, mean_op=False)
        torch.cuda.synchronize()
        print(json.dumps({"case": "prep", "heads": args.heads, "steps": args.steps}))
        return
    q8, qs, k8, ks = stages.quantize_qk(q, k)
    v8, meta, _ = stages.prepare_v(v, active=True, mean_op=False)
    del q, k, v
    out = torch.empty((args.heads, S, D), dtype=torch.bfloat16, device="cuda")
    times = []
    for _ in range(args.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        stages.attention_fp8(q8, qs, k8, ks, v8, meta, heads=args.heads, sq=S, sk=S, dv=D, expcast=True,
                             has_mean=True, scale=D ** -0.5, out=out)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    print(json.dumps({"case": "attn", "heads": args.heads, "ms": times,
                      "tflops": [flops(h=args.heads) / (t * 1e-3) / 1e12 for t in times]}))


def run_schedule(args):
    """Config 5's denoising loop on one GPU: 50 steps with fresh seeded Q/K/V per step
    (centres drifting), every mode, one LayoutCache per mode and layer.  With 50 steps the
    smoothing window is steps 0-12 and the layout is refreshed at steps 0, 4, 8 and 12
    (core.py:182-211).  Reports the mean step time per phase (refresh / smoothed with the
    cached layout / unsmoothed) and over the whole loop, CUDA events around each call."""
    from vc_attention_b200 import Config, LayoutCache, attention
    from vc_attention_b200.synthetic import make_qkv

    heads, seq, total = args.heads, args.seq, 50
    arms = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False),
            "combined": (True, True)}
    out = {"case": "schedule", "workload": f"c5 generator: B1 H{heads} S{seq} D128 bf16, {total} steps",
           "modes": {}}
    for mode, (smooth, cast) in arms.items():
        cfg = Config(v_smooth=smooth, expcast=cast)
        cache = LayoutCache(cfg)
        phases = {"refresh": [], "smoothed_cached": [], "unsmoothed": []}
        for step in range(total):
            q, k, v = make_qkv("c5", 11, device="cuda", heads=heads, seq=seq, step=step)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            _, stats = attention(q, k, v, cfg, cache=cache, step=step, total_steps=total, request_id=mode,
                                 layer_id=0)
            e.record()
            e.synchronize()
            phase = ("refresh" if stats["layout_refreshed"] else
                     "smoothed_cached" if stats["smoothing_active"] else "unsmoothed")
            phases[phase].append(s.elapsed_time(e))
        mean = {k: (sum(v) / len(v) if v else None) for k, v in phases.items()}
        steps_ms = [t for v in phases.values() for t in v]
        out["modes"][mode] = {
            "steps": {k: len(v) for k, v in phases.items()},
            "ms": mean,
            "mean_ms": sum(steps_ms) / len(steps_ms),
            "tflops_mean": 4.0 * heads * seq * seq * 128 / (sum(steps_ms) / len(steps_ms) * 1e-3) / 1e12,
        }
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-config4", action="store_true", help="skip the configuration-4 object at N > 1")
    ap.add_argument("--case", choices=("attn", "prep", "ulysses", "schedule"),
                    help="attn / prep: small single-GPU cases for profilers; ulysses: config 4 "
                         "sequence-sharded; schedule: config 5's 50-step loop in every mode")
    ap.add_argument("--heads", type=int, default=16, help="heads of the --case run")
    ap.add_argument("--seq", type=int, default=65536, help="sequence length of --case schedule")
    args = ap.parse_args()
    if args.case in ("attn", "prep"):
        run_case(args)
        return
    if args.case == "schedule":
        run_schedule(args)
        return
    world, rank, local = dist_setup()
    try:
        if args.case == "ulysses":
            run_ulysses(args, world, rank, local)
        elif args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
