"""Seeded synthetic Q/K/V for the five benchmark configurations.

There is no public dataset behind the reference's numbers; these generators
produce inputs with the shapes and value distributions the benchmark
configurations describe (post-RoPE-like K channel offsets, clustered V).
The plain replay generator mirrors replay.py:42-49 of the reference.
Everything is drawn from one ``torch.Generator`` seeded by a single int, on
the requested device (CPU and CUDA generators give different streams).
"""
from __future__ import annotations

import torch

CONFIGS = {
    # name: (B, H, S, D, dtype, v_kind)
    "c1": (1, 2, 2048, 128, torch.float32, "mixture"),
    "c2": (1, 24, 16384, 128, torch.bfloat16, "gaussian"),
    "c3": (1, 40, 32768, 128, torch.bfloat16, "dirichlet"),
    "c4": (1, 24, 131072, 128, torch.bfloat16, "dirichlet"),
    "c5": (1, 24, 65536, 128, torch.bfloat16, "drift"),
}


def _randn(shape, g, device):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32)


def make_qkv(name, seed, *, device="cpu", heads=None, seq=None, batch=None, step=0, dtype=None):
    """Return (q, k, v) in BNSD for configuration ``name`` ("c1".."c5").

    ``heads``/``seq``/``batch`` override the configuration's size (smaller
    parity cases use the same distributions); ``step`` selects the c5
    denoising step (fresh Q/K/V per step, centres drifting by N(0, 0.05)
    per step)."""
    b, h, s, d, dt, kind = CONFIGS[name]
    b = batch or b
    h = heads or h
    s = seq or s
    dt = dtype or dt
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) + (int(step) if kind == "drift" else 0))
    q = _randn((b, h, s, d), g, device) / d ** 0.5
    k = _randn((b, h, s, d), g, device) / d ** 0.5
    k += _randn((b, h, 1, d), g, device) * 1.5
    if kind == "gaussian":
        v = _randn((b, h, s, d), g, device)
    else:
        if kind == "drift":
            gc = torch.Generator(device=device)
            gc.manual_seed(int(seed) ^ 0x5EED)
            centers = _randn((b, h, 8, d), gc, device) * 2.0
            for _ in range(int(step)):
                centers += _randn((b, h, 8, d), gc, device) * 0.05
        else:
            centers = _randn((b, h, 8, d), g, device) * 2.0
        if kind == "dirichlet":
            # K: 4 outlier channels per head with a large offset (config 3/4).
            idx = torch.randperm(d, generator=torch.Generator().manual_seed(int(seed)))[:4].to(device)
            k[..., idx] += _randn((b, h, 1, 4), g, device) * 8.0
            w = torch.empty((b, h, s, 8), device=device).exponential_(generator=g)
            w = w / w.sum(-1, keepdim=True)
            v = w @ centers + _randn((b, h, s, d), g, device) * 0.3
        else:
            ids = torch.randint(0, 8, (b, h, s), generator=g, device=device)
            v = torch.gather(centers, 2, ids[..., None].expand(b, h, s, d)) + _randn((b, h, s, d), g, device) * 0.3
    return q.to(dt), k.to(dt), v.to(dt)


def replay_synthetic(tokens, heads, dim, seed, clustered):
    """The reference replay generator (replay.py:42-49), CPU."""
    generator = torch.Generator().manual_seed(seed)
    q, k, v = [torch.randn((1, heads, tokens, dim), generator=generator) for _ in range(3)]
    if clustered:
        centers = torch.randn((1, heads, 8, dim), generator=generator) * 8
        ids = torch.randint(0, 8, (1, heads, tokens, 1), generator=generator).expand_as(v)
        v = centers.gather(-2, ids) + 0.1 * v
    return q, k, v


def flops(b, h, sq, sk, d):
    """Algorithmic FLOPs of one forward: 2*S*S*D for QK^T plus 2*S*S*D for PV."""
    return 4 * b * h * sq * sk * d
