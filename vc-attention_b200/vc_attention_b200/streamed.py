"""Attention on host-resident Q/K/V: transfers overlapped with the forward.

For callers whose activations live in (pinned) host memory, e.g. offloaded
layers of a video DiT.  Heads are independent (the reference loops heads
outermost, csrc/kernels.cu:313), so the B*H heads are cut into chunks and a
pipeline runs over them on one GPU:

    copy stream        H2D of Q/K/V, chunk after chunk, into a ring of
                       device input buffers
    compute streams    layout + quantisation + fused attention; chunks take
                       the compute streams in turn, so the small launches and
                       the last partial wave of one chunk overlap the next
    copy stream        D2H of each chunk's output once its forward is done

Events order the stages; a buffer set is refilled once the forward that read
it is done.  The ring is one allocation per input, and the streams are made
once per device and reused, so repeated calls take the same blocks from the
caching allocator.  (A ring as large as the inputs, 1 GB at configuration 3,
made repeated calls stall on fresh device allocations.)
The result is the same as ``attention`` on the whole tensors: every chunk
runs the same forward on its heads, and the layout cache keeps one entry per
chunk (key ``(layer_id, first_head)``) with the usual refresh schedule.
"""
from __future__ import annotations

import math
import threading

import torch

from .core import Config, LayoutCache, _validate


_BUFFER_SETS = 8          # chunk-sized input sets in the device ring
_COMPUTE_STREAMS = 3      # compute streams the chunks rotate over
_streams = {}
_streams_lock = threading.Lock()


def _chunks(n, size):
    return [(a, min(a + size, n)) for a in range(0, n, size)]


def _pipeline_streams(device):
    """(h2d, d2h, [compute...]) for ``device``, made once and reused, so the
    caching allocator keeps serving the same per-stream pools."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    with _streams_lock:
        if key not in _streams:
            with torch.cuda.device(key):
                _streams[key] = (torch.cuda.Stream(), torch.cuda.Stream(),
                                 [torch.cuda.Stream() for _ in range(_COMPUTE_STREAMS)])
        return _streams[key]


@torch.no_grad()
def attention_streamed(q, k, v, config=None, *, cache=None, step=0, total_steps=1, request_id=None, layer_id=0,
                       scale=None, device=None, chunk_heads=None, out=None, synchronize=True):
    """``attention`` for BNSD tensors in host memory; returns (output on the
    host, stats).  Pinned inputs (``tensor.pin_memory()``) let the copies
    overlap the compute; ``out`` may be a preallocated pinned host tensor.
    ``chunk_heads`` sets how many of the B*H heads go through the pipeline
    at a time (default: a twentieth of them, at least one).  With
    ``synchronize=False`` the call returns once the work is queued (the
    output is complete when the device's current stream reaches this point)
    and does not read the device status word.  The caller then owns that
    check: ``stats["status"]`` is the status word (device int32) and
    ``check_streamed(stats)`` reads it once the stream has reached it,
    raises what ``attention`` raises (ValueError for non-finite inputs,
    RuntimeError for an expired device wait or a failed layout check) and,
    on any raise, rolls the layout cache back to its state before the call."""
    cfg = config or Config()
    _validate(q, k, v, False, None)
    if q.device.type != "cpu":
        raise ValueError("attention_streamed takes host tensors; use attention for device tensors")
    from .b200_backend import _attention

    device = torch.device(device if device is not None else "cuda")
    b, h, sq, d = q.shape
    sk, dv = k.shape[2], v.shape[3]
    bh = b * h
    qf, kf, vf = (x.reshape(bh, x.shape[2], x.shape[3]) for x in (q, k, v))
    if out is None:
        out = torch.empty((b, h, sq, dv), dtype=q.dtype, pin_memory=True)
    elif out.shape != (b, h, sq, dv) or out.dtype != q.dtype or out.device.type != "cpu":
        raise ValueError("out must be a host tensor of the output's shape and dtype")
    of = out.view(bh, sq, dv)
    size = chunk_heads or max(1, math.ceil(bh / 20))
    parts = _chunks(bh, size)
    if cache is None:
        cache = LayoutCache(cfg)
        request_id = "one-shot" if request_id is None else request_id
    scale = d ** -0.5 if scale is None else scale

    # One status word for all chunks, read once at the end: a per-chunk read
    # would wait for the device and serialise the pipeline.  A failure rolls
    # the whole cache back, as attention does for its one entry.
    saved = (cache._request_id, dict(cache._states), {key: dict(val) for key, val in cache._states.items()})
    with torch.cuda.device(device):
        main = torch.cuda.current_stream()
        status = torch.zeros(1, dtype=torch.int32, device=device)
        h2d, d2h, compute = _pipeline_streams(device)
        n = min(size, bh)
        shapes = ((sq, d), (sk, d), (sk, dv))
        nbuf = min(len(parts), _BUFFER_SETS)
        ring = [torch.empty((nbuf * n, x, y), dtype=q.dtype, device=device) for x, y in shapes]
        for t in ring:
            for c in (h2d, *compute):
                t.record_stream(c)
        bufs = [tuple(t[i * n:(i + 1) * n].unsqueeze(0) for t in ring) for i in range(nbuf)]
        in_ready = [torch.cuda.Event() for _ in range(nbuf)]
        in_free = [torch.cuda.Event() for _ in range(nbuf)]
        stats = None
        h2d.wait_stream(main)
        for c in compute:
            c.wait_stream(main)
        for i, (a, e) in enumerate(parts):
            s, m = i % nbuf, e - a
            dq, dk, dvv = (t[:, :m] for t in bufs[s])
            with torch.cuda.stream(h2d):
                if i >= nbuf:
                    h2d.wait_event(in_free[s])          # the forward of chunk i-nbuf is done with these buffers
                dq.copy_(qf[a:e].unsqueeze(0), non_blocking=True)
                dk.copy_(kf[a:e].unsqueeze(0), non_blocking=True)
                dvv.copy_(vf[a:e].unsqueeze(0), non_blocking=True)
                in_ready[s].record()
            cs = compute[i % len(compute)]
            with torch.cuda.stream(cs):
                cs.wait_event(in_ready[s])
                res, stats = _attention(dq, dk, dvv, cfg, cache=cache, step=step, total_steps=total_steps,
                                        request_id=request_id, layer_id=(layer_id, a), scale=scale, status=status)
                in_free[s].record(cs)
                res.record_stream(d2h)
            with torch.cuda.stream(d2h):
                d2h.wait_stream(cs)
                of[a:e].copy_(res.view(m, sq, dv), non_blocking=True)
        for c in compute:
            main.wait_stream(c)
        main.wait_stream(d2h)
        main.wait_stream(h2d)

        def rollback():
            cache._request_id, states, fields = saved
            cache._states = states
            for key, val in states.items():
                val.clear()
                val.update(fields[key])

        stats = dict(stats, streamed_chunks=len(parts), status=status, rollback=rollback)
        if synchronize:
            check_streamed(stats)
    return out, stats


def check_streamed(stats):
    """Reads the status word of an ``attention_streamed`` call (waiting for
    the device's current stream) and raises what ``attention`` raises, after
    rolling the layout cache back to its state before that call."""
    from .b200_backend import raise_for_status

    try:
        raise_for_status(stats["status"])
    except (ValueError, RuntimeError):
        stats["rollback"]()
        raise
