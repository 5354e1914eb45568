"""VC-Attention public API for the B200 backend.

Mirrors czfsdg/vc-attention src/vc_attention/core.py: the same ``Config``
fields and validation (core.py:15-57), the same request-scoped
``LayoutCache`` step schedule (core.py:166-211) and the same
``attention(q, k, v, config, *, cache, step, total_steps, request_id,
layer_id, scale, causal, mask)`` signature returning ``(output, stats)``
(core.py:243-351).  The one backend here is ``"b200_fp8"``: every kernel runs
on an sm_100 GPU through libvcb.so, and there is no CPU fallback.  The
reference's own ``reference``/``cuda_fp8``/``npu_fp8`` backends stay in the
upstream package; this package adds the value that upstream's whitelist at
core.py:47 would dispatch to ``b200_backend._attention``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BACKENDS = ("b200_fp8",)


@dataclass(frozen=True)
class Config:
    expcast: bool = False
    v_smooth: bool = False
    quantize: bool = True
    q_block: int = 128
    k_quant_block: int = 256
    kv_block: int = 128
    clusters: int = 8
    iterations: int = 2
    active_fraction: float = 0.25
    refresh_interval: int = 4
    mean_dtype: str = "float16"
    backend: str = "b200_fp8"
    k_smooth: bool = True
    qk_hadamard: bool = True

    def __post_init__(self):
        # Field checks as core.py:32-52.
        for name in ("k_smooth", "qk_hadamard"):
            if not isinstance(getattr(self, name), bool):
                raise ValueError(f"{name} must be a bool")
        for name in ("q_block", "k_quant_block", "kv_block", "clusters", "iterations", "refresh_interval"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, int) or value < 1:
                raise ValueError(f"{name} must be a positive integer")
        if not math.isfinite(self.active_fraction) or not 0 <= self.active_fraction <= 1:
            raise ValueError("active_fraction must be in [0, 1]")
        if self.mean_dtype not in ("float16", "bfloat16", "float32"):
            raise ValueError("Unsupported mean_dtype")
        if self.backend not in BACKENDS:
            raise ValueError("backend must be b200_fp8 (reference, cuda_fp8 and npu_fp8 live in upstream vc_attention)")
        if not self.quantize:
            raise ValueError("b200_fp8 requires quantize=True")
        if self.k_quant_block % self.kv_block:
            raise ValueError("b200_fp8 requires kv_block to divide k_quant_block")
        # Geometry of the sm_100a kernels (tiles of 128 query rows x 128 keys).
        if self.kv_block != 128:
            raise ValueError("b200_fp8 requires kv_block == 128")
        if self.q_block < 32 or self.q_block > 256 or self.q_block % 32:
            raise ValueError("b200_fp8 q_block must be a multiple of 32 in [32, 256]")
        if self.k_quant_block > 4096:
            raise ValueError("b200_fp8 k_quant_block must be <= 4096")
        if self.clusters > 32:
            raise ValueError("b200_fp8 supports at most 32 clusters")


def group_values(v, *, clusters, iterations, centers=None):
    """Lloyd clustering with a stable permutation (core.py:138-163), on the GPU.
    Returns (pi int32 [B, H, S], centers float32 [B, H, count, D])."""
    from .b200_backend import group_values as native

    return native(v, clusters=clusters, iterations=iterations, centers=centers)


def _mark_use(t):
    """Tell the caching allocator that ``t`` is used on the current stream, so
    that a cached layout made on one stream and read on another is not handed
    out again before that stream is done with it."""
    if t is not None and t.is_cuda:
        t.record_stream(torch.cuda.current_stream(t.device))


class LayoutCache:
    """Request-scoped layout state (core.py:166-211). Callers must supply a real request identifier."""

    def __init__(self, config):
        self.config = config
        self._request_id = None
        self._states = {}

    @property
    def entries(self):
        return len(self._states)

    def reset(self):
        self._request_id = None
        self._states.clear()

    def _snapshot(self, layer_id):
        state = self._states.get(layer_id)
        return (self._request_id, dict(self._states), state, None if state is None else dict(state))

    def _restore(self, snap, layer_id):
        """Undo a layout() call whose forward failed (the same state objects come back)."""
        request_id, states, state, fields = snap
        self._request_id = request_id
        self._states = states
        if state is not None:
            state.clear()
            state.update(fields)
            self._states[layer_id] = state

    def layout(self, v, *, step, total_steps, request_id, layer_id):
        if request_id is None:
            raise ValueError("A persistent layout cache requires request_id")
        if total_steps < 1 or not 0 <= step < total_steps:
            raise ValueError("Invalid denoising step/total_steps")
        if request_id != self._request_id:
            self.reset()
            self._request_id = request_id
        signature = (tuple(v.shape), str(v.device), v.dtype, total_steps)
        state = self._states.get(layer_id)
        if state is not None and (state["signature"] != signature or step < state["step"]):
            state = None
            self._states.pop(layer_id, None)
        active = self.config.v_smooth and step < math.ceil(total_steps * self.config.active_fraction)
        refresh = active and (state is None or step - state["refresh_step"] >= self.config.refresh_interval)
        if refresh:
            if state is not None:
                _mark_use(state["centers"])
            pi, centers = group_values(
                v,
                clusters=self.config.clusters,
                iterations=self.config.iterations,
                centers=None if state is None else state["centers"],
            )
            state = {"signature": signature, "pi": pi, "centers": centers, "refresh_step": step, "step": step}
            self._states[layer_id] = state
        if state is not None:
            state["step"] = step
            _mark_use(state["pi"])
        return (None if state is None else state["pi"]), active, refresh

    def peek(self, v, *, step, total_steps, request_id, layer_id):
        """What ``layout`` would decide for this call, without changing the
        cache or clustering anything: ``(pi, active, refresh)``, where ``pi`` is
        the cached permutation when the call would reuse it (active and no
        refresh) and None otherwise.  ``v`` is V or any tensor with V's shape,
        device and dtype.

        The reference gathers K and V through ``pi`` on every call
        (cuda_backend.py:49-51).  A producer that keeps K and V in layout order
        (for example by writing the QKV projection's rows through ``pi``) asks
        here before it writes them, and passes ``kv_order="layout"`` to
        ``attention`` when ``pi`` is not None; the forward then skips the
        gather."""
        if request_id is None:
            raise ValueError("A persistent layout cache requires request_id")
        if total_steps < 1 or not 0 <= step < total_steps:
            raise ValueError("Invalid denoising step/total_steps")
        state = self._states.get(layer_id) if request_id == self._request_id else None
        signature = (tuple(v.shape), str(v.device), v.dtype, total_steps)
        if state is not None and (state["signature"] != signature or step < state["step"]):
            state = None
        active = self.config.v_smooth and step < math.ceil(total_steps * self.config.active_fraction)
        refresh = active and (state is None or step - state["refresh_step"] >= self.config.refresh_interval)
        reuse = active and not refresh and state is not None
        return (state["pi"] if reuse else None), active, refresh


def to_layout_order(x, pi):
    """Rows of ``x`` [B, H, S, D] in layout order: row r of the result is row
    ``pi[b, h, r]`` of ``x`` (the gather of cuda_backend.py:49-51).  For
    producers without a fused epilogue, and for tests."""
    return x.gather(-2, pi.long().unsqueeze(-1).expand_as(x))


def _validate(q, k, v, causal, mask):
    """core.py:214-232.  Finiteness is checked on the device by the kernels
    that read Q, K and V; a non-finite input raises the same ValueError after
    the launch and leaves any layout cache as it was."""
    if causal:
        raise ValueError("This experiment does not support causal attention")
    if mask is not None:
        raise ValueError("This experiment does not support a mask/bias")
    if any(x.ndim != 4 for x in (q, k, v)):
        raise ValueError("Expected BNSD tensors")
    if q.shape[:2] != k.shape[:2] or k.shape[:2] != v.shape[:2]:
        raise ValueError("Batch and heads must match; GQA is not implemented")
    if k.shape[-2] != v.shape[-2] or q.shape[-1] != k.shape[-1]:
        raise ValueError("Incompatible Q/K/V shape")
    if any(0 in x.shape for x in (q, k, v)):
        raise ValueError("Empty Q/K/V are not supported")
    if any(x.device != q.device or x.dtype != q.dtype for x in (k, v)):
        raise ValueError("Q/K/V must have the same device and dtype")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("Inputs must be FP16/BF16/FP32 before quantization")


@torch.no_grad()
def attention(
    q,
    k,
    v,
    config=None,
    *,
    cache=None,
    step=0,
    total_steps=1,
    request_id=None,
    layer_id=0,
    scale=None,
    causal=False,
    mask=None,
    status=None,
    kv_order="natural",
):
    """Return (output, counters) as core.attention does (core.py:243-351).

    ``status`` (an addition to the reference's signature, default None) is
    for callers that read the device status once per step instead of once
    per call.  By default the call waits for the current stream, reads the
    status word the kernels write, and raises ValueError for non-finite
    Q/K/V (as the reference's isfinite check does) or RuntimeError for an
    expired device wait.  Given a caller-owned int32 CUDA tensor of one
    element, the call only queues the work; the word is cleared and then
    receives this call's flags on the device (use one word per call whose
    flags must be kept apart); the caller later calls
    ``b200_backend.raise_for_status(status)``
    and, if it raises, ``counters["rollback"]()`` to put the layout cache
    back as it was before this call.

    ``kv_order`` (also an addition, default "natural") set to "layout" says
    that K and V already come in the cached layout's order: row r is token
    ``pi[r]`` of the call's sequence, with ``pi`` as ``cache.peek`` returns it
    for this step.  The forward then reads them as they are instead of
    gathering them.  It is valid only on a step that reuses a cached layout;
    on any other step the call raises ValueError and leaves the cache as it
    was.  The output rows follow Q, whose order never changes."""
    cfg = config or Config()
    _validate(q, k, v, causal, mask)
    if kv_order not in ("natural", "layout"):
        raise ValueError('kv_order must be "natural" or "layout"')
    from .b200_backend import _attention

    return _attention(q, k, v, cfg, cache=cache, step=step, total_steps=total_steps,
                      request_id=request_id, layer_id=layer_id,
                      scale=q.shape[-1] ** -0.5 if scale is None else scale, status=status,
                      kv_order=kv_order)
