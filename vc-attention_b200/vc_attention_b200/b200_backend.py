"""B200 (sm_100a) entry point of VC-Attention.

Mirrors czfsdg/vc-attention src/vc_attention/cuda_backend.py: the extension
loader with its version gate (cuda_backend.py:8-19), ``group_values``
(:22-23), ``_attention`` (:26-66) and ``preflight`` (:69-88), plus the other
exports of the reference's native module (bindings.cpp:231-248):
``expcast_codes`` and ``preprocess_qk``.  Every call goes through the C ABI
of libvcb.so; PyTorch supplies device memory and the current stream.
Permutations are applied inside the kernels, so K and V are never gathered
or copied to FP32 here (the reference did both, cuda_backend.py:47-51).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _abi

_DTYPES = {torch.float32: _abi.VCB_F32, torch.float16: _abi.VCB_F16, torch.bfloat16: _abi.VCB_BF16}
_MEAN_TYPES = {"float32": 0, "float16": 1, "bfloat16": 2}     # cuda_backend.py:52


def _extension():
    """Load libvcb.so or raise RuntimeError; no fallback (cuda_backend.py:8-19)."""
    try:
        return _abi.load()
    except OSError as exc:
        raise RuntimeError("libvcb.so failed to load. No reference fallback was used. "
                           "Original error: " + str(exc)) from exc


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_b200(t, what="b200_fp8"):
    if t.device.type != "cuda":
        raise ValueError(f"{what} requires CUDA tensors; no CPU fallback")
    if torch.cuda.get_device_capability(t.device) != (10, 0):
        raise ValueError(f"{what} requires a B200-class GPU (compute capability 10.0)")


def _flat(x):
    b, h, s, d = x.shape
    return x.contiguous().view(b * h, s, d)


def expcast_codes(x):
    """ExpCast bytes of FP32 inputs (bindings.cpp:219-227)."""
    if x.dtype != torch.float32:
        raise ValueError("ExpCast expects FP32 input")
    _require_b200(x, "expcast_codes")
    lib = _extension()
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _abi.check(lib, lib.vcb_expcast_codes(x.data_ptr(), out.data_ptr(), x.numel(), _stream(x.device)))
    return out


def preprocess_qk(q, k, k_smooth, hadamard):
    """Post-RoPE K centering and normalised Q/K Hadamard in FP32 (bindings.cpp:68-98)."""
    _require_b200(q, "preprocess_qk")
    if q.dim() != 4 or k.dim() != 4 or q.shape[:2] != k.shape[:2] or q.shape[3] != k.shape[3]:
        raise ValueError("Q/K shapes must match as [B, H, N, D]")
    if k.dtype != q.dtype or q.dtype not in _DTYPES:
        raise ValueError("Q/K must share an FP32/FP16/BF16 dtype")
    d = q.shape[3]
    if d > 128:
        raise ValueError("Q/K preprocessing supports head dimensions <= 128")
    width = 1 << (d - 1).bit_length() if hadamard else d
    lib = _extension()
    b, h = q.shape[:2]
    qf, kf = _flat(q), _flat(k)
    q_out = torch.empty((b, h, q.shape[2], width), dtype=torch.float32, device=q.device)
    k_out = torch.empty((b, h, k.shape[2], width), dtype=torch.float32, device=q.device)
    ws = torch.empty(lib.vcb_qk_workspace(b * h, k.shape[2]), dtype=torch.uint8, device=q.device)
    a = _abi.QKArgs(q=qf.data_ptr(), k=kf.data_ptr(), dtype=_DTYPES[q.dtype], heads=b * h, sq=q.shape[2],
                    sk=k.shape[2], d=d, pi=None, k_smooth=int(bool(k_smooth)), hadamard=int(bool(hadamard)),
                    q_out=q_out.data_ptr(), k_out=k_out.data_ptr(), workspace=ws.data_ptr(),
                    workspace_bytes=ws.numel())
    with torch.cuda.device(q.device):
        _abi.check(lib, lib.vcb_preprocess_qk(ctypes.byref(a), _stream(q.device)))
    return [q_out, k_out]


def group_values(v, *, clusters, iterations, centers=None):
    """Native Lloyd clustering with a stable permutation (bindings.cpp:182-217).
    Returns (pi int32 [B, H, S], centers float32 [B, H, count, D])."""
    _require_b200(v, "group_values")
    if v.dim() != 4 or v.numel() == 0:
        raise ValueError("group_values expects nonempty [B,H,N,D]")
    if v.dtype not in _DTYPES:
        raise ValueError("V must be FP32/FP16/BF16")
    if clusters < 1 or iterations < 1:
        raise ValueError("clusters and iterations must be positive")
    b, h, s, d = v.shape
    count = min(clusters, s)
    if centers is not None:
        if (centers.device != v.device or centers.dtype != torch.float32 or
                tuple(centers.shape) != (b, h, count, d)):
            raise ValueError("Invalid cached centers")
        centers = centers.contiguous()
    lib = _extension()
    vf = _flat(v)
    pi = torch.empty((b, h, s), dtype=torch.int32, device=v.device)
    out_centers = torch.empty((b, h, count, d), dtype=torch.float32, device=v.device)
    ws = torch.empty(lib.vcb_group_workspace(b * h, s, d, clusters), dtype=torch.uint8, device=v.device)
    a = _abi.GroupArgs(v=vf.data_ptr(), dtype=_DTYPES[v.dtype], heads=b * h, s=s, d=d, clusters=clusters,
                       iterations=iterations, centers_in=None if centers is None else centers.data_ptr(),
                       centers_out=out_centers.data_ptr(), pi=pi.data_ptr(), workspace=ws.data_ptr(),
                       workspace_bytes=ws.numel())
    with torch.cuda.device(v.device):
        _abi.check(lib, lib.vcb_group_values(ctypes.byref(a), _stream(v.device)))
    return pi, out_centers


def forward_args(q, k, v, cfg, pi, active, scale, out):
    """Fill the vcb_forward argument struct for [B, H, S, D] tensors."""
    b, h, sq, d = q.shape
    return _abi.ForwardArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), dtype=_DTYPES[q.dtype], heads=b * h, sq=sq,
        sk=k.shape[2], d=d, dv=v.shape[3], pi=None if pi is None else pi.data_ptr(), q_block=cfg.q_block,
        k_quant_block=cfg.k_quant_block, kv_block=cfg.kv_block, smooth=int(bool(active)),
        expcast=int(bool(cfg.expcast)), mean_type=_MEAN_TYPES[cfg.mean_dtype], scale=float(scale),
        k_smooth=int(cfg.k_smooth), hadamard=int(cfg.qk_hadamard), out=out.data_ptr())


def forward(q, k, v, cfg, *, pi, active, scale, out=None, workspace=None, status=None, check_status=True):
    """One fused forward through vcb_forward on the current stream.
    q/k/v: contiguous [B, H, S, D]; pi: int32 [B, H, Sk] or None."""
    lib = _extension()
    if out is None:
        out = torch.empty((*q.shape[:3], v.shape[3]), dtype=q.dtype, device=q.device)
    a = forward_args(q, k, v, cfg, pi, active, scale, out)
    need = lib.vcb_forward_workspace(ctypes.byref(a))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=q.device)
    a.workspace = workspace.data_ptr()
    a.workspace_bytes = workspace.numel()
    a.status = status.data_ptr()
    with torch.cuda.device(q.device):
        _abi.check(lib, lib.vcb_forward(ctypes.byref(a), _stream(q.device)))
        if check_status:
            raise_for_status(status)
    return out


def raise_for_status(status):
    """Reads the device status word (waits for the current stream) and raises
    what the reference raises: ValueError for non-finite inputs, RuntimeError
    for an expired device wait or a failed layout check."""
    lib = _extension()
    flags = ctypes.c_int32(0)
    with torch.cuda.device(status.device):
        _abi.check(lib, lib.vcb_read_status(status.data_ptr(), _stream(status.device), ctypes.byref(flags)))
    if flags.value & _abi.FLAG_NONFINITE:
        raise ValueError("Q/K/V must be finite")
    if flags.value & _abi.FLAG_TIMEOUT:
        raise RuntimeError("b200_fp8 attention kernel: a bounded device wait expired")
    if flags.value & _abi.FLAG_INTERNAL:
        raise RuntimeError("b200_fp8 attention kernel: device layout check failed")


@torch.no_grad()
def _attention(q, k, v, cfg, *, cache, step, total_steps, request_id, layer_id, scale, status=None,
               kv_order="natural"):
    """cuda_backend._attention (cuda_backend.py:26-66) for sm_100a.  With a
    caller-owned ``status`` word the call does not wait for the device; the
    caller reads the word later (raise_for_status) and owns the cache rollback.
    With ``kv_order="layout"`` K and V are already in the cached layout's
    order and are read without the gather of cuda_backend.py:49-51."""
    from .core import LayoutCache

    _require_b200(q)
    if q.shape[-1] > 128 or v.shape[-1] > 128:
        raise ValueError("b200_fp8 supports Q/K/V head dimensions <= 128")
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("scale must be positive and finite")
    _extension()
    if cache is None:
        cache = LayoutCache(cfg)
        request_id = "one-shot" if request_id is None else request_id
    elif cache.config != cfg:
        raise ValueError("cache.config must match config")
    if status is not None and (status.device != q.device or status.dtype != torch.int32 or status.numel() != 1):
        raise ValueError("status must be a one-element int32 tensor on the inputs' device")
    if kv_order == "layout":
        cached, _, _ = cache.peek(v, step=step, total_steps=total_steps, request_id=request_id, layer_id=layer_id)
        if cached is None:
            raise ValueError('kv_order="layout" needs a step that reuses a cached layout '
                             "(LayoutCache.peek returns its pi)")
    snapshot = cache._snapshot(layer_id)
    with torch.cuda.device(q.device):
        pi, active, refreshed = cache.layout(v, step=step, total_steps=total_steps, request_id=request_id,
                                             layer_id=layer_id)
        qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
        try:
            output = forward(qc, kc, vc, cfg, pi=pi if kv_order == "natural" else None, active=active,
                             scale=scale, status=status, check_status=status is None)
        except (ValueError, RuntimeError):
            cache._restore(snapshot, layer_id)
            raise
    extra = {} if status is None else {"rollback": lambda: cache._restore(snapshot, layer_id)}
    return output, {**extra,
        "backend": "b200_fp8",
        "smoothing_active": active,
        "layout_refreshed": refreshed,
        "expcast": cfg.expcast,
        "k_smooth": cfg.k_smooth,
        "qk_hadamard": cfg.qk_hadamard,
        "numerical_contract_version": 2,
        "tiles": math.ceil(q.shape[-2] / cfg.q_block) * math.ceil(k.shape[-2] / cfg.kv_block),
        "native_fused_attention": True,
        "native_fp8_matmul": True,
    }


def build_info():
    import json

    return json.loads(_extension().vcb_build_info().decode())


def wait_selftest(complete=False, device="cuda:0"):
    """Runs the self-test of the attention kernel's bounded waits
    (``vcb_wait_selftest``) and returns its report and the device status word.
    With ``complete=False`` the awaited phase never completes: the kernel gives
    up after its 2 s limit, drains, frees tensor memory and sets the timeout
    flag; ``raise_for_status(result["status"])`` then raises RuntimeError."""
    device = torch.device(device)
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise RuntimeError("wait_selftest requires a B200-class GPU (compute capability 10.0)")
    lib = _extension()
    gen = torch.Generator().manual_seed(7)
    src = torch.randint(-2**31, 2**31 - 1, (256,), dtype=torch.int32, generator=gen).to(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    report = torch.empty(4, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        _abi.check(lib, lib.vcb_wait_selftest(int(bool(complete)), src.data_ptr(), status.data_ptr(),
                                              report.data_ptr(), _stream(device)))
    gave_up, completed, copy_intact, elapsed_ms = report.tolist()
    return {"gave_up": gave_up, "completed": completed, "copy_intact": bool(copy_intact),
            "elapsed_ms": elapsed_ms, "status": status}


def preflight(device="cuda:0"):
    """Fail loudly unless ExpCast bytes and the fused FP8 path work (cuda_backend.py:69-88)."""
    from .core import Config, attention

    device = torch.device(device)
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise RuntimeError("Preflight requires a B200-class GPU (compute capability 10.0)")
    # Known answers of the reference's ExpCast test (test_core.py:19-22).
    x = torch.tensor([0, -1, -1.6, -8, -14, -100, -float("inf")], device=device) / math.log2(math.e)
    got = expcast_codes(x).tolist()
    if got != [120, 112, 107, 56, 8, 0, 0]:
        raise RuntimeError(f"ExpCast preflight failed: {got}")
    # Exactly representable FP8 data gives an independent oracle (cuda_backend.py:79-85).
    q = torch.zeros(1, 1, 19, 16, device=device)
    k = torch.zeros(1, 1, 35, 16, device=device)
    v = torch.full((1, 1, 35, 16), 3.0, device=device)
    for cast in (False, True):
        actual, _ = attention(q, k, v, Config(expcast=cast))
        torch.testing.assert_close(actual, torch.full_like(actual, 3), rtol=2e-5, atol=2e-5)
    torch.cuda.synchronize(device)
    return {"device": str(device), "name": torch.cuda.get_device_name(device), "preflight": "passed",
            **build_info()}


if __name__ == "__main__":
    import argparse
    import json

    parser = argparse.ArgumentParser()
    parser.add_argument("--device", default="cuda:0")
    args = parser.parse_args()
    print(json.dumps(preflight(args.device), indent=2))
