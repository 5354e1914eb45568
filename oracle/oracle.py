"""CPU restatement of the VC-Attention reference backend.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against, and the CPU baseline that bench.py times beside it.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
may import it; the product package never does.

It restates czfsdg/vc-attention src/vc_attention/core.py (the ``reference``
backend) with numpy for the streaming attention and the C library in
oracle/vc_oracle.c for every byte-level step (E4M3 encoding, ExpCast, the
Hadamard butterfly, block scales, V tiles, Lloyd clustering, stable sort).
The fixed reduction orders that make those steps bit-exact against the GPU
are documented in vc_oracle.c.  Arrays are [heads, tokens, channels] with
batch and heads flattened, float32.
"""
from __future__ import annotations

import ctypes
import math
import os
import pathlib
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libvc_oracle.so"
MEAN_DTYPES = {"float32": 0, "float16": 1, "bfloat16": 2}

_lib = None
_lock = threading.Lock()

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build():
    """Compile oracle/vc_oracle.c into oracle/_build (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                build()
            L = ctypes.CDLL(str(LIB_PATH))
            i64, i32 = ctypes.c_int64, ctypes.c_int
            L.vco_e4m3_encode_n.argtypes = [_f32p, _u8p, i64]
            L.vco_e4m3_decode_n.argtypes = [_u8p, _f32p, i64]
            L.vco_expcast_fma.argtypes = [_f32p, _u8p, i64]
            L.vco_expcast_fp64.argtypes = [_f32p, _u8p, i64]
            L.vco_fused_codes.argtypes = [_f32p, _f32p, _f32p, i64, _u8p]
            L.vco_hadamard_rows.argtypes = [_f32p, i64, i32, _f32p]
            L.vco_k_mean.argtypes = [_f32p, i64, i64, i32, _f32p]
            L.vco_quant_blocks.argtypes = [_f32p, i64, i64, i32, i32, i64, _u8p, _f32p]
            L.vco_linspace_indices.argtypes = [i64, i32, _i64p]
            L.vco_group_values.argtypes = [_f32p, i64, i64, i32, i32, i32, ctypes.c_void_p,
                                           _f32p, _i32p, _u8p]
            L.vco_group_values.restype = i32
            L.vco_value_tiles.argtypes = [_f32p, i64, i64, i32, ctypes.c_void_p, i32, i32, i32,
                                          _u8p, _f32p, _f32p]
            L.vco_constants.argtypes = [i32]
            L.vco_constants.restype = i32
            _lib = L
    return _lib


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


# ---------------------------------------------------------------- byte level
def e4m3_encode(x):
    """torch float8_e4m3fn cast of clamped values (core.py:113, :121)."""
    x = _f32(x)
    out = np.empty(x.shape, np.uint8)
    lib().vco_e4m3_encode_n(x.reshape(-1), out.reshape(-1), x.size)
    return out


def e4m3_decode(b):
    """E4M3 byte -> float32 (csrc/kernels.cu:54-59, signed)."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.empty(b.shape, np.float32)
    lib().vco_e4m3_decode_n(b.reshape(-1), out.reshape(-1), b.size)
    return out


def expcast_codes(x, *, fp64=True):
    """ExpCast bytes (core.py:60-68).  fp64=True is the reference's FP64
    widened evaluation; fp64=False is the single-rounding FP32 FMA of the
    contract (csrc/kernels.cu:61-65)."""
    x = _f32(x)
    out = np.empty(x.shape, np.uint8)
    fn = lib().vco_expcast_fp64 if fp64 else lib().vco_expcast_fma
    fn(x.reshape(-1), out.reshape(-1), x.size)
    return out


def fused_codes(s, a, b):
    """The fused attention kernel's encode (vc_oracle.c vco_fused_codes):
    RNE(fmaf(s, a, b) * 2^24), negatives to 0; a, b broadcast against s."""
    s = _f32(s)
    a, b = (_f32(np.broadcast_to(x, s.shape)) for x in (a, b))
    out = np.empty(s.shape, np.uint8)
    lib().vco_fused_codes(s.reshape(-1), a.reshape(-1), b.reshape(-1), s.size, out.reshape(-1))
    return out


def hadamard(x):
    """Normalised Sylvester transform with zero padding (core.py:71-85)."""
    x = _f32(x)
    d = x.shape[-1]
    width = 1 << (d - 1).bit_length()
    rows = x.size // d
    out = np.empty(x.shape[:-1] + (width,), np.float32)
    lib().vco_hadamard_rows(x.reshape(-1), rows, d, out.reshape(-1))
    return out


def k_mean(k):
    """Per-head channel mean over tokens in the fixed order of vc_oracle.c."""
    k = _f32(k)
    h, s, d = k.shape
    out = np.empty((h, d), np.float32)
    lib().vco_k_mean(k.reshape(-1), h, s, d, out.reshape(-1))
    return out


def preprocess_qk(q, k, *, k_smooth, qk_hadamard, pi=None):
    """core.py:88-99: demean K over tokens, then rotate Q and K.  With a
    permutation pi, K rows are gathered (core.py:289) before the demean; the
    mean itself is summed in original token order (the fixed order of
    vc_oracle.c), which is the same set of tokens."""
    q, k = _f32(q), _f32(k)
    mean = k_mean(k)[:, None, :] if k_smooth else None
    if pi is not None:
        k = np.take_along_axis(k, np.asarray(pi, dtype=np.int64)[:, :, None], axis=1)
    if k_smooth:
        k = k - mean
    if qk_hadamard:
        q, k = hadamard(q), hadamard(k)
    return q, k


def padded_rows(n, block):
    """Rows of a payload buffer: whole quantisation blocks and whole 128-row tiles."""
    unit = block * 128 // math.gcd(block, 128)
    return -(-n // unit) * unit


def quantize_blocks(x, block):
    """core.py:118-135 as bytes: payload [heads, S_pad, 128], scales [heads, nblk]."""
    x = _f32(x)
    h, s, w = x.shape
    assert w <= 128
    s_pad = padded_rows(s, block)
    payload = np.empty((h, s_pad, 128), np.uint8)
    scales = np.empty((h, -(-s // block)), np.float32)
    lib().vco_quant_blocks(x.reshape(-1), h, s, w, block, s_pad, payload.reshape(-1), scales.reshape(-1))
    return payload, scales


def dequantize(payload, scales, block, s, w):
    """payload.float() * scale, as the reference multiplies back (core.py:134)."""
    vals = e4m3_decode(payload[:, :s, :w])
    rows = np.arange(s) // block
    return vals * scales[:, rows][:, :, None]


def linspace_indices(s, count):
    out = np.empty(count, np.int64)
    lib().vco_linspace_indices(s, count, out)
    return out


def group_values(v, *, clusters, iterations, centers=None):
    """Lloyd clustering + stable permutation (core.py:138-163).
    Returns (pi int32 [heads, S], centers float32 [heads, count, D], labels)."""
    v = _f32(v)
    h, s, d = v.shape
    count = min(clusters, s)
    cin = None
    if centers is not None:
        cin = _f32(centers)
        assert cin.shape == (h, count, d)
    cout = np.empty((h, count, d), np.float32)
    pi = np.empty((h, s), np.int32)
    labels = np.empty((h, s), np.uint8)
    lib().vco_group_values(v.reshape(-1), h, s, d, clusters, iterations,
                           None if cin is None else cin.ctypes.data, cout.reshape(-1),
                           pi.reshape(-1), labels.reshape(-1))
    return pi, cout, labels


def value_tiles(v, pi, *, active, mean_dtype, kv_block):
    """core.py:102-115 per kv_block tile, after the permutation.
    Returns payload [heads, T, 128, kv_block] u8, vscale and mu [heads, T, 128]."""
    v = _f32(v)
    h, s, dv = v.shape
    t = -(-s // kv_block)
    payload = np.empty((h, t, 128, kv_block), np.uint8)
    vscale = np.empty((h, t, 128), np.float32)
    mu = np.empty((h, t, 128), np.float32)
    pik = None
    if pi is not None:
        pik = np.ascontiguousarray(pi, dtype=np.int32)
    lib().vco_value_tiles(v.reshape(-1), h, s, dv, None if pik is None else pik.ctypes.data,
                          int(bool(active)), MEAN_DTYPES[mean_dtype], kv_block,
                          payload.reshape(-1), vscale.reshape(-1), mu.reshape(-1))
    return payload, vscale, mu


# ------------------------------------------------------------------ attention
class Prepared:
    """Everything the streaming loop of core.py:307-340 consumes."""

    def __init__(self, q, k, v, *, pi, active, q_block, k_quant_block, kv_block, mean_dtype,
                 k_smooth, qk_hadamard):
        q, k, v = _f32(q), _f32(k), _f32(v)
        self.sq, self.sk, self.dv = q.shape[1], k.shape[1], v.shape[2]
        qf, kf = preprocess_qk(q, k, k_smooth=k_smooth, qk_hadamard=qk_hadamard, pi=pi)
        self.w = qf.shape[2]
        self.q8, self.qs = quantize_blocks(qf, q_block)
        self.k8, self.ks = quantize_blocks(kf, k_quant_block)
        self.qd = dequantize(self.q8, self.qs, q_block, self.sq, self.w)
        self.kd = dequantize(self.k8, self.ks, k_quant_block, self.sk, self.w)
        self.v8, self.vscale, self.mu = value_tiles(v, pi, active=active, mean_dtype=mean_dtype,
                                                    kv_block=kv_block)
        self.kv_block = kv_block


def stream(prep: Prepared, rows, *, expcast, scale, head=None):
    """Online softmax over KV tiles for the given query rows (core.py:307-340).
    rows: slice of query rows; head: None for all heads or one head index."""
    hs = slice(None) if head is None else slice(head, head + 1)
    qd = prep.qd[hs, rows]
    nh, nq = qd.shape[0], qd.shape[1]
    dv, bk = prep.dv, prep.kv_block
    rowmax = np.full((nh, nq, 1), -np.inf, np.float32)
    denom = np.zeros((nh, nq, 1), np.float32)
    acc = np.zeros((nh, nq, dv), np.float32)
    sc = np.float32(scale)
    for j, ks in enumerate(range(0, prep.sk, bk)):
        n = min(bk, prep.sk - ks)
        kt = prep.kd[hs, ks:ks + n]
        scores = np.matmul(qd, kt.transpose(0, 2, 1)) * sc
        newmax = np.maximum(rowmax, scores.max(-1, keepdims=True))
        with np.errstate(invalid="ignore"):
            alpha = np.exp(rowmax - newmax)
        shifted = scores - newmax
        if expcast:
            p8 = e4m3_decode(expcast_codes(shifted))
            probability = p8 / np.float32(256.0)
        else:
            probability = np.exp(shifted)
            p8 = e4m3_decode(e4m3_encode(probability * np.float32(256.0)))
        rowmass = probability.sum(-1, keepdims=True, dtype=np.float32)
        resid = e4m3_decode(prep.v8[hs, j, :dv, :n]).transpose(0, 2, 1)
        mu = prep.mu[hs, j, None, :dv]
        vs = prep.vscale[hs, j, None, :dv]
        contribution = (np.matmul(p8, resid) / np.float32(256.0) + rowmass * mu) * vs
        acc = alpha * acc + contribution
        denom = alpha * denom + rowmass
        rowmax = newmax
    return acc / denom


def attention(q, k, v, *, expcast, active, pi=None, q_block=128, k_quant_block=256,
              kv_block=128, mean_dtype="float16", scale=None, k_smooth=True, qk_hadamard=True,
              threads=1, row_chunk=512):
    """Full quantised reference forward for [heads, S, D] float32 inputs.
    Returns float32 [heads, Sq, Dv] (the reference casts to the input dtype
    afterwards, core.py:341)."""
    if scale is None:
        scale = q.shape[-1] ** -0.5
    prep = Prepared(q, k, v, pi=pi, active=active, q_block=q_block, k_quant_block=k_quant_block,
                    kv_block=kv_block, mean_dtype=mean_dtype, k_smooth=k_smooth,
                    qk_hadamard=qk_hadamard)
    if threads <= 1:
        return stream(prep, slice(None), expcast=expcast, scale=scale)
    out = np.empty((q.shape[0], prep.sq, prep.dv), np.float32)
    jobs = [(h, r) for h in range(q.shape[0]) for r in range(0, prep.sq, row_chunk)]

    def run(job):
        h, r = job
        out[h:h + 1, r:r + row_chunk] = stream(prep, slice(r, r + row_chunk), expcast=expcast,
                                               scale=scale, head=h)

    with ThreadPoolExecutor(max_workers=threads) as pool:
        list(pool.map(run, jobs))
    return out


def metrics(actual, reference):
    """rmse / relative_rmse / max_abs / cosine exactly as replay.py:20-32."""
    x = np.asarray(actual, np.float64).reshape(-1)
    ref = np.asarray(reference, np.float64).reshape(-1)
    if not np.isfinite(x).all():
        raise ValueError("Nonfinite attention output")
    delta = x - ref
    mse = float(np.mean(delta * delta))
    energy = float(np.mean(ref * ref))
    denom = max(np.linalg.norm(x) * np.linalg.norm(ref), 1e-8)
    return {
        "rmse": math.sqrt(mse),
        "relative_rmse": math.sqrt(mse / max(energy, 1e-30)),
        "max_abs": float(np.abs(delta).max()),
        "cosine": float(np.dot(x, ref) / denom),
    }


def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
