"""Stage-level calls of libvcb.so: the fused forward split into its three
kernels, each through its own C-ABI entry point.  Used to check every
intermediate byte (E4M3 payloads, scales, V tiles) and to time the kernels
one by one.  Inputs are [B, H, S, D] CUDA tensors; outputs use the flat
[B*H, ...] layouts of include/vcb.h."""
from __future__ import annotations

import ctypes

import torch

from . import _abi
from .b200_backend import _DTYPES, _MEAN_TYPES, _extension, _flat, _stream


def _i(t):
    return None if t is None else t.data_ptr()


def quantize_qk(q, k, *, pi=None, q_block=128, k_quant_block=256, k_smooth=True, hadamard=True, status=None):
    """vcb_quantize_qk: returns (q8 [BH, Sq_pad, 128] u8, q_scale, k8, k_scale)."""
    lib = _extension()
    b, h, sq, d = q.shape
    sk = k.shape[2]
    heads = b * h
    dev = q.device
    q8 = torch.empty((heads, lib.vcb_padded_rows(sq, q_block), 128), dtype=torch.uint8, device=dev)
    k8 = torch.empty((heads, lib.vcb_padded_rows(sk, k_quant_block), 128), dtype=torch.uint8, device=dev)
    qs = torch.empty((heads, -(-sq // q_block)), dtype=torch.float32, device=dev)
    ks = torch.empty((heads, -(-sk // k_quant_block)), dtype=torch.float32, device=dev)
    ws = torch.empty(lib.vcb_qk_workspace(heads, sk), dtype=torch.uint8, device=dev)
    qf, kf = _flat(q), _flat(k)
    a = _abi.QKArgs(q=qf.data_ptr(), k=kf.data_ptr(), dtype=_DTYPES[q.dtype], heads=heads, sq=sq, sk=sk, d=d,
                    pi=_i(pi), k_smooth=int(k_smooth), hadamard=int(hadamard), q_block=q_block,
                    k_quant_block=k_quant_block, q8=q8.data_ptr(), k8=k8.data_ptr(), q_scale=qs.data_ptr(),
                    k_scale=ks.data_ptr(), status=_i(status), workspace=ws.data_ptr(), workspace_bytes=ws.numel())
    with torch.cuda.device(dev):
        _abi.check(lib, lib.vcb_quantize_qk(ctypes.byref(a), _stream(dev)))
    return q8, qs, k8, ks


def prepare_v(v, *, pi=None, active=True, mean_dtype="float16", kv_block=128, status=None, mean_op=True):
    """vcb_prepare_v: returns (v8 [BH, T, 128, 128] u8, v_meta [BH, T, 2, 128] f32,
    mean_op [BH, T, 128, 16] bf16 as uint16, or None when not active or not
    asked for: only the exp-mode attention kernel reads it, the ExpCast one
    takes the means from v_meta)."""
    lib = _extension()
    b, h, s, dv = v.shape
    heads = b * h
    t = -(-s // kv_block)
    v8 = torch.empty((heads, t, 128, kv_block), dtype=torch.uint8, device=v.device)
    meta = torch.empty((heads, t, 2, 128), dtype=torch.float32, device=v.device)
    mop = torch.empty((heads, t, 128, 16), dtype=torch.int16, device=v.device) if active and mean_op else None
    vf = _flat(v)
    a = _abi.VArgs(v=vf.data_ptr(), dtype=_DTYPES[v.dtype], heads=heads, s=s, dv=dv, pi=_i(pi), active=int(active),
                   mean_type=_MEAN_TYPES[mean_dtype], kv_block=kv_block, v8=v8.data_ptr(), v_meta=meta.data_ptr(),
                   v_mean_op=_i(mop), status=_i(status))
    with torch.cuda.device(v.device):
        _abi.check(lib, lib.vcb_prepare_v(ctypes.byref(a), _stream(v.device)))
    return v8, meta, mop


def _attn_args(q8, qs, k8, ks, v8, meta, mop, out, *, heads, sq, sk, dv, q_block, k_quant_block, expcast,
               has_mean, scale, status):
    return _abi.AttnArgs(q8=q8.data_ptr(), q_scale=qs.data_ptr(), k8=k8.data_ptr(), k_scale=ks.data_ptr(),
                         v8=v8.data_ptr(), v_meta=meta.data_ptr(), v_mean_op=_i(mop), heads=heads, sq=sq, sk=sk,
                         dv=dv,
                         q_block=q_block, k_quant_block=k_quant_block, kv_block=128, expcast=int(expcast),
                         has_mean=int(has_mean), scale=float(scale), out=out.data_ptr(),
                         out_dtype=_DTYPES[out.dtype], status=_i(status))


def attention_fp8(q8, qs, k8, ks, v8, meta, *, heads, sq, sk, dv, mean_op=None, q_block=128, k_quant_block=256,
                  expcast=True, has_mean=True, scale, out_dtype=torch.bfloat16, out=None, status=None):
    """vcb_attention_fp8 on prepared operands (mean_op: the third output of
    prepare_v, needed with has_mean when not expcast); returns [heads, sq, dv]."""
    lib = _extension()
    if out is None:
        out = torch.empty((heads, sq, dv), dtype=out_dtype, device=q8.device)
    a = _attn_args(q8, qs, k8, ks, v8, meta, mean_op, out, heads=heads, sq=sq, sk=sk, dv=dv, q_block=q_block,
                   k_quant_block=k_quant_block, expcast=expcast, has_mean=has_mean, scale=scale, status=status)
    with torch.cuda.device(q8.device):
        _abi.check(lib, lib.vcb_attention_fp8(ctypes.byref(a), _stream(q8.device)))
    return out


def attention_fp8_probe(q8, qs, k8, ks, v8, meta, *, heads, sq, sk, dv, head, q_tile, tile_begin=0,
                        tile_count=None, mean_op=None, q_block=128, k_quant_block=256, expcast=True, has_mean=True, scale,
                        out_dtype=torch.bfloat16, status=None):
    """vcb_attention_fp8_probe: the full attention plus a dump of one CTA's
    softmax.  Returns (out, logits [n, 128, 128] f32, codes [n, 128, 128] u8,
    rowstat [n, 128, 4] f32 = running max, slope A, offset B, alpha) for KV
    tiles [tile_begin, tile_begin + n) of (head, q_tile)."""
    lib = _extension()
    dev = q8.device
    n = -(-sk // 128) - tile_begin if tile_count is None else tile_count
    out = torch.empty((heads, sq, dv), dtype=out_dtype, device=dev)
    logits = torch.empty((n, 128, 128), dtype=torch.float32, device=dev)
    codes = torch.empty((n, 128, 128), dtype=torch.uint8, device=dev)
    rowstat = torch.empty((n, 128, 4), dtype=torch.float32, device=dev)
    a = _attn_args(q8, qs, k8, ks, v8, meta, mean_op, out, heads=heads, sq=sq, sk=sk, dv=dv, q_block=q_block,
                   k_quant_block=k_quant_block, expcast=expcast, has_mean=has_mean, scale=scale, status=status)
    pr = _abi.AttnProbe(head=head, q_tile=q_tile, tile_begin=tile_begin, tile_count=n, logits=logits.data_ptr(),
                        codes=codes.data_ptr(), rowstat=rowstat.data_ptr())
    with torch.cuda.device(dev):
        _abi.check(lib, lib.vcb_attention_fp8_probe(ctypes.byref(a), ctypes.byref(pr), _stream(dev)))
    return out, logits, codes, rowstat
