"""vcb_quantize_qk_static: the Q/K quantiser for callers that cannot allocate
device memory (its K-mean scratch is a fixed array inside libvcb.so).

Checked through the C ABI against vcb_quantize_qk with a caller workspace,
bit for bit (the tolerance of every byte-level test here), on two calls in a
row, plus the size limit.  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import has_b200
from vc_attention_b200 import _abi

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_b200(), reason="needs a B200 GPU")]

SCRATCH_LIMIT = 8 << 20


def _args(q, k, outs, pi=None, workspace=None):
    heads, sq, d = q.shape
    sk = k.shape[1]
    q8, qs, k8, ks = outs
    a = _abi.QKArgs(q=q.data_ptr(), k=k.data_ptr(), dtype=_abi.VCB_BF16, heads=heads, sq=sq, sk=sk, d=d,
                    pi=None if pi is None else pi.data_ptr(), k_smooth=1, hadamard=1, q_block=128,
                    k_quant_block=256, q8=q8.data_ptr(), k8=k8.data_ptr(), q_scale=qs.data_ptr(),
                    k_scale=ks.data_ptr())
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel()
    return a


def _outputs(lib, heads, sq, sk):
    dev = "cuda"
    return (torch.full((heads, lib.vcb_padded_rows(sq, 128), 128), 0xAB, dtype=torch.uint8, device=dev),
            torch.full((heads, -(-sq // 128)), float("nan"), device=dev),
            torch.full((heads, lib.vcb_padded_rows(sk, 256), 128), 0xCD, dtype=torch.uint8, device=dev),
            torch.full((heads, -(-sk // 256)), float("nan"), device=dev))


def test_static_scratch_matches_caller_workspace_twice():
    lib = _abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(17)
    for call in range(2):
        heads, sq, sk = 6, 1000 + 64 * call, 3000 - 128 * call
        q = torch.randn(heads, sq, 128, device="cuda", generator=g).to(torch.bfloat16)
        k = (torch.randn(heads, sk, 128, device="cuda", generator=g)
             + torch.randn(heads, 1, 128, device="cuda", generator=g) * 1.5).to(torch.bfloat16)
        pi = torch.stack([torch.randperm(sk, device="cuda", generator=g) for _ in range(heads)]).int()
        ws = torch.empty(lib.vcb_qk_workspace(heads, sk), dtype=torch.uint8, device="cuda")
        want = _outputs(lib, heads, sq, sk)
        _abi.check(lib, lib.vcb_quantize_qk(ctypes.byref(_args(q, k, want, pi, ws)), stream))
        got = _outputs(lib, heads, sq, sk)
        _abi.check(lib, lib.vcb_quantize_qk_static(ctypes.byref(_args(q, k, got, pi)), stream))
        torch.cuda.synchronize()
        # the second call runs on different sizes over the scratch the first
        # one left behind; both must equal the caller-workspace result
        for w, o in zip(want, got):
            assert np.array_equal(w.cpu().numpy().view(np.uint8), o.cpu().numpy().view(np.uint8))


def test_static_scratch_rejects_sizes_beyond_the_limit():
    lib = _abi.load()
    heads, sk = 64, 256 * 300                 # 64 * 301 * 512 bytes > 8 MiB
    assert heads * (1 + sk // 256) * 512 > SCRATCH_LIMIT
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    a = _abi.QKArgs(q=dummy.data_ptr(), k=dummy.data_ptr(), dtype=_abi.VCB_BF16, heads=heads, sq=128, sk=sk,
                    d=128, k_smooth=1, hadamard=1, q_block=128, k_quant_block=256, q8=dummy.data_ptr(),
                    k8=dummy.data_ptr(), q_scale=dummy.data_ptr(), k_scale=dummy.data_ptr())
    rc = lib.vcb_quantize_qk_static(ctypes.byref(a), None)
    assert rc == _abi.VCB_ERR_INVALID_ARGUMENT
    assert "at most" in _abi.last_error(lib)
