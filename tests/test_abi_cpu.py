"""The C-ABI library loads on a machine without a GPU, exports every symbol
include/vcb.h declares, and rejects bad arguments before touching the device."""
import ctypes
import pathlib
import re

import pytest

from vc_attention_b200 import _abi

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "vcb.h"


def declared_symbols():
    return sorted(set(re.findall(r"^VCB_API [^(]*?\b(vcb_\w+)\(", HEADER.read_text(), flags=re.M)))


def test_header_declares_the_bound_api():
    assert declared_symbols() == sorted(_abi.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.vcb_abi_version() == 2
    assert lib.vcb_numerical_contract_version() == 2
    import json
    info = json.loads(lib.vcb_build_info().decode())
    assert info["target"] == "sm_100a" and info["fully_fused_attention"] is True


def test_padded_rows_and_workspace_sizes():
    lib = _abi.load()
    assert lib.vcb_padded_rows(100, 128) == 128
    assert lib.vcb_padded_rows(300, 256) == 512
    assert lib.vcb_padded_rows(300, 64) == 384
    assert lib.vcb_padded_rows(100, 96) == 384
    assert lib.vcb_qk_workspace(2, 1000) > 0
    a = _abi.ForwardArgs(heads=40, sq=32768, sk=32768, d=128, dv=128, q_block=128, k_quant_block=256, kv_block=128)
    ws = lib.vcb_forward_workspace(ctypes.byref(a))
    # q8 + k8 + v8 (1 byte each) + scales + V metadata + K-mean scratch
    assert 3 * 40 * 32768 * 128 < ws < 3 * 40 * 32768 * 128 * 1.1
    # the bf16 mean operand [heads, T, 128, 16] is laid out only for V-Smooth
    # in the exp modes; the ExpCast kernel reads the means from v_meta
    sizes = {}
    for smooth, expcast in ((0, 0), (1, 0), (0, 1), (1, 1)):
        a.smooth, a.expcast = smooth, expcast
        sizes[smooth, expcast] = lib.vcb_forward_workspace(ctypes.byref(a))
    assert sizes[1, 0] - sizes[0, 0] == 40 * 256 * 128 * 16 * 2
    assert sizes[1, 1] == sizes[0, 1] == sizes[0, 0]


@pytest.mark.parametrize("field,value,match", [
    ("q_block", 48, "q_block"), ("kv_block", 64, "kv_block"), ("k_quant_block", 200, "k_quant_block"),
    ("mean_type", 3, "mean_type"), ("dtype", 9, "dtype"),
])
def test_forward_rejects_bad_geometry_without_a_device(field, value, match):
    lib = _abi.load()
    a = _abi.ForwardArgs(q=16, k=16, v=16, out=16, workspace=256, workspace_bytes=1 << 40, dtype=2, heads=1,
                         sq=128, sk=128, d=128, dv=128, q_block=128, k_quant_block=256, kv_block=128,
                         mean_type=1, scale=0.1)
    setattr(a, field, value)
    rc = lib.vcb_forward(ctypes.byref(a), None)
    assert rc == _abi.VCB_ERR_INVALID_ARGUMENT
    assert match in _abi.last_error(lib)


def test_null_pointers_are_rejected():
    lib = _abi.load()
    assert lib.vcb_forward(None, None) == _abi.VCB_ERR_INVALID_ARGUMENT
    a = _abi.GroupArgs(heads=1, s=10, d=16, clusters=8, iterations=2)
    assert lib.vcb_group_values(ctypes.byref(a), None) == _abi.VCB_ERR_INVALID_ARGUMENT
    a = _abi.AttnArgs(heads=1, sq=1, sk=1, dv=1, q_block=128, k_quant_block=256, kv_block=128, scale=1.0)
    assert lib.vcb_attention_fp8(ctypes.byref(a), None) == _abi.VCB_ERR_INVALID_ARGUMENT
    assert lib.vcb_expcast_codes(None, None, -1, None) == _abi.VCB_ERR_INVALID_ARGUMENT
    assert lib.vcb_wait_selftest(0, None, None, None, None) == _abi.VCB_ERR_INVALID_ARGUMENT
    # a misaligned copy source is refused before any CUDA call
    assert lib.vcb_wait_selftest(0, 8, None, 16, None) == _abi.VCB_ERR_INVALID_ARGUMENT
    assert "aligned" in _abi.last_error(lib)


def test_check_raises_value_error_for_invalid_arguments():
    lib = _abi.load()
    with pytest.raises(ValueError, match="null"):
        _abi.check(lib, lib.vcb_forward(None, None))
