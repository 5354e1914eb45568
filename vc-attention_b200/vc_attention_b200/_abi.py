"""ctypes binding of libvcb.so (include/vcb.h).

The structures below mirror the C declarations field for field.  Calls pass
raw device pointers (``tensor.data_ptr()``) and the current PyTorch CUDA
stream; PyTorch only allocates memory and orders streams.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libvcb.so"
ABI_VERSION = 2
NUMERICAL_CONTRACT_VERSION = 2

VCB_OK = 0
VCB_ERR_INVALID_ARGUMENT = 1
VCB_ERR_UNSUPPORTED_DEVICE = 2
VCB_ERR_CUDA = 3
VCB_ERR_WORKSPACE = 4

VCB_F32, VCB_F16, VCB_BF16 = 0, 1, 2
FLAG_NONFINITE = 1
FLAG_TIMEOUT = 2
FLAG_INTERNAL = 4

c_int, c_int64, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p


class QKArgs(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("dtype", c_int), ("heads", c_int64), ("sq", c_int64),
                ("sk", c_int64), ("d", c_int), ("pi", c_void_p), ("k_smooth", c_int), ("hadamard", c_int),
                ("q_out", c_void_p), ("k_out", c_void_p), ("q_block", c_int), ("k_quant_block", c_int),
                ("q8", c_void_p), ("k8", c_void_p), ("q_scale", c_void_p), ("k_scale", c_void_p),
                ("status", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t)]


class GroupArgs(ctypes.Structure):
    _fields_ = [("v", c_void_p), ("dtype", c_int), ("heads", c_int64), ("s", c_int64), ("d", c_int),
                ("clusters", c_int), ("iterations", c_int), ("centers_in", c_void_p), ("centers_out", c_void_p),
                ("pi", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t)]


class VArgs(ctypes.Structure):
    _fields_ = [("v", c_void_p), ("dtype", c_int), ("heads", c_int64), ("s", c_int64), ("dv", c_int),
                ("pi", c_void_p), ("active", c_int), ("mean_type", c_int), ("kv_block", c_int), ("v8", c_void_p),
                ("v_meta", c_void_p), ("v_mean_op", c_void_p), ("status", c_void_p)]


class AttnArgs(ctypes.Structure):
    _fields_ = [("q8", c_void_p), ("q_scale", c_void_p), ("k8", c_void_p), ("k_scale", c_void_p),
                ("v8", c_void_p), ("v_meta", c_void_p), ("v_mean_op", c_void_p), ("heads", c_int64),
                ("sq", c_int64), ("sk", c_int64),
                ("dv", c_int), ("q_block", c_int), ("k_quant_block", c_int), ("kv_block", c_int),
                ("expcast", c_int), ("has_mean", c_int), ("scale", c_float), ("out", c_void_p),
                ("out_dtype", c_int), ("status", c_void_p)]


class AttnProbe(ctypes.Structure):
    _fields_ = [("head", c_int64), ("q_tile", c_int64), ("tile_begin", c_int), ("tile_count", c_int),
                ("logits", c_void_p), ("codes", c_void_p), ("rowstat", c_void_p)]


class ForwardArgs(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("dtype", c_int), ("heads", c_int64),
                ("sq", c_int64), ("sk", c_int64), ("d", c_int), ("dv", c_int), ("pi", c_void_p),
                ("q_block", c_int), ("k_quant_block", c_int), ("kv_block", c_int), ("smooth", c_int),
                ("expcast", c_int), ("mean_type", c_int), ("scale", c_float), ("k_smooth", c_int),
                ("hadamard", c_int), ("out", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
                ("status", c_void_p)]


# name -> (restype, argtypes); every symbol include/vcb.h declares.
SIGNATURES = {
    "vcb_abi_version": (c_int, []),
    "vcb_numerical_contract_version": (c_int, []),
    "vcb_build_info": (ctypes.c_char_p, []),
    "vcb_last_error": (c_size_t, [ctypes.c_char_p, c_size_t]),
    "vcb_check_device": (c_int, [c_int]),
    "vcb_expcast_codes": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "vcb_padded_rows": (c_int64, [c_int64, c_int]),
    "vcb_qk_workspace": (c_size_t, [c_int64, c_int64]),
    "vcb_preprocess_qk": (c_int, [ctypes.POINTER(QKArgs), c_void_p]),
    "vcb_quantize_qk": (c_int, [ctypes.POINTER(QKArgs), c_void_p]),
    "vcb_quantize_qk_static": (c_int, [ctypes.POINTER(QKArgs), c_void_p]),
    "vcb_group_workspace": (c_size_t, [c_int64, c_int64, c_int, c_int]),
    "vcb_group_values": (c_int, [ctypes.POINTER(GroupArgs), c_void_p]),
    "vcb_prepare_v": (c_int, [ctypes.POINTER(VArgs), c_void_p]),
    "vcb_attention_fp8": (c_int, [ctypes.POINTER(AttnArgs), c_void_p]),
    "vcb_attention_fp8_probe": (c_int, [ctypes.POINTER(AttnArgs), ctypes.POINTER(AttnProbe), c_void_p]),
    "vcb_forward_workspace": (c_size_t, [ctypes.POINTER(ForwardArgs)]),
    "vcb_forward": (c_int, [ctypes.POINTER(ForwardArgs), c_void_p]),
    "vcb_read_status": (c_int, [c_void_p, c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "vcb_wait_selftest": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"libvcb error {code}: {message}")
        self.code = code


def load(path=None):
    """Load libvcb.so once; raise RuntimeError if it is missing or stale."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = pathlib.Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libvcb.so not found at {p}. Build it with `python __graft_entry__.py build` "
                "(or `make -C vc-attention_b200/csrc`). No reference fallback was used.")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.vcb_abi_version() != ABI_VERSION or lib.vcb_numerical_contract_version() != NUMERICAL_CONTRACT_VERSION:
            raise RuntimeError("Stale libvcb.so: rebuild with `make -C vc-attention_b200/csrc`")
        _lib = lib
        return lib


def last_error(lib):
    buf = ctypes.create_string_buffer(512)
    lib.vcb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(lib, rc):
    if rc != VCB_OK:
        msg = last_error(lib)
        if rc == VCB_ERR_INVALID_ARGUMENT:
            raise ValueError(msg)
        raise NativeError(rc, msg)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())
