"""ctypes binding of libsamrs_b200.so (the C ABI in include/samrs_b200.h).

The library is built in-tree by sam-rs_b200/build.py. Loading fails loudly when it is missing: there
is no CPU or PyTorch fallback behind the package's ops.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsamrs_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "samrs_b200.h")

F32, F16, BF16 = 0, 1, 2
IMPL_AUTO, IMPL_SIMT, IMPL_TC = 0, 1, 2
EPI_BIAS, EPI_BIAS_RESIDUAL, EPI_BIAS_GELU = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_LAUNCH, ERR_DEVICE, ERR_NODEVICE = 0, -1, -2, -3, -4, -5

_lib = None


class SamrsError(RuntimeError):
    """An entry point returned a nonzero code; the message is samrs_last_error()."""

    def __init__(self, code, msg):
        super().__init__(f"samrs error {code}: {msg}")
        self.code = code


def header_symbols():
    """Names of every function declared in include/samrs_b200.h."""
    text = open(HEADER).read()
    return re.findall(r"SAMRS_API\s+[\w\s\*]+?\b(samrs_\w+)\s*\(", text)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python sam-rs_b200/build.py` "
                               "(the package has no fallback path)")
        l = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        l.samrs_relpos_attn_fwd.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, f32, i32, vp]
        l.samrs_relpos_attn_fwd_ex.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, f32, i32, i32, vp]
        l.samrs_relpos_softmax_fwd.argtypes = [vp, vp, vp, vp, i64, i32, i32, i32, f32, i32, vp]
        l.samrs_qkv_split_fwd.argtypes = [vp, vp, vp, i64, i32, i32, i32, i32, vp]
        l.samrs_qkv_split_window_fwd.argtypes = [vp, vp, vp, i64, i32, i32, i32, i32, i32, i32, vp]
        l.samrs_window_merge_fwd.argtypes = [vp, vp, i64, i32, i32, i32, i32, i32, i32, vp]
        l.samrs_linear_fwd.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, vp]
        l.samrs_qkv_linear_window_fwd.argtypes = [vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, i32, vp]
        l.samrs_layer_norm_fwd.argtypes = [vp, vp, vp, vp, i64, i32, f32, i32, vp]
        l.samrs_test_hooks.argtypes = [i64, i32]
        l.samrs_last_error.restype = ctypes.c_char_p
        l.samrs_device_status.argtypes = [vp, i32]
        l.samrs_recompute_count.argtypes = [vp, ctypes.POINTER(i64), i32]
        l.samrs_selftest_ex2.argtypes = [vp, vp, vp, i64, vp]
        l.samrs_global_policy.argtypes = [vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i32), i32]
        for name in ("samrs_relpos_attn_fwd", "samrs_relpos_attn_fwd_ex", "samrs_relpos_softmax_fwd",
                     "samrs_qkv_split_fwd", "samrs_qkv_split_window_fwd", "samrs_window_merge_fwd",
                     "samrs_abi_version", "samrs_device_status", "samrs_recompute_count",
                     "samrs_selftest_ex2", "samrs_linear_fwd", "samrs_qkv_linear_window_fwd",
                     "samrs_layer_norm_fwd", "samrs_test_hooks", "samrs_global_policy"):
            getattr(l, name).restype = i32
        _lib = l
    return _lib


def check(rc):
    if rc != OK:
        raise SamrsError(rc, lib().samrs_last_error().decode())
    return rc
