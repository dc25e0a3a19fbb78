"""ctypes binding of libkz (include/kz.h), the package's only compute backend.

There is no CPU fallback: if the library is missing or the current device is
not an sm_100 GPU, every compute entry point raises.  Arguments are plain
integers (device pointers, sizes, a CUDA stream handle); no torch types cross
the C ABI.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libkz.so")
INCLUDE_H = os.path.join(os.path.dirname(_HERE), "include", "kz.h")

KZ_OK = 0
KZ_ERR_INVALID_ARGUMENT = 1
KZ_ERR_NONFINITE = 2
KZ_ERR_CUDA = 3
KZ_ERR_UNSUPPORTED_DEVICE = 4
KZ_ERR_DEVICE_TIMEOUT = 5

KZ_ACT_NONE, KZ_ACT_RELU, KZ_ACT_GELU = 0, 1, 2
KZ_PARTIALS_WORDS = 1024
KZ_IPC_HANDLE_BYTES = 64

_P, _I64, _I, _D, _F, _U64, _SZ = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double,
                                    ctypes.c_float, ctypes.c_uint64, ctypes.c_size_t)

# name -> (restype, argtypes); mirrors include/kz.h
SIGNATURES = {
    "kz_last_error": (ctypes.c_char_p, []),
    "kz_version": (_I, []),
    "kz_device_supported": (_I, [_I]),
    "kz_randn_host": (_I, [_P, _I64, _F, _U64]),
    "kz_device_status": (_I, [ctypes.POINTER(_I), _I, _P]),
    "kz_absmax_f32": (_I, [_P, _I64, _P, _P]),
    "kz_quantize_partials_f32": (_I, [_P, _I64, _P, _P, _P, _P, _P]),
    "kz_quantize_tensor_f32": (_I, [_P, _I64, _P, _P, _P, _P, _P]),
    "kz_layernorm_partials_f32": (_I, [_P, _I64, _I64, _P, _P, _F, _P, _P, _P]),
    "kz_add_layernorm_partials_f32": (_I, [_P, _P, _I64, _I64, _P, _P, _F, _P, _P, _P, _P]),
    "kz_attention_f32": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64,
                              _I, _F, _P, _I64, _P, _P]),
    "kz_attention_smem_bytes": (_I, [_I64, _I64]),
    "kz_quantize_cols_workspace_bytes": (_SZ, [_I64, _I64]),
    "kz_quantize_cols_f32": (_I, [_P, _I64, _I64, _P, _P, _P, _P, _SZ, _P]),
    "kz_quantize_cols_f32_noalloc": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "kz_quantize_rows_f32": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "kz_dequantize_i8_f32": (_I, [_P, _I64, _D, _P, _P]),
    "kz_dequantize_uses_table": (_I, [_D]),
    "kz_dequantize_cols_i8_f32": (_I, [_P, _I64, _I64, _P, _P, _P]),
    "kz_qlinear_w8a32_f32": (_I, [_P, _I64, _I64, _P, _D, _P, _I64, _I, _P, _P]),
    "kz_set_sm_count_target": (_I, [_I]),
    "kz_gemm_i8": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _I, _P, _P, _I64, _P, _P]),
    "kz_gemm_i8_gated": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _I, _P, _P, _I64, _P, _P,
                              ctypes.c_uint32, _I, _I64, _P]),
    "kz_gemm_i8_allgather": (_I, [_P, _P, _P, _I, _I, _P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _P,
                                  ctypes.c_uint32, _I64, _I, _P]),
    "kz_peer_alloc": (_I, [_SZ, ctypes.POINTER(_P), _P]),
    "kz_peer_open": (_I, [_P, ctypes.POINTER(_P)]),
    "kz_peer_close": (_I, [_P]),
    "kz_peer_free": (_I, [_P]),
    "kz_copy_and_flag": (_I, [_P, _P, _SZ, _P, ctypes.c_uint32, _P]),
}

_lib = None
_lock = threading.Lock()


class KzError(RuntimeError):
    """A libkz call failed; `code` is the kz_status_code."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def load():
    """The loaded library; raises ImportError when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libkz.so not found at {LIB_PATH}: build it with `make -C kansaiml_b200/csrc` "
                    "(or __graft_entry__.build()); kansaiml_b200 has no CPU fallback")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error():
    return load().kz_last_error().decode(errors="replace")


def check(status, what=""):
    if status != KZ_OK:
        msg = last_error()
        if status == KZ_ERR_NONFINITE:
            raise ValueError(f"{what}: {msg}")
        if status == KZ_ERR_INVALID_ARGUMENT:
            raise KzError(status, f"{what}: invalid argument: {msg}")
        raise KzError(status, f"{what}: {msg}")


def call(name, *args):
    """Calls `name` and raises on a non-zero status."""
    check(getattr(load(), name)(*args), name)
