"""TEST INFRASTRUCTURE ONLY: numpy front end of the C restatement (kz_oracle.c).

Every function here is a checker for the CUDA library; see kz_oracle.c for the
reference file:line each one restates.  Arrays are numpy, C-contiguous.
"""
import ctypes
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkz_oracle.so")

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, D, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_int
        L.kzo_absmax_f32.argtypes = [P, I64, ctypes.POINTER(D)]
        L.kzo_scale_from_absmax.argtypes = [D]
        L.kzo_scale_from_absmax.restype = D
        L.kzo_quantize_tensor_f32.argtypes = [P, I64, P, ctypes.POINTER(D)]
        L.kzo_quantize_with_absmax_f32.argtypes = [P, I64, D, P, ctypes.POINTER(D)]
        L.kzo_quantize_cols_f32.argtypes = [P, I64, I64, P, P]
        L.kzo_quantize_rows_f32.argtypes = [P, I64, I64, P, P]
        L.kzo_dequantize_i8.argtypes = [P, I64, D, P]
        L.kzo_matmul_f32.argtypes = [P, P, P, I64, I64, I64, I]
        L.kzo_add_bias_f32.argtypes = [P, P, I64, I64]
        L.kzo_act_f32.argtypes = [P, I64, I]
        L.kzo_qlinear_w8a32.argtypes = [P, I64, I64, P, D, P, I64, I, P, I]
        L.kzo_gemm_i8_i32.argtypes = [P, P, P, I64, I64, I64, I]
        L.kzo_epilogue_f32.argtypes = [P, I64, I64, P, I64, P, I64, P, I, P]
        L.kzo_layernorm_f32.argtypes = [P, P, I64, I64, P, P, ctypes.c_float, P, P]
        L.kzo_expf_f32.argtypes = [P, I64, P]
        L.kzo_attention_f32.argtypes = [P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, P, I64, I64, I64, I,
                                        ctypes.c_float, P, I64, I]
        _lib = L
    return _lib


class NonFiniteError(ValueError):
    pass


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i8(a):
    return np.ascontiguousarray(a, dtype=np.int8)


def default_threads():
    return os.cpu_count() or 1


def absmax(x):
    x = _f32(x)
    out = ctypes.c_double()
    if lib().kzo_absmax_f32(_p(x), x.size, ctypes.byref(out)):
        raise NonFiniteError("absmax: non-finite value")
    return out.value


def scale_from_absmax(m):
    return lib().kzo_scale_from_absmax(float(m))


def quantize_tensor(x):
    """quantize.py:66-70 -> (int8 codes shaped like x, double scale)."""
    x = _f32(x)
    q = np.empty(x.shape, np.int8)
    s = ctypes.c_double()
    if lib().kzo_quantize_tensor_f32(_p(x), x.size, _p(q), ctypes.byref(s)):
        raise NonFiniteError("quantize: non-finite value")
    return q, s.value


def quantize_with_absmax(x, max_abs):
    x = _f32(x)
    q = np.empty(x.shape, np.int8)
    s = ctypes.c_double()
    lib().kzo_quantize_with_absmax_f32(_p(x), x.size, float(max_abs), _p(q), ctypes.byref(s))
    return q, s.value


def quantize_cols(w):
    """Per-output-channel quantize of a [K, N] weight -> (codes [N, K], scales [N])."""
    w = _f32(w)
    K, N = w.shape
    qT = np.empty((N, K), np.int8)
    s = np.empty(N, np.float64)
    if lib().kzo_quantize_cols_f32(_p(w), K, N, _p(qT), _p(s)):
        raise NonFiniteError("quantize_cols: non-finite value")
    return qT, s


def quantize_rows(x):
    x = _f32(x)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float64)
    if lib().kzo_quantize_rows_f32(_p(x), M, K, _p(q), _p(s)):
        raise NonFiniteError("quantize_rows: non-finite value")
    return q, s


def dequantize(q, scale):
    q = _i8(q)
    out = np.empty(q.shape, np.float32)
    lib().kzo_dequantize_i8(_p(q), q.size, float(scale), _p(out))
    return out


def matmul_f32(a, b, threads=None):
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    out = np.empty((M, N), np.float32)
    lib().kzo_matmul_f32(_p(a), _p(b), _p(out), M, K, N, threads or default_threads())
    return out


def qlinear_w8a32(x, q, scale, bias=None, act=0, threads=None):
    """Reference qlinear (quantize.py:115-122) + optional act: q is [K, N] row-major."""
    x, q = _f32(x), _i8(q)
    M, K = x.shape
    K2, N = q.shape
    assert K == K2
    b = _f32(bias) if bias is not None else None
    out = np.empty((M, N), np.float32)
    lib().kzo_qlinear_w8a32(_p(x), M, K, _p(q), float(scale), _p(b), N, act, _p(out), threads or default_threads())
    return out


def gemm_i8(a, b, threads=None):
    """acc = a @ b.T with a [M, K] int8 and b [N, K] int8 -> int32 [M, N]."""
    a, b = _i8(a), _i8(b)
    M, K = a.shape
    N, K2 = b.shape
    assert K == K2
    out = np.empty((M, N), np.int32)
    lib().kzo_gemm_i8_i32(_p(a), _p(b), _p(out), M, N, K, threads or default_threads())
    return out


def epilogue(acc, row_scale, col_scale, bias=None, act=0):
    """y = act(((float)acc * row_scale) * col_scale + bias), fp32 throughout.

    row_scale / col_scale: a scalar (per-tensor) or a vector (per-row / per-column),
    given as doubles or floats; they are narrowed to float32 once, as the GPU does.
    """
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    M, N = acc.shape
    rs = np.atleast_1d(np.asarray(row_scale, dtype=np.float64)).astype(np.float32)
    cs = np.atleast_1d(np.asarray(col_scale, dtype=np.float64)).astype(np.float32)
    b = _f32(bias) if bias is not None else None
    out = np.empty((M, N), np.float32)
    lib().kzo_epilogue_f32(_p(acc), M, N, _p(rs), 0 if rs.size == 1 else 1, _p(cs), 0 if cs.size == 1 else 1,
                           _p(b), act, _p(out))
    return out


def w8a8_linear(x, w_qT, w_scales, bias=None, act=0, per_row=False, threads=None):
    """The W8A8 quantized linear: quantize x (per-tensor or per-row), int8 GEMM
    against K-major codes, fused epilogue.  Returns (y, x_codes, x_scale(s), acc)."""
    if per_row:
        xq, xs = quantize_rows(x)
    else:
        xq, xs = quantize_tensor(x)
    acc = gemm_i8(xq, w_qT, threads)
    y = epilogue(acc, xs, w_scales, bias, act)
    return y, xq, xs, acc


def layernorm(x, gamma=None, beta=None, eps=1e-5, residual=None):
    """The reference's LayerNorm over the last axis (nn.py:323-331, ordered
    fp32 sums, kz_oracle.c).  With `residual`, the LayerNorm of x + residual;
    returns y, or (y, x + residual)."""
    x = _f32(x)
    D = x.shape[-1]
    M = x.size // D
    r = _f32(residual) if residual is not None else None
    g = _f32(gamma) if gamma is not None else None
    b = _f32(beta) if beta is not None else None
    y = np.empty(x.shape, np.float32)
    total = np.empty(x.shape, np.float32) if r is not None else None
    lib().kzo_layernorm_f32(_p(x), _p(r), M, D, _p(g), _p(b), float(np.float32(eps)), _p(total), _p(y))
    return y if r is None else (y, total)


def attention(q, k, v, heads, mask=None, causal=False, exp="rn"):
    """The reference's scaled dot-product attention core (nn.py:410-423 composed
    from Tensor ops, kz_oracle.c): q [B, Sq, H*dk], k and v [B, Sk, H*dk],
    heads split along the last axis; returns the heads-merged [B, Sq, H*dk].
    mask: additive, broadcastable to [B, H, Sq, Sk]; causal: keys j > i masked
    (-1e9).  exp: "rn" the correctly rounded fp32 exp (the CUDA kernel's),
    "libm" the host's expf (the reference's std::exp)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Sq, D = q.shape
    Sk = k.shape[1]
    dk = D // heads
    out = np.empty((B, Sq, D), np.float32)
    m = None
    strides = (0, 0, 0)
    if mask is not None and not causal:
        m = np.ascontiguousarray(np.broadcast_to(_f32(mask), (B, heads, Sq, Sk)))
        strides = (heads * Sq * Sk, Sq * Sk, Sk)
    scale = float(np.float32(1.0 / math.sqrt(dk)))      # nn.py:414, from_flat of a Python float
    lib().kzo_attention_f32(_p(q), _p(k), _p(v), B, heads, Sq, Sk, dk, D, D, D, _p(m), *strides, int(causal),
                            scale, _p(out), D, 1 if exp == "libm" else 0)
    return out


def expf_host(x):
    """The host libm's expf of every element (the reference's exp_fwd)."""
    x = _f32(x)
    out = np.empty_like(x)
    lib().kzo_expf_f32(_p(x), x.size, _p(out))
    return out
