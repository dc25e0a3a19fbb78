"""Int8 quantization with the reference's API (python/kansai/quantize.py).

Same names, arguments and results as the reference module:

* ``quantize_symmetric(tensor) -> (q: list[int], scale: float, shape: list)``
  (quantize.py:50-70) -- bit-exact codes and the identical double scale;
* ``dequantize(q, scale, shape) -> Tensor`` (quantize.py:73-77) -- bit-exact;
* ``QTensor`` (quantize.py:80-112) with ``q``, ``scale``, ``shape``,
  ``from_tensor``, ``dequantize``, ``nbytes`` (== numel, the 4x claim);
* ``qlinear(x, qweight, bias)`` (quantize.py:115-122) and ``QLinear(linear)``
  (quantize.py:125-144) -- by default with the reference's exact semantics
  (W8A32: x @ dequantize(W) + b, bit-identical fp32 results).

What differs is where the work happens: codes live in device memory and every
numeric step runs in libkz on the GPU.  ``QTensor.q`` is materialised as a
Python list only when read.  NaN/Inf inputs raise ValueError, as Python's
round() makes the reference do.

Extensions (no reference implementation; the reference's rounding rules applied
to new granularities, quantize.py:35-44 lists them as future work):

* ``per_channel=True``: one scale per output feature, i.e. per column of the
  reference's [in, out] weight (nn.py:74-81); codes stored K-major [out, in];
* W8A8: activations quantized per tensor (or per row) on the fly, an
  int8 x int8 -> int32 tensor-core GEMM, and the rescale / bias / activation
  fused into its epilogue.  ``QLinear(linear, per_channel=True)`` uses it.
"""
import ctypes
import math

import numpy as np
import torch

from . import _lib
from .tensor import Tensor, as_tensor, ptr, require_cuda, stream_handle

_ACTS = {None: _lib.KZ_ACT_NONE, "none": _lib.KZ_ACT_NONE, "relu": _lib.KZ_ACT_RELU, "gelu": _lib.KZ_ACT_GELU}

# ------------------------------------------------------------- workspaces
_partials_cache = {}


def new_partials(device):
    """A zero-filled KZ_PARTIALS_WORDS buffer (the fused quantize keeps its
    grid barrier in the last two words, which must start at zero)."""
    return torch.zeros(_lib.KZ_PARTIALS_WORDS, dtype=torch.int32, device=device)


def partials_buffer(device):
    """A KZ_PARTIALS_WORDS scratch buffer private to (device, current stream):
    calls on one stream are ordered, so they may share it."""
    key = (device.index, stream_handle(device))
    buf = _partials_cache.get(key)
    if buf is None:
        buf = new_partials(device)
        _partials_cache[key] = buf
    return buf


def _dev_tensor(t, what):
    if not isinstance(t, Tensor):
        t = as_tensor(t)
    require_cuda(t.data, what)
    x = t.data
    if not x.is_contiguous():
        x = x.contiguous()
    return x


# ------------------------------------------------------- device primitives

def quantize_tensor_device(x):
    """Per-tensor quantize of a contiguous fp32 CUDA tensor.
    Returns (codes int8 like x, scale float64[1], scale float32[1])."""
    dev = x.device
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    s64 = torch.empty(1, dtype=torch.float64, device=dev)
    s32 = torch.empty(1, dtype=torch.float32, device=dev)
    _lib.call("kz_quantize_tensor_f32", ptr(x), x.numel(), ptr(q), ptr(s64), ptr(s32),
              ptr(partials_buffer(dev)), stream_handle(dev))
    return q, s64, s32


def quantize_partials_device(x, partials, q=None, s64=None, s32=None):
    """Per-tensor quantize of a contiguous fp32 CUDA tensor with the absmax
    given by `partials` (kz_quantize_partials_f32).  Writes into q / s64 / s32
    when given (e.g. one row chunk of a larger code buffer).  Returns
    (codes int8 like x, scale float64[1], scale float32[1])."""
    dev = x.device
    if q is None:
        q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    if s64 is None:
        s64 = torch.empty(1, dtype=torch.float64, device=dev)
    if s32 is None:
        s32 = torch.empty(1, dtype=torch.float32, device=dev)
    _lib.call("kz_quantize_partials_f32", ptr(x), x.numel(), ptr(partials), ptr(q), ptr(s64), ptr(s32),
              stream_handle(dev))
    return q, s64, s32


def layernorm_partials_device(x, weight=None, bias=None, eps=1e-5, partials=None, residual=None):
    """LayerNorm over the last axis of a contiguous fp32 CUDA tensor, plus the
    absmax partials of the result (kz_layernorm_partials_f32).  With
    `residual` (same shape), the LayerNorm of x + residual, the sum returned
    too (kz_add_layernorm_partials_f32).  Returns (y, partials) or
    (y, partials, x + residual)."""
    dev = x.device
    D = x.shape[-1]
    M = x.numel() // D
    if partials is None:
        partials = partials_buffer(dev)
    y = torch.empty(x.shape, dtype=torch.float32, device=dev)
    w = _dev_tensor(weight, "layernorm weight") if weight is not None else None
    b = _dev_tensor(bias, "layernorm bias") if bias is not None else None
    if residual is None:
        _lib.call("kz_layernorm_partials_f32", ptr(x), M, D, ptr(w), ptr(b), float(eps), ptr(y), ptr(partials),
                  stream_handle(dev))
        return y, partials
    if tuple(residual.shape) != tuple(x.shape):
        raise ValueError(f"add_layernorm: residual shape {list(residual.shape)} != {list(x.shape)}")
    total = torch.empty(x.shape, dtype=torch.float32, device=dev)
    _lib.call("kz_add_layernorm_partials_f32", ptr(x), ptr(residual), M, D, ptr(w), ptr(b), float(eps), ptr(total),
              ptr(y), ptr(partials), stream_handle(dev))
    return y, partials, total


def _rows_view(t, what):
    """(batch, seq, features) CUDA fp32 view whose rows are evenly strided and
    whose features are contiguous: returns its row stride in floats."""
    if t.dtype != torch.float32 or not t.is_cuda or t.dim() != 3:
        raise ValueError(f"attention: {what} must be a 3-d fp32 CUDA tensor")
    if t.shape[2] > 1 and t.stride(2) != 1:
        raise ValueError(f"attention: {what} needs contiguous features")
    if t.shape[1] > 1:
        rs = t.stride(1)
    else:   # one row per batch: the batch stride is the row stride
        rs = t.stride(0) if t.shape[0] > 1 else t.shape[2]
    if t.shape[0] > 1 and t.stride(0) != t.shape[1] * rs:
        raise ValueError(f"attention: {what}'s batches must follow each other row by row")
    return rs


def attention_device(q, k, v, heads, mask=None, causal=False, partials=None):
    """softmax(q k^T / sqrt(d_k) + mask) v per head, fp32, in the reference's
    operation order (kz_attention_f32; MultiHeadAttention.forward,
    nn.py:410-427).  q [B, Sq, H*d_k], k and v [B, Sk, H*d_k] (views with
    strided rows allowed, e.g. slices of one fused q|k|v projection); mask
    additive, broadcastable to [B, H, Sq, Sk]; causal: keys after each query
    masked, as causal_mask() does (mask then unused).  Returns the
    heads-merged [B, Sq, H*d_k] output and the absmax partials of it."""
    dev = q.device
    B, Sq, D = q.shape
    Sk = k.shape[1]
    if D % heads:
        raise ValueError(f"attention: {D} features do not split into {heads} heads")
    if tuple(k.shape) != (B, Sk, D) or tuple(v.shape) != (B, Sk, D):
        raise ValueError(f"attention: q {list(q.shape)}, k {list(k.shape)}, v {list(v.shape)} do not match")
    dk = D // heads
    qrs, krs, vrs = _rows_view(q, "q"), _rows_view(k, "k"), _rows_view(v, "v")
    if partials is None:
        partials = partials_buffer(dev)
    out = torch.empty((B, Sq, D), dtype=torch.float32, device=dev)
    m, ms = None, (0, 0, 0)
    if mask is not None and not causal:
        m = mask.to(device=dev, dtype=torch.float32)
        try:
            m = m.expand(B, heads, Sq, Sk)
        except RuntimeError as e:
            raise ValueError(f"attention: mask {list(mask.shape)} does not broadcast to "
                             f"{[B, heads, Sq, Sk]}") from e
        if Sk > 1 and m.stride(3) != 1:
            m = m.contiguous()
        ms = (m.stride(0), m.stride(1), m.stride(2))
    scale = float(np.float32(1.0 / math.sqrt(dk)))   # nn.py:414: from_flat([1 / sqrt(d_k)])
    _lib.call("kz_attention_f32", ptr(q), ptr(k), ptr(v), B, heads, Sq, Sk, dk, qrs, krs, vrs, ptr(m), *ms,
              int(bool(causal)), scale, ptr(out), D, ptr(partials), stream_handle(dev))
    return out, partials


def absmax_partials_device(x, partials=None):
    dev = x.device
    if partials is None:
        partials = new_partials(dev)
    _lib.call("kz_absmax_f32", ptr(x), x.numel(), ptr(partials), stream_handle(dev))
    return partials


def quantize_cols_device(w):
    """Per-output-channel quantize of a [K, N] fp32 weight.
    Returns (codes [N, K] K-major, scales float64[N], scales float32[N])."""
    K, N = w.shape
    dev = w.device
    qT = torch.empty((N, K), dtype=torch.int8, device=dev)
    s64 = torch.empty(N, dtype=torch.float64, device=dev)
    s32 = torch.empty(N, dtype=torch.float32, device=dev)
    wsb = _lib.load().kz_quantize_cols_workspace_bytes(K, N)
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=dev)
    _lib.call("kz_quantize_cols_f32", ptr(w), K, N, ptr(qT), ptr(s64), ptr(s32), ptr(ws), ws.numel(),
              stream_handle(dev))
    return qT, s64, s32


def quantize_rows_device(x):
    M, K = x.shape
    dev = x.device
    q = torch.empty((M, K), dtype=torch.int8, device=dev)
    s64 = torch.empty(M, dtype=torch.float64, device=dev)
    s32 = torch.empty(M, dtype=torch.float32, device=dev)
    _lib.call("kz_quantize_rows_f32", ptr(x), M, K, ptr(q), ptr(s64), ptr(s32), stream_handle(dev))
    return q, s64, s32


def gemm_i8_device(a, b, row_scale=None, col_scale=None, bias=None, act=None, out=None, out_i32=None,
                   a_kblock=None, m=None, partials=None):
    """acc = a @ b.T on the tensor cores with the fused epilogue.
    a: int8 [M, K] (or the blocked [G, M, K/G] layout with a_kblock = K/G);
    b: int8 [N, K].  row_scale / col_scale: float32 CUDA tensors of 1 element
    (per-tensor) or M / N elements.  Returns (out_f32 or None, out_i32 or None)."""
    N, K = b.shape
    M = m if m is not None else a.shape[0]
    dev = b.device
    want_f32 = out is not None or row_scale is not None
    if want_f32 and out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
    rs_stride = 0 if row_scale is None or row_scale.numel() == 1 else 1
    cs_stride = 0 if col_scale is None or col_scale.numel() == 1 else 1
    ldo = N
    _lib.call("kz_gemm_i8", ptr(a), ptr(b), M, N, K, int(a_kblock or K), ptr(row_scale), rs_stride,
              ptr(col_scale), cs_stride, ptr(bias), _ACTS[act], ptr(out) if want_f32 else None, ptr(out_i32), ldo,
              ptr(partials), stream_handle(dev))
    return (out if want_f32 else None), out_i32


def device_status(device=None, clear=True):
    """The sticky device status word (0 = no device-side error)."""
    if device is not None:
        with torch.cuda.device(device):
            return device_status(None, clear)
    code = ctypes.c_int(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    _lib.check(_lib.load().kz_device_status(ctypes.byref(code), 1 if clear else 0, stream_handle(dev)),
               "kz_device_status")
    return code.value


# ------------------------------------------------------------ QTensor

class QActivation:
    """An activation quantized per tensor for the W8A8 path: int8 codes in the
    activation's own layout and its scale (float64 and float32, one element
    each, on the device).  ``qlinear`` accepts it in place of an fp32 input and
    skips its own quantize step, which lets the producer of the activation
    supply the absmax: a LayerNorm (``layernorm``) or the epilogue of the
    previous int8 GEMM (``from_partials``)."""

    __slots__ = ("codes", "scale64", "scale_f32")

    def __init__(self, codes, scale64, scale_f32):
        self.codes, self.scale64, self.scale_f32 = codes, scale64, scale_f32

    @property
    def shape(self):
        return list(self.codes.shape)

    @property
    def scale(self):
        return float(self.scale64.item())

    @classmethod
    def from_tensor(cls, x):
        return cls(*quantize_tensor_device(_dev_tensor(x, "QActivation")))

    @classmethod
    def from_partials(cls, x, partials):
        """x's codes from absmax partials that describe exactly x (e.g. the
        partials the GEMM that produced x wrote): one pass over x."""
        return cls(*quantize_partials_device(_dev_tensor(x, "QActivation"), partials))

    @classmethod
    def layernorm(cls, x, weight=None, bias=None, eps=1e-5):
        """LayerNorm (nn.py:308-331) of x, quantized per tensor: the LayerNorm
        kernel emits the absmax partials, so the quantize is a single pass."""
        y, partials = layernorm_partials_device(_dev_tensor(x, "QActivation.layernorm"), weight, bias, eps)
        return cls(*quantize_partials_device(y, partials))

    @classmethod
    def add_layernorm(cls, x, residual, weight=None, bias=None, eps=1e-5):
        """x + residual (a pre-LN block's residual connection, nn.py:476-477)
        and the LayerNorm of that sum quantized per tensor, from one LayerNorm
        kernel that also writes the sum.  Returns (Tensor sum, QActivation)."""
        y, partials, total = layernorm_partials_device(_dev_tensor(x, "QActivation.add_layernorm"), weight, bias,
                                                       eps, residual=_dev_tensor(residual, "QActivation.add_layernorm"))
        return Tensor(total), cls(*quantize_partials_device(y, partials))


class QTensor:
    """An int8 tensor plus its scale(s) and shape (quantize.py:80-112).

    ``granularity`` is "tensor" (one double scale, codes in the tensor's own
    row-major layout, the reference's scheme) or "channel" (one scale per
    column of a 2-D [K, N] weight, codes stored K-major [N, K] for the GEMM).
    """

    __slots__ = ("_codes", "_s64", "_s32", "_scale_host", "shape", "granularity", "_q_list", "_kmajor")

    def __init__(self, q, scale, shape, granularity=None, device=None):
        """Reference constructor: ``QTensor(q: list, scale: float, shape)``.
        ``q`` is flat and row-major in the tensor's own layout.  A list of
        scales (one per column of a 2-D [K, N] weight) makes a per-channel
        QTensor."""
        shape = [int(d) for d in shape]
        per_col = np.ndim(scale) > 0 if not isinstance(scale, torch.Tensor) else scale.numel() > 1
        self.granularity = granularity or ("channel" if per_col else "tensor")
        self.shape = shape
        arr = np.asarray(q, dtype=np.int64).reshape(shape)
        if arr.size and (arr.min() < -128 or arr.max() > 127):
            raise ValueError("QTensor: codes must fit int8")
        if self.granularity == "channel":
            if len(shape) != 2:
                raise ValueError("a per-channel QTensor is a 2-D [in, out] weight")
            arr = arr.T
        dev = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self._codes = torch.from_numpy(np.ascontiguousarray(arr.astype(np.int8))).to(dev)
        if isinstance(scale, torch.Tensor):
            self._s64 = scale.to(dev, torch.float64).reshape(-1)
        else:
            self._s64 = torch.tensor(np.atleast_1d(np.asarray(scale, np.float64)), device=dev)
        self._s32 = self._s64.to(torch.float32)
        self._scale_host = None
        self._q_list = None
        self._kmajor = None

    @classmethod
    def _from_device(cls, codes, s64, s32, shape, granularity):
        obj = cls.__new__(cls)
        obj._codes, obj._s64, obj._s32 = codes, s64, s32
        obj.shape = [int(d) for d in shape]
        obj.granularity = granularity
        obj._scale_host = None
        obj._q_list = None
        obj._kmajor = None
        return obj

    @staticmethod
    def from_tensor(tensor, per_channel=False) -> "QTensor":
        """quantize_symmetric on the device (quantize.py:96-98)."""
        x = _dev_tensor(tensor, "QTensor.from_tensor")
        if per_channel:
            if x.dim() != 2:
                raise ValueError("per-channel quantization needs a 2-D [in, out] weight")
            qT, s64, s32 = quantize_cols_device(x)
            qt = QTensor._from_device(qT, s64, s32, list(x.shape), "channel")
        else:
            q, s64, s32 = quantize_tensor_device(x)
            qt = QTensor._from_device(q, s64, s32, list(x.shape), "tensor")
        qt._check_finite()
        return qt

    def _check_finite(self):
        s = self._s64.cpu().numpy()
        if not np.all(np.isfinite(s)):
            raise ValueError("quantize_symmetric: input contains NaN or Inf")

    # ---------------------------------------------------------- accessors
    @property
    def scale(self):
        """float (per tensor) or list of floats (per channel), the exact doubles."""
        if self._scale_host is None:
            s = self._s64.cpu().numpy()
            self._scale_host = float(s[0]) if self.granularity == "tensor" else [float(v) for v in s]
        return self._scale_host

    @property
    def q(self):
        """Codes as a flat Python list in the tensor's row-major layout."""
        if self._q_list is None:
            c = self._codes.cpu().numpy()
            if self.granularity == "channel":
                c = c.T
            self._q_list = c.reshape(-1).astype(np.int64).tolist()
        return self._q_list

    @property
    def codes(self):
        """Device int8 codes: row-major like the tensor ("tensor"), or [N, K] ("channel")."""
        return self._codes

    @property
    def scale_f32(self):
        return self._s32

    @property
    def scale_f64(self):
        return self._s64

    @property
    def device(self):
        return self._codes.device

    def kmajor(self):
        """[N, K] int8 codes for the GEMM's B operand (a 2-D [K, N] weight)."""
        if self.granularity == "channel":
            return self._codes
        if self._kmajor is None:
            if len(self.shape) != 2:
                raise ValueError("only a 2-D [in, out] weight has a K-major form")
            self._kmajor = self._codes.t().contiguous()
        return self._kmajor

    def dequantize(self) -> Tensor:
        """quantize.py:100-101 -> 76-77, on the device, bit-exact."""
        dev = self._codes.device
        require_cuda(self._codes, "QTensor.dequantize")
        if self.granularity == "tensor":
            out = torch.empty(self.shape, dtype=torch.float32, device=dev)
            _lib.call("kz_dequantize_i8_f32", ptr(self._codes), self._codes.numel(), self.scale, ptr(out),
                      stream_handle(dev))
        else:
            K, N = self.shape
            out = torch.empty((K, N), dtype=torch.float32, device=dev)
            _lib.call("kz_dequantize_cols_i8_f32", ptr(self._codes), K, N, ptr(self._s64), ptr(out),
                      stream_handle(dev))
        return Tensor(out)

    def nbytes(self) -> int:
        """1 byte per element (quantize.py:103-109)."""
        return int(self._codes.numel())

    def __repr__(self):
        if self.granularity == "tensor":
            return f"QTensor(shape={self.shape}, scale={self.scale:.6g}, nbytes={self.nbytes()})"
        return f"QTensor(shape={self.shape}, per_channel=True, nbytes={self.nbytes()})"


# ------------------------------------------------------------ functions

def quantize_symmetric(tensor):
    """quantize.py:50-70: (q list[int] in [-127, 127], scale float, shape list)."""
    qt = QTensor.from_tensor(tensor)
    return qt.q, qt.scale, list(qt.shape)


def dequantize(q, scale, shape) -> Tensor:
    """quantize.py:73-77: q[i] * scale (double) narrowed to fp32, reshaped."""
    if isinstance(q, QTensor):
        return q.dequantize()
    n = int(np.prod(shape)) if len(shape) else 1
    if len(q) != n:
        raise RuntimeError("from_flat: data length does not match shape")
    return QTensor(q, float(scale), shape, granularity="tensor").dequantize()


def _flatten_rows(x):
    t = x.data if isinstance(x, Tensor) else x
    lead = list(t.shape[:-1])
    return t.reshape(-1, t.shape[-1]), lead


def qlinear(x, qweight: QTensor, bias=None, activations=None, act=None, out_partials=None) -> Tensor:
    """quantize.py:115-122: a Linear forward with an int8 weight.

    activations="fp32" (default for a per-tensor weight): the reference's
    semantics, x @ dequantize(W) + b, bit-identical (kz_qlinear_w8a32_f32).
    activations="int8" / "int8_per_row" (default "int8" for a per-channel
    weight): W8A8 on the tensor cores with the epilogue fused.
    act: optional "relu" / "gelu" applied in the same kernel (the value is the
    same as applying nn.ReLU / nn.GELU afterwards).
    x may be a QActivation (already quantized per tensor): the W8A8 GEMM then
    consumes its codes directly.  out_partials (W8A8 only): a KZ_PARTIALS_WORDS
    buffer that receives the absmax partials of the output, for
    QActivation.from_partials.
    """
    if isinstance(x, QActivation):
        codes = x.codes.reshape(-1, x.codes.shape[-1])
        M, K = codes.shape
        if len(qweight.shape) != 2 or qweight.shape[0] != K:
            raise RuntimeError("matmul: incompatible shapes")
        if K % 16:
            raise ValueError(f"W8A8 qlinear needs in_features % 16 == 0 (got {K})")
        b = _dev_tensor(bias, "qlinear bias").reshape(-1) if bias is not None else None
        out, _ = gemm_i8_device(codes, qweight.kmajor(), row_scale=x.scale_f32, col_scale=qweight.scale_f32, bias=b,
                                act=act, partials=out_partials)
        return Tensor(out.reshape(x.shape[:-1] + [qweight.shape[1]]))
    if activations is None:
        activations = "fp32" if qweight.granularity == "tensor" else "int8"
    if out_partials is not None and activations == "fp32":
        raise ValueError("out_partials needs the W8A8 path")
    xt = _dev_tensor(x, "qlinear")
    x2, lead = _flatten_rows(xt)
    x2 = x2.contiguous()
    M, K = x2.shape
    if len(qweight.shape) != 2 or qweight.shape[0] != K:
        raise RuntimeError("matmul: incompatible shapes")
    N = qweight.shape[1]
    dev = x2.device
    b = None
    if bias is not None:
        b = _dev_tensor(bias, "qlinear bias").reshape(-1)
        if b.numel() != N:
            raise RuntimeError("add: shapes are not broadcast-compatible")
    if activations == "fp32":
        if qweight.granularity != "tensor":
            raise ValueError("W8A32 qlinear needs a per-tensor weight (the reference's scheme)")
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
        _lib.call("kz_qlinear_w8a32_f32", ptr(x2), M, K, ptr(qweight.codes), qweight.scale, ptr(b), N, _ACTS[act],
                  ptr(out), stream_handle(dev))
    elif activations in ("int8", "int8_per_row"):
        if K % 16:
            raise ValueError(f"W8A8 qlinear needs in_features % 16 == 0 (got {K})")
        if activations == "int8":
            xq, _, xs32 = quantize_tensor_device(x2)
        else:
            xq, _, xs32 = quantize_rows_device(x2)
        out, _ = gemm_i8_device(xq, qweight.kmajor(), row_scale=xs32, col_scale=qweight.scale_f32, bias=b, act=act,
                                partials=out_partials)
    else:
        raise ValueError(f"unknown activations mode {activations!r}")
    return Tensor(out.reshape(lead + [N]))


class QLinear:
    """Inference-only quantized Linear built from an nn.Linear (quantize.py:125-144).

    ``QLinear(linear)`` keeps the reference's exact semantics (per-tensor
    weight, fp32 activations).  ``QLinear(linear, per_channel=True)`` is the
    W8A8 tensor-core path (per-channel weight, activations quantized per
    tensor on the fly; ``activations="int8_per_row"`` quantizes per row).
    The bias stays fp32.
    """

    def __init__(self, linear, per_channel=False, activations=None):
        self.qweight = QTensor.from_tensor(linear.weight, per_channel=per_channel)
        self.bias = as_tensor(linear.bias, device=self.qweight.device) if linear.bias is not None else None
        self.activations = activations

    def __call__(self, x, act=None, out_partials=None):
        return qlinear(x, self.qweight, self.bias, activations=self.activations, act=act, out_partials=out_partials)

    def forward(self, x, act=None):
        return self(x, act)

    @property
    def in_features(self):
        return self.qweight.shape[0]

    @property
    def out_features(self):
        return self.qweight.shape[1]

    def parameters(self):
        return []

    def __repr__(self):
        return f"QLinear({self.in_features}, {self.out_features}, {self.qweight.granularity})"


def scale_of(max_abs: float) -> float:
    """quantize.py:68."""
    return max_abs / 127.0 if max_abs > 0.0 else 1.0


__all__ = ["quantize_symmetric", "dequantize", "QTensor", "qlinear", "QLinear", "scale_of"]
