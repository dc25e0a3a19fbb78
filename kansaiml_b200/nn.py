"""Model hosts for the quantized path, with the reference's nn names (python/kansai/nn.py).

Only the layers the int8 configurations need: Linear (nn.py:74-81, weight
[in, out] with std 1/sqrt(in) from the reference's own randn stream, zero
bias), ReLU / GELU (nn.py:216-218 and the exact-erf GELU), Sequential
(nn.py:649-656), and the transformer pieces of config 3 (LayerNorm nn.py:308-331,
MultiHeadAttention nn.py:334-427, TransformerBlock nn.py:430-478, Embedding
nn.py:624-646).  Inference only: no autograd.

Sequential fuses ``QLinear`` followed by ``ReLU`` / ``GELU`` into the
quantized kernel's epilogue; the activation is applied to the same fp32 value,
so the result equals running the two layers one after the other.
"""
import math

import torch

from .quantize import QActivation, QLinear, attention_device, layernorm_partials_device, partials_buffer
from .tensor import Tensor, as_tensor, from_flat, ones, randn, zeros


class Module:
    training = False

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    def named_parameters(self, prefix=""):
        """nn.py:19-39: (dotted name, Tensor) for every trainable parameter
        (requires_grad), recursing into sub-Modules and lists of them."""
        for name, value in vars(self).items():
            full = f"{prefix}{name}"
            if isinstance(value, Tensor) and value.requires_grad:
                yield full, value
            elif isinstance(value, Module):
                yield from value.named_parameters(full + ".")
            elif isinstance(value, (list, tuple)):
                for i, item in enumerate(value):
                    if isinstance(item, Module):
                        yield from item.named_parameters(f"{full}.{i}.")

    def parameters(self):
        return [t for _, t in self.named_parameters()]

    def eval(self):
        return self


class Linear(Module):
    """nn.py:74-81: weight [in, out] ~ N(0, 1/in) from randn(seed), bias zeros."""

    def __init__(self, in_features, out_features, seed=0, device=None):
        std = 1.0 / math.sqrt(in_features)
        self.weight = randn([in_features, out_features], std=std, requires_grad=True, seed=seed, device=device)
        self.bias = zeros([out_features], requires_grad=True, device=device)

    def forward(self, x):
        return as_tensor(x).matmul(self.weight).add(self.bias)


class ReLU(Module):
    def forward(self, x):
        return as_tensor(x).relu()


class GELU(Module):
    def forward(self, x):
        return as_tensor(x).gelu()


_FUSABLE = {ReLU: "relu", GELU: "gelu"}


class Sequential(Module):
    def __init__(self, *layers):
        self.layers = list(layers)

    def forward(self, x):
        i, n = 0, len(self.layers)
        while i < n:
            layer = self.layers[i]
            nxt = self.layers[i + 1] if i + 1 < n else None
            if isinstance(layer, QLinear) and type(nxt) in _FUSABLE:
                x = layer(x, act=_FUSABLE[type(nxt)])
                i += 2
                continue
            x = layer(x)
            i += 1
        return x


class LayerNorm(Module):
    """nn.py:308-331: normalises the last axis, biased variance, eps 1e-5.
    The forward runs libkz's LayerNorm kernel, which follows the reference's
    operation order (ordered fp32 sums, mul by the reciprocal), so the output
    equals the reference's bit for bit."""

    def __init__(self, num_features, eps=1e-5, device=None):
        self.num_features = num_features
        self.eps = eps
        self.weight = ones([num_features], requires_grad=True, device=device)
        self.bias = zeros([num_features], requires_grad=True, device=device)

    def forward(self, x):
        t = as_tensor(x).data
        if t.shape[-1] != self.num_features:
            raise RuntimeError("mul: shapes are not broadcast-compatible")
        y, _ = layernorm_partials_device(t.contiguous(), self.weight, self.bias, self.eps)
        return Tensor(y)


class Embedding(Module):
    """nn.py:624-646: weight [vocab, dim] ~ N(0, 1) from randn(seed); forward
    takes (nested) integer ids."""

    def __init__(self, num_embeddings, embedding_dim, seed=0, device=None):
        self.weight = randn([num_embeddings, embedding_dim], std=1.0, requires_grad=True, seed=seed, device=device)

    def forward(self, ids):
        idx = ids if isinstance(ids, torch.Tensor) else torch.as_tensor(ids, dtype=torch.long)
        idx = idx.to(self.weight.data.device)
        return Tensor(self.weight.data[idx])


class MultiHeadAttention(Module):
    """nn.py:334-427: raw [d, d] projections w_q, w_k, w_v, w_o (no bias),
    scaled dot-product attention with an optional additive mask, fp32.
    ``quantize(per_channel=True)`` swaps the four projections for int8 QLinear
    layers (bias-free); attention scores and softmax stay fp32.  With a
    per-channel weight, self-attention (query, key and value the same input)
    runs the three input projections as ONE int8 GEMM over the concatenated
    [d, 3d] weight: per-channel codes and scales are per column, so each
    column is the same as its separate projection's, bit for bit.  The
    attention between the projections is one kz_attention_f32 kernel that
    takes the reference's own operation order (scores, scale, mask, max, exp,
    ordered sum, reciprocal, ordered weighted sum of v, nn.py:410-423)."""

    def __init__(self, d_model, num_heads, seed=0, device=None):
        if d_model % num_heads:
            raise ValueError(f"MultiHeadAttention: d_model={d_model} must be divisible by num_heads={num_heads}")
        self.d_model, self.num_heads, self.d_k = d_model, num_heads, d_model // num_heads
        std = 1.0 / math.sqrt(d_model)
        self.w_q = randn([d_model, d_model], std=std, requires_grad=True, seed=seed, device=device)
        self.w_k = randn([d_model, d_model], std=std, requires_grad=True, seed=seed + 1, device=device)
        self.w_v = randn([d_model, d_model], std=std, requires_grad=True, seed=seed + 2, device=device)
        self.w_o = randn([d_model, d_model], std=std, requires_grad=True, seed=seed + 3, device=device)
        self.q_proj = None
        self.qkv = None

    def quantize(self, per_channel=True, activations=None):
        class _W:  # a Linear-shaped view of a bias-free projection
            def __init__(self, w):
                self.weight, self.bias = w, None
        self.q_proj = [QLinear(_W(w), per_channel=per_channel, activations=activations)
                       for w in (self.w_q, self.w_k, self.w_v, self.w_o)]
        if per_channel and activations in (None, "int8"):
            qkv = torch.cat([self.w_q.data, self.w_k.data, self.w_v.data], dim=1)
            self.qkv = QLinear(_W(Tensor(qkv)), per_channel=True, activations=activations)
        return self

    def _proj(self, x, i, w):
        if self.q_proj is not None:
            return self.q_proj[i](x)
        return x.matmul(w)

    def forward(self, query, key, value, mask=None):
        if self.qkv is not None and query is key and key is value:
            return self._self_attention(query, mask)
        if isinstance(query, QActivation):
            raise ValueError("a pre-quantized input needs the fused self-attention path")
        q_in, k_in, v_in = as_tensor(query), as_tensor(key), as_tensor(value)
        q = self._proj(q_in, 0, self.w_q).data
        k = self._proj(k_in, 1, self.w_k).data
        v = self._proj(v_in, 2, self.w_v).data
        causal = self._causal(mask, q.shape[1], k.shape[1])
        m = as_tensor(mask).data if mask is not None and not causal else None
        att, _ = attention_device(q, k, v, self.num_heads, mask=m, causal=causal)
        return self._proj(Tensor(att), 3, self.w_o)

    @staticmethod
    def _causal(mask, sq, sk):
        """A causal_mask() of exactly this (query, key) length goes to the
        kernel as the causal flag; any other mask is added to the scores as
        given, so a wrong-sized one fails to broadcast, as the reference's
        scores.add(mask) does."""
        return (getattr(mask, "causal", False) and sq == sk
                and tuple(as_tensor(mask).shape[-2:]) == (sq, sk))


    def _self_attention(self, x, mask):
        """One int8 GEMM for q, k and v; the fp32 attention kernel reads q, k
        and v straight out of its [b, s, 3d] output and writes the heads-merged
        result with its absmax partials, so the int8 output projection's
        quantize is a single pass.  A causal_mask() goes to the kernel as the
        causal flag: keys past each query get weight 0, exactly what its -1e9
        entries give (their exponentials are 0), without reading the mask or
        the key tiles past the diagonal."""
        b, s, _ = x.shape
        d = self.d_model
        qkv = self.qkv(x).data.reshape(b, s, 3 * d)
        causal = self._causal(mask, s, s)
        m = as_tensor(mask).data if mask is not None and not causal else None
        att, partials = attention_device(qkv[:, :, :d], qkv[:, :, d:2 * d], qkv[:, :, 2 * d:], self.num_heads,
                                         mask=m, causal=causal)
        return self.q_proj[3](QActivation.from_partials(att, partials))


class TransformerBlock(Module):
    """nn.py:430-478: pre-LN attention and GELU feed-forward, both residual."""

    def __init__(self, d_model, num_heads, d_ff, seed=0, device=None):
        self.ln1 = LayerNorm(d_model, device=device)
        self.attn = MultiHeadAttention(d_model, num_heads, seed=seed, device=device)
        self.ln2 = LayerNorm(d_model, device=device)
        self.fc1 = Linear(d_model, d_ff, seed=seed + 100, device=device)
        self.gelu = GELU()
        self.fc2 = Linear(d_ff, d_model, seed=seed + 101, device=device)

    def quantize(self, per_channel=True, activations=None):
        """Every Linear weight to int8 (fc1, fc2 and the four attention projections)."""
        self.attn.quantize(per_channel, activations)
        self.fc1 = QLinear(self.fc1, per_channel=per_channel, activations=activations)
        self.fc2 = QLinear(self.fc2, per_channel=per_channel, activations=activations)
        return self

    def _w8a8(self):
        return isinstance(self.fc1, QLinear) and self.attn.qkv is not None

    def forward(self, x, mask=None):
        x = as_tensor(x)
        if self._w8a8():
            x, pending = self._forward_w8a8(x, mask)
            return x.add(pending)
        normed = self.ln1(x)
        x = x.add(self.attn(normed, normed, normed, mask=mask))
        h = self.ln2(x)
        if isinstance(self.fc1, QLinear):
            h = self.fc1(h, act="gelu")
        else:
            h = self.gelu(self.fc1(h))
        return x.add(self.fc2(h))

    def _forward_w8a8(self, x, mask, pending=None):
        """The same block with every activation quantized where it is made:
        LayerNorm -> quantize is one LayerNorm kernel (with the absmax) plus
        one quantize pass; fc1's GEMM epilogue (bias + GELU) also emits the
        absmax of its output, so fc2's input is quantized in one pass.  The
        residual adds are folded into the LayerNorm that follows each one: the
        block's input is x + pending (pending None: x), and it returns
        (x, pending) with its output x + pending, for the next LayerNorm to
        add."""
        ln1, ln2 = self.ln1, self.ln2
        if pending is None:
            qa = QActivation.layernorm(x, ln1.weight, ln1.bias, ln1.eps)
        else:
            x, qa = QActivation.add_layernorm(x, pending, ln1.weight, ln1.bias, ln1.eps)
        x, qb = QActivation.add_layernorm(x, self.attn(qa, qa, qa, mask=mask), ln2.weight, ln2.bias, ln2.eps)
        partials = partials_buffer(x.data.device)
        h = self.fc1(qb, act="gelu", out_partials=partials)
        return x, self.fc2(QActivation.from_partials(h, partials))


class CausalMask(Tensor):
    """A mask tensor known to be causal_mask()'s (or a leading square slice of
    one): attention passes it on as the kernel's causal flag instead of
    reading it."""
    __slots__ = ()
    causal = True


def causal_mask(seq, device=None):
    """Additive causal mask [1, 1, seq, seq] (0 allowed, -1e9 masked), the
    convention of examples/tinyshakespeare/train_shakespeare.py:96-97."""
    vals = torch.full((seq, seq), -1e9, dtype=torch.float32).triu(1)
    return CausalMask(from_flat(vals.reshape(-1).tolist(), [1, 1, seq, seq], device=device).data)
