"""Seeded synthetic models and inputs for the benchmark configurations, shared
by bench.py and the tests (no datasets or checkpoints are involved).

Config 3 is an int8 decoder-only transformer with the layout of the
reference's examples/tinyshakespeare/train_shakespeare.py:79-111 (token +
learned position embeddings, pre-LN TransformerBlocks under one causal mask,
final LayerNorm, Linear head): d_model 256, 4 heads, FFN 1024 with GELU,
vocab 65, context 256, 2 blocks.  Every Linear weight is drawn ~ N(0, 0.02)
from a seeded numpy stream and quantized per output channel; activations are
quantized per tensor on the fly (W8A8 on the int8 tensor cores, bias, GELU
and rescale fused); LayerNorm, attention scores and softmax stay fp32.
"""
import numpy as np
import torch

from . import nn
from .quantize import QActivation, QLinear
from .tensor import Tensor, from_numpy


def _param(a, device):
    t = from_numpy(a, device)
    t.requires_grad = True
    return t


class Decoder(nn.Module):
    """Config 3 decoder.  ``fp32`` keeps the unquantized weights (numpy) so a
    CPU restatement can rebuild the same model."""

    def __init__(self, vocab=65, d_model=256, heads=4, d_ff=1024, layers=2, ctx=256, seed=0, device="cuda"):
        rs = np.random.RandomState(seed)

        def normal(*shape):
            return (rs.standard_normal(shape) * 0.02).astype(np.float32)

        self.vocab, self.d_model, self.heads, self.ctx = vocab, d_model, heads, ctx
        self.tok = nn.Embedding(vocab, d_model, seed=seed, device=device)
        self.pos = nn.Embedding(ctx, d_model, seed=seed + 1, device=device)
        self.fp32 = {"tok": self.tok.weight.numpy(), "pos": self.pos.weight.numpy(), "blocks": []}
        self.blocks = []
        for i in range(layers):
            blk = nn.TransformerBlock(d_model, heads, d_ff, seed=seed + 10 + i, device=device)
            w = {name: normal(d_model, d_model) for name in ("w_q", "w_k", "w_v", "w_o")}
            for name, value in w.items():
                setattr(blk.attn, name, _param(value, device))
            w["fc1"], w["fc2"] = normal(d_model, d_ff), normal(d_ff, d_model)
            blk.fc1.weight = _param(w["fc1"], device)
            blk.fc2.weight = _param(w["fc2"], device)
            w["fc1_b"], w["fc2_b"] = blk.fc1.bias.numpy(), blk.fc2.bias.numpy()
            blk.quantize(per_channel=True, activations="int8")
            self.blocks.append(blk)
            self.fp32["blocks"].append(w)
        self.ln = nn.LayerNorm(d_model, device=device)
        head = nn.Linear(d_model, vocab, seed=seed + 99, device=device)
        self.fp32["head"], self.fp32["head_b"] = normal(d_model, vocab), head.bias.numpy()
        head.weight = _param(self.fp32["head"], device)
        self.head = QLinear(head, per_channel=True, activations="int8")
        self.mask = nn.causal_mask(ctx, device=device)

    def forward(self, ids):
        """ids: int64 [B, S] (S <= ctx) on the model's device -> logits [B, S, vocab]."""
        s = ids.shape[1]
        x = Tensor(self.tok.weight.data[ids] + self.pos.weight.data[:s])
        mask = self.mask if s == self.ctx else nn.CausalMask(self.mask.data[:, :, :s, :s].contiguous())
        # each block's feed-forward residual is added inside the next LayerNorm
        pending = None
        for blk in self.blocks:
            if blk._w8a8():
                x, pending = blk._forward_w8a8(x, mask, pending)
            else:
                x = blk(x if pending is None else x.add(pending), mask=mask)
                pending = None
        ln = self.ln
        if pending is None:
            qa = QActivation.layernorm(x, ln.weight, ln.bias, ln.eps)
        else:
            _, qa = QActivation.add_layernorm(x, pending, ln.weight, ln.bias, ln.eps)
        return self.head(qa)


def config3_ids(batch=32, ctx=256, vocab=65, seed=0, device="cuda"):
    """Token ids ~ U{0 .. vocab-1}, int64 [batch, ctx]."""
    ids = np.random.RandomState(seed).randint(0, vocab, (batch, ctx))
    return torch.from_numpy(ids.astype(np.int64)).to(device)
