"""GPU parity for config 3: the int8 2-layer decoder (d_model 256, 4 heads,
FFN 1024 with GELU, vocab 65, context 256, batch 32 = 8192 tokens), every
Linear per-channel int8 with per-tensor int8 activations; LayerNorm, attention
and softmax fp32.

1. Layer by layer: every quantized Linear call inside the forward is redone
   by the oracle from the input that layer received on the device (fp32, or
   int8 codes + scale when the producer quantized it).  The activation codes
   and scale, the int32 accumulators (sampled rows) and the fp32 outputs must
   be bit-exact (GELU layers: 1e-5 relative, CUDA erff).  fc2's input codes,
   quantized from the absmax partials of fc1's epilogue, must equal the
   oracle's per-tensor quantize of fc1's output exactly.
2. End to end: the logits are compared with an fp32 numpy forward that runs
   every Linear through the oracle.  LayerNorm and softmax reduce in a
   different order in numpy and torch, so an activation lying on a rounding
   boundary can quantize one code apart; the logits must agree to 2e-3
   relative (Frobenius) and in at least 99% of the argmax tokens.
"""
import math

import numpy as np
import pytest
import torch

from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu

ACTS = {None: 0, "relu": 1, "gelu": 2}


@pytest.fixture(scope="module")
def model_and_ids(cuda_device):
    from kansaiml_b200 import workloads
    torch.manual_seed(0)
    return workloads.Decoder(seed=3), workloads.config3_ids(seed=4)


def test_layerwise_bit_exact(model_and_ids, monkeypatch):
    from kansaiml_b200 import quantize as kq
    model, ids = model_and_ids
    calls = []
    inner = kq.qlinear

    def recording(x, qweight, bias=None, activations=None, act=None, out_partials=None):
        out = inner(x, qweight, bias, activations=activations, act=act, out_partials=out_partials)
        K = qweight.shape[0]
        if isinstance(x, kq.QActivation):
            xin = (x.codes.cpu().numpy().reshape(-1, K), x.scale)
        else:
            xin = x.numpy().reshape(-1, K)
        calls.append((xin, qweight, bias, act, out.numpy()))
        return out

    monkeypatch.setattr(kq, "qlinear", recording)
    model(ids)
    # per block: fused qkv, output projection, fc1, fc2; then the head
    assert len(calls) == 2 * 4 + 1
    rows = np.random.RandomState(0).choice(ids.numel(), 128, replace=False)
    for i, (x, qw, bias, act, y) in enumerate(calls):
        wq = qw.codes.cpu().numpy()
        ws = qw.scale_f32.cpu().numpy()
        if isinstance(x, tuple):
            xq, xs = x
            if i > 0 and calls[i - 1][3] == "gelu":   # fc2: codes from fc1's epilogue partials
                xq_o, xs_o = ocpu.quantize_tensor(calls[i - 1][4].reshape(xq.shape))
                assert xs == xs_o, f"call {i}"
                np.testing.assert_array_equal(xq, xq_o, err_msg=f"call {i}")
        else:
            xq, xs = ocpu.quantize_tensor(x)
        acc = ocpu.gemm_i8(xq[rows], wq)
        b = bias.numpy() if bias is not None else None
        yo = ocpu.epilogue(acc, xs, ws, b, ACTS[act])
        yg = y.reshape(-1, wq.shape[0])[rows]
        if act == "gelu":
            np.testing.assert_allclose(yg, yo, rtol=1e-5, atol=1e-6, err_msg=f"call {i}")
        else:
            assert yg.tobytes() == yo.tobytes(), f"call {i}"


def test_layernorm_quantize_vs_oracle(cuda_device):
    """QActivation.layernorm (LayerNorm kernel + absmax partials + one quantize
    pass) against numpy LayerNorm + the oracle's quantize: the scale within
    1e-6 relative, the codes equal except where the two fp32 LayerNorms land
    on opposite sides of a rounding boundary (then one code apart, rarely)."""
    import kansaiml_b200 as kz
    from kansaiml_b200 import quantize as kq
    rs = np.random.RandomState(8)
    x = (rs.standard_normal((4096, 256)) * 3 + 1).astype(np.float32)
    g = rs.uniform(0.5, 1.5, 256).astype(np.float32)
    b = rs.standard_normal(256).astype(np.float32) * 0.1
    qa = kq.QActivation.layernorm(kz.from_numpy(x), kz.from_numpy(g), kz.from_numpy(b), 1e-5)
    ln = _ln(x) * g + b
    q_o, s_o = ocpu.quantize_tensor(ln.astype(np.float32))
    assert abs(qa.scale - s_o) <= 1e-6 * s_o
    codes = qa.codes.cpu().numpy()
    diff = np.abs(codes.astype(np.int32) - q_o.reshape(codes.shape).astype(np.int32))
    assert diff.max() <= 1
    assert (diff != 0).mean() <= 1e-3


def test_block_forward_matches_the_unfused_composition(model_and_ids):
    """A quantized TransformerBlock's forward (residual adds folded into the
    LayerNorms) equals the same block composed from separate adds and
    LayerNorms, bit for bit."""
    from kansaiml_b200 import quantize as kq
    from kansaiml_b200.tensor import Tensor
    model, ids = model_and_ids
    blk, mask = model.blocks[0], model.mask
    x = Tensor(model.tok.weight.data[ids] + model.pos.weight.data[: ids.shape[1]])
    y = blk(x, mask=mask).data
    ln1, ln2 = blk.ln1, blk.ln2
    qa = kq.QActivation.layernorm(x, ln1.weight, ln1.bias, ln1.eps)
    x1 = x.add(blk.attn(qa, qa, qa, mask=mask))
    qb = kq.QActivation.layernorm(x1, ln2.weight, ln2.bias, ln2.eps)
    parts = kq.new_partials(x.data.device)
    h = blk.fc1(qb, act="gelu", out_partials=parts)
    ref = x1.add(blk.fc2(kq.QActivation.from_partials(h, parts))).data
    assert torch.equal(y, ref)


def test_add_layernorm_equals_add_then_layernorm(cuda_device):
    """kz_add_layernorm_partials_f32 (the residual add folded into the
    LayerNorm that follows it) against torch's add followed by the plain
    LayerNorm kernel: the sum, the normalised output, the codes and the scale
    are bit-identical."""
    import kansaiml_b200 as kz
    from kansaiml_b200 import quantize as kq
    rs = np.random.RandomState(12)
    x = (rs.standard_normal((1000, 256)) * 2).astype(np.float32)
    r = rs.standard_normal((1000, 256)).astype(np.float32)
    g = rs.uniform(0.5, 1.5, 256).astype(np.float32)
    b = rs.standard_normal(256).astype(np.float32) * 0.1
    xt, rt, gt, bt = (kz.from_numpy(a) for a in (x, r, g, b))
    total, qa = kq.QActivation.add_layernorm(xt, rt, gt, bt, 1e-5)
    plain_sum = xt.data + rt.data
    y_ref, parts = kq.layernorm_partials_device(plain_sum, gt, bt, 1e-5, partials=kq.new_partials(plain_sum.device))
    q_ref = kq.QActivation.from_partials(kz.Tensor(y_ref), parts)
    assert torch.equal(total.data, plain_sum)
    assert torch.equal(qa.codes, q_ref.codes) and qa.scale == q_ref.scale


def test_causal_flag_matches_the_explicit_mask(cuda_device):
    """causal_mask() reaches attention as is_causal.  Its -1e9 entries give
    weight exactly 0 (every row keeps its own position, so the shifted
    exponentials underflow), so the result agrees with the explicit mask's to
    fp32 rounding."""
    from kansaiml_b200 import nn as knn
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    q, k, v = (torch.randn((4, 4, 256, 64), device="cuda", generator=g) for _ in range(3))
    mask = knn.causal_mask(256, device="cuda")
    assert getattr(mask, "causal", False)
    sdpa = torch.nn.functional.scaled_dot_product_attention
    flagged = sdpa(q, k, v, is_causal=True)
    explicit = sdpa(q, k, v, attn_mask=mask.data)
    torch.testing.assert_close(flagged, explicit, rtol=1e-5, atol=1e-6)


def _ln(x, eps=1e-5):
    mean = x.mean(-1, keepdims=True, dtype=np.float32)
    c = x - mean
    var = (c * c).mean(-1, keepdims=True, dtype=np.float32)
    return (c / np.sqrt(var + np.float32(eps))).astype(np.float32)


def _linear(x, w, bias=None, act=0):
    shape = x.shape
    wq, ws = ocpu.quantize_cols(w)
    y, _, _, _ = ocpu.w8a8_linear(x.reshape(-1, shape[-1]), wq, ws, bias, act)
    return y.reshape(shape[:-1] + (w.shape[1],))


def _attention(h, w, heads, mask):
    b, s, d = h.shape
    dk = d // heads

    def split(t):
        return t.reshape(b, s, heads, dk).transpose(0, 2, 1, 3)

    q, k, v = (split(_linear(h, w[n])) for n in ("w_q", "w_k", "w_v"))
    scores = np.matmul(q, k.transpose(0, 1, 3, 2)) * np.float32(1.0 / math.sqrt(dk)) + mask
    scores = scores - scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(-1, keepdims=True)
    att = np.matmul(p, v).transpose(0, 2, 1, 3).reshape(b, s, d)
    return _linear(np.ascontiguousarray(att, dtype=np.float32), w["w_o"])


def test_end_to_end_vs_oracle(model_and_ids):
    model, ids = model_and_ids
    logits = model(ids).numpy()
    f = model.fp32
    idn = ids.cpu().numpy()
    s = idn.shape[1]
    x = (f["tok"][idn] + f["pos"][:s]).astype(np.float32)
    mask = np.triu(np.full((s, s), -1e9, np.float32), 1)
    for w in f["blocks"]:
        h = _ln(x)
        x = x + _attention(h, w, model.heads, mask)
        h = _ln(x)
        h = _linear(h, w["fc1"], w["fc1_b"], act=2)
        x = x + _linear(h, w["fc2"], w["fc2_b"])
    ref = _linear(_ln(x), f["head"], f["head_b"])
    rel = np.linalg.norm(logits - ref) / np.linalg.norm(ref)
    agree = (logits.argmax(-1) == ref.argmax(-1)).mean()
    assert rel <= 2e-3, rel
    assert agree >= 0.99, agree
