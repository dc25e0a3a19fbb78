"""GPU parity of kz_attention_f32, the fp32 attention core between config 3's
int8 projections.

The kernel takes the reference's own operation order (MultiHeadAttention.forward,
nn.py:410-423, composed from Tensor ops: ordered dot products without FMA,
scale, mask, row max, exp, ordered sum, reciprocal, ordered weighted sum of v)
and rounds exp correctly from a double exp.  So it must equal the oracle's
restatement with that exp (`exp="rn"`) bit for bit; the oracle with the host's
expf equals the reference's own forward bit for bit (tests/test_oracle_golden.py),
and the two exps differ only on near-midpoint inputs.
"""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(q, k, v, heads, mask=None, causal=False):
    from kansaiml_b200 import quantize as kq
    parts = kq.new_partials(torch.device("cuda"))
    m = _dev(mask) if mask is not None else None
    y, parts = kq.attention_device(_dev(q), _dev(k), _dev(v), heads, mask=m, causal=causal, partials=parts)
    torch.cuda.synchronize()
    return y.cpu().numpy(), parts.cpu().numpy()


def _check_partials(y, parts):
    count = int(parts[0])
    assert 1 <= count <= 1021
    absmax = np.abs(y).max() if y.size else np.float32(0)
    assert parts[1:1 + count].astype(np.uint32).max() == np.float32(absmax).view(np.uint32)


def test_golden_cases_bit_exact(cuda_device):
    """Every golden case (causal, broadcast additive mask, none; d_k 32 / 64 /
    128; rows and keys across the 64-wide tiles): the kernel equals the
    oracle's reference-order restatement bit for bit, and differs from the
    reference's own output exactly where that oracle does."""
    g = golden("attention_cases.npz")
    for i, (B, Sq, Sk, D, H, kind) in enumerate(inputs.ATTENTION_CASES):
        q, k, v, mask = inputs.attention_inputs(i)
        causal = kind == "causal"
        y, parts = _run(q, k, v, H, mask=None if causal else mask, causal=causal)
        y_o = ocpu.attention(q, k, v, H, mask=None if causal else mask, causal=causal, exp="rn")
        assert y.tobytes() == y_o.tobytes(), i
        ref = g[f"c{i}__y"]
        np.testing.assert_array_equal(y.view(np.int32) != ref.view(np.int32),
                                      y_o.view(np.int32) != ref.view(np.int32), err_msg=str(i))
        _check_partials(y, parts)
        if causal:   # the explicit -1e9 mask gives the same bits as the flag
            y_m, _ = _run(q, k, v, H, mask=mask)
            assert y_m.tobytes() == y.tobytes(), i


def test_config3_fused_qkv_layout_bit_exact(cuda_device):
    """Config 3's shape (batch 32, context 256, d_model 256, 4 heads, causal),
    with q, k and v read as strided slices of one [b, s, 3d] projection
    output, as the model runs it."""
    from kansaiml_b200 import quantize as kq
    B, S, D, H = 32, 256, 256, 4
    rs = np.random.RandomState(31)
    qkv = (rs.standard_normal((B, S, 3 * D)) * 1.5).astype(np.float32)
    t = _dev(qkv)
    parts = kq.new_partials(t.device)
    y, parts = kq.attention_device(t[:, :, :D], t[:, :, D:2 * D], t[:, :, 2 * D:], H, causal=True, partials=parts)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    y_o = ocpu.attention(qkv[:, :, :D], qkv[:, :, D:2 * D], qkv[:, :, 2 * D:], H, causal=True, exp="rn")
    assert y.tobytes() == y_o.tobytes()
    _check_partials(y, parts.cpu().numpy())


@pytest.mark.parametrize("B,Sq,Sk,D,H", [(2, 130, 300, 128, 1), (3, 1, 65, 96, 3), (1, 200, 7, 256, 4)])
def test_cross_attention_masked_ragged(cuda_device, B, Sq, Sk, D, H):
    """Cross-attention (seq_q != seq_k) with a per-batch additive mask, ragged
    lengths on both sides of the 64-wide tiles, a single query row."""
    rs = np.random.RandomState(B * 1000 + Sq + Sk)
    q = rs.standard_normal((B, Sq, D)).astype(np.float32) * 2
    k = rs.standard_normal((B, Sk, D)).astype(np.float32) * 2
    v = rs.standard_normal((B, Sk, D)).astype(np.float32)
    mask = (rs.uniform(-4, 0, (B, 1, Sq, Sk)) * (rs.uniform(size=(B, 1, Sq, Sk)) < 0.4)).astype(np.float32)
    y, parts = _run(q, k, v, H, mask=mask)
    assert y.tobytes() == ocpu.attention(q, k, v, H, mask=mask, exp="rn").tobytes()
    _check_partials(y, parts)


def test_rejects_what_it_does_not_cover(cuda_device):
    """Head widths other than 32 / 64 / 128, causal with seq_q != seq_k and key
    counts past the on-chip score rows raise instead of computing."""
    from kansaiml_b200 import _lib
    from kansaiml_b200 import quantize as kq
    x = torch.zeros((1, 8, 48), device="cuda")
    with pytest.raises(RuntimeError, match="d_k"):
        kq.attention_device(x, x, x, 1)
    q, kv = torch.zeros((1, 8, 64), device="cuda"), torch.zeros((1, 9, 64), device="cuda")
    with pytest.raises(RuntimeError, match="causal"):
        kq.attention_device(q, kv, kv, 1, causal=True)
    limit = next(s for s in range(64, 4096, 64) if _lib.load().kz_attention_smem_bytes(s + 1, 64) == 0)
    long_kv = torch.zeros((1, limit + 1, 64), device="cuda")
    with pytest.raises(RuntimeError, match="seq_k"):
        kq.attention_device(q, long_kv, long_kv, 1)
    y, _ = kq.attention_device(torch.zeros((0, 8, 64), device="cuda"), kv[:0], kv[:0], 1)
    assert y.shape == (0, 8, 64)


def test_module_cross_attention_uses_the_kernel(cuda_device):
    """MultiHeadAttention.forward with distinct query and key/value inputs
    (fp32 projections): the attention between them is the kernel's, so it
    equals the oracle's core run on the device's own projections."""
    from kansaiml_b200 import nn as knn
    from kansaiml_b200.tensor import Tensor
    mha = knn.MultiHeadAttention(128, 2, seed=4, device="cuda")
    rs = np.random.RandomState(8)
    xq = Tensor(_dev(rs.standard_normal((2, 40, 128)).astype(np.float32)))
    xkv = Tensor(_dev(rs.standard_normal((2, 70, 128)).astype(np.float32)))
    inner = {}
    from kansaiml_b200 import quantize as kq
    orig = knn.attention_device

    def spy(q, k, v, heads, mask=None, causal=False, partials=None):
        out = orig(q, k, v, heads, mask=mask, causal=causal, partials=partials)
        inner["qkv"] = (q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy())
        inner["y"] = out[0].cpu().numpy()
        return out

    knn.attention_device = spy
    try:
        mha(xq, xkv, xkv)
    finally:
        knn.attention_device = orig
    q, k, v = inner["qkv"]
    assert inner["y"].tobytes() == ocpu.attention(q, k, v, 2, exp="rn").tobytes()
    assert kq.device_status() == 0
