"""Host-side API of kansaiml_b200 on CPU (data movement only, no compute):
the reference's Tensor surface, factories and error behaviour."""
import numpy as np
import pytest

import kansaiml_b200 as kz


def test_from_flat_tolist_roundtrip():
    t = kz.from_flat([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], [2, 3], device="cpu")
    assert t.shape == [2, 3] and t.numel() == 6
    assert t.tolist() == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    with pytest.raises(RuntimeError, match="data length does not match shape"):
        kz.from_flat([1.0, 2.0], [3], device="cpu")


def test_tensor_nested_list():
    t = kz.tensor([[0, 0], [0, 1], [1, 0], [1, 1]], device="cpu")
    assert t.shape == [4, 2]
    assert t.tolist() == [0.0, 0.0, 0.0, 1.0, 1.0, 0.0, 1.0, 1.0]


def test_slice_and_cat():
    vals = np.arange(28, dtype=np.float32)
    t = kz.from_flat(vals, [7, 4], device="cpu")
    a, b = t.slice(0, 0, 3), t.slice(0, 3, 7)
    assert a.shape == [3, 4] and b.shape == [4, 4]
    assert kz.cat([a, b], 0).tolist() == vals.tolist()
    with pytest.raises(RuntimeError):
        t.slice(0, 5, 9)


def test_linear_init_matches_reference_hash():
    import inputs
    from conftest import golden
    g = golden("mlp_config1.npz")
    l1 = kz.nn.Linear(784, 256, seed=1, device="cpu")
    l2 = kz.nn.Linear(256, 10, seed=2, device="cpu")
    assert inputs.sha(l1.weight.numpy()) == str(g["w1_sha256"])
    assert inputs.sha(l2.weight.numpy()) == str(g["w2_sha256"])
    assert l1.bias.tolist() == [0.0] * 256


def test_compute_on_cpu_tensor_fails_loudly():
    from kansaiml_b200.quantize import QTensor
    t = kz.from_flat([1.0, 2.0], [2], device="cpu")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        QTensor.from_tensor(t)


def test_qtensor_reference_constructor_and_nbytes():
    from kansaiml_b200.quantize import QTensor
    q = QTensor([1, -2, 3, 127], 0.5, [2, 2], device="cpu")
    assert q.q == [1, -2, 3, 127]
    assert q.scale == 0.5 and q.shape == [2, 2] and q.nbytes() == 4
    with pytest.raises(ValueError):
        QTensor([300], 1.0, [1], device="cpu")
    pc = QTensor([1, 2, 3, 4, 5, 6], [0.1, 0.2, 0.3], [2, 3], device="cpu")
    assert pc.granularity == "channel"
    assert pc.codes.shape == (3, 2)          # stored K-major [N, K]
    assert pc.q == [1, 2, 3, 4, 5, 6]         # read back in the [K, N] layout
    assert pc.scale == [0.1, 0.2, 0.3]


def test_causal_mask_values_and_marker():
    """causal_mask(seq) holds the reference's additive causal mask (0 on and
    below the diagonal, -1e9 above it; train_shakespeare.py:96-97) and carries
    the causal marker the fused self-attention keys on; a plain Tensor of the
    same values does not."""
    from kansaiml_b200 import nn
    m = nn.causal_mask(5, device="cpu")
    assert getattr(m, "causal", False) and isinstance(m, kz.Tensor)
    assert m.shape == [1, 1, 5, 5]
    want = np.triu(np.full((5, 5), -1e9, np.float32), 1)
    np.testing.assert_array_equal(np.asarray(m.tolist(), np.float32).reshape(5, 5), want)
    assert not getattr(kz.Tensor(m.data.clone()), "causal", False)


def test_attention_host_checks():
    """attention_device rejects, before any device work: CPU tensors (no CPU
    fallback), a model width that the heads do not divide, q / k / v shapes
    that disagree, and batches that are not laid out row after row; the
    causal flag is taken only for a causal_mask() of the exact (query, key)
    length."""
    import torch

    from kansaiml_b200 import nn
    from kansaiml_b200.quantize import attention_device
    x = torch.zeros((2, 8, 64))
    with pytest.raises(ValueError, match="CUDA"):
        attention_device(x, x, x, 2)
    with pytest.raises(ValueError, match="heads"):
        attention_device(x, x, x, 3)
    with pytest.raises(ValueError, match="do not match"):
        attention_device(x, torch.zeros((2, 9, 64)), x, 2)
    m = nn.causal_mask(8, device="cpu")
    assert nn.MultiHeadAttention._causal(m, 8, 8)
    assert not nn.MultiHeadAttention._causal(m, 8, 9)
    assert not nn.MultiHeadAttention._causal(m, 4, 4)
    assert not nn.MultiHeadAttention._causal(kz.Tensor(m.data.clone()), 8, 8)
    assert not nn.MultiHeadAttention._causal(None, 8, 8)


def test_kansai_import_path_is_this_backend():
    """The reference's import lines (tests/test_quantize.py:22-23 style) resolve
    to this backend's objects, and both packages load side by side with the
    reference's own (registered under another name by the oracle)."""
    import kansai
    from kansai.quantize import QLinear, QTensor, dequantize, qlinear, quantize_symmetric
    from kansai import nn
    import kansai.distributed as kdist
    import kansaiml_b200.quantize as impl
    assert QLinear is impl.QLinear and QTensor is impl.QTensor and qlinear is impl.qlinear
    assert quantize_symmetric is impl.quantize_symmetric and dequantize is impl.dequantize
    assert nn is kz.nn and kdist is kz.distributed and kansai.Tensor is kz.Tensor
    t = kansai.tensor([[0, 1], [1, 0]], device="cpu")
    c = kansai.tensor([[1, 0], [0, 1]], device="cpu")
    assert kansai.where(c, t, kansai.zeros([2, 2], device="cpu")).tolist() == [0.0, 0.0, 0.0, 0.0]
    with kansai.no_grad():
        assert t.shape == [2, 2]
