"""KAN1 checkpoints (python/kansai/serialize.py): format interop with the
reference's own serialize module (run unmodified over its compiled core), the
reference's error checks, and the int8 extension for quantized layers."""
import os
import struct

import numpy as np
import pytest

from oracle import refpkg


def _mlp(seed0):
    from kansaiml_b200 import nn
    return nn.Sequential(nn.Linear(784, 256, seed=seed0), nn.ReLU(), nn.Linear(256, 10, seed=seed0 + 1))


def _params(module):
    return {n: t.numpy() for n, t in module.named_parameters()}


def test_roundtrip_cpu(tmp_path):
    from kansaiml_b200 import serialize
    a, b = _mlp(1), _mlp(7)
    path = str(tmp_path / "m.kan")
    serialize.save(a, path)
    serialize.load(b, path)
    pa, pb = _params(a), _params(b)
    assert list(pa) == ["layers.0.weight", "layers.0.bias", "layers.2.weight", "layers.2.bias"]
    for n in pa:
        assert pa[n].tobytes() == pb[n].tobytes(), n


@pytest.mark.skipif(not refpkg.reference_available(), reason="reference checkout / compiled core not present")
def test_interop_with_reference(tmp_path):
    """A checkpoint written here loads in the reference and vice versa."""
    from kansaiml_b200 import serialize
    ref = refpkg.import_reference_kansai()
    import kansai_reference.serialize as rser
    import kansai_reference.nn as rnn
    ours = _mlp(3)
    p1 = str(tmp_path / "ours.kan")
    serialize.save(ours, p1)
    theirs = rnn.Sequential(rnn.Linear(784, 256, seed=11), rnn.ReLU(), rnn.Linear(256, 10, seed=12))
    rser.load(theirs, p1)
    for (n, t), (rn, rt) in zip(ours.named_parameters(), theirs.named_parameters()):
        assert n == rn
        assert np.asarray(rt.tolist(), np.float32).tobytes() == t.numpy().reshape(-1).tobytes(), n
    theirs2 = rnn.Sequential(rnn.Linear(784, 256, seed=21), rnn.ReLU(), rnn.Linear(256, 10, seed=22))
    p2 = str(tmp_path / "theirs.kan")
    rser.save(theirs2, p2)
    mine = _mlp(5)
    serialize.load(mine, p2)
    for (n, t), (rn, rt) in zip(mine.named_parameters(), theirs2.named_parameters()):
        assert np.asarray(rt.tolist(), np.float32).tobytes() == t.numpy().reshape(-1).tobytes(), n
    assert ref is not None


def test_reference_error_checks(tmp_path):
    from kansaiml_b200 import serialize
    m = _mlp(1)
    good = str(tmp_path / "g.kan")
    serialize.save(m, good)
    raw = open(good, "rb").read()
    bad = str(tmp_path / "b.kan")
    open(bad, "wb").write(b"NOPE" + raw[4:])
    with pytest.raises(ValueError, match="not a Kansai checkpoint"):
        serialize.load(_mlp(2), bad)
    from kansaiml_b200 import nn
    other = nn.Sequential(nn.Linear(784, 128, seed=1), nn.ReLU(), nn.Linear(128, 10, seed=2))
    with pytest.raises(ValueError, match="shape mismatch"):
        serialize.load(other, good)
    small = nn.Sequential(nn.Linear(784, 256, seed=1))
    with pytest.raises(ValueError, match="doesn't expect"):
        serialize.load(small, good)
    open(bad, "wb").write(raw[:-100])
    with pytest.raises(ValueError, match="runs past the end"):
        serialize.load(_mlp(2), bad)


def _quantized_module(per_channel, seed):
    """A Module holding one QLinear built from the reference constructor
    QTensor(q, scale, shape) (no GPU needed)."""
    from kansaiml_b200 import nn
    from kansaiml_b200.quantize import QLinear, QTensor
    from kansaiml_b200.tensor import from_numpy
    rs = np.random.RandomState(seed)
    K, N = 64, 48
    q = rs.randint(-127, 128, (K, N))
    scale = rs.uniform(1e-3, 1e-2, N).tolist() if per_channel else float(rs.uniform(1e-3, 1e-2))
    ql = QLinear.__new__(QLinear)
    ql.qweight = QTensor(q.reshape(-1).tolist(), scale, [K, N])
    ql.bias = from_numpy(rs.standard_normal(N).astype(np.float32))
    ql.activations = None
    holder = nn.Module()
    holder.proj = ql
    holder.ln = nn.LayerNorm(N)
    return holder


@pytest.mark.parametrize("per_channel", [False, True])
def test_quantized_roundtrip(tmp_path, per_channel):
    from kansaiml_b200 import serialize
    a, b = _quantized_module(per_channel, 1), _quantized_module(per_channel, 2)
    path = str(tmp_path / "q.kan")
    serialize.save(a, path)
    with open(path, "rb") as f:
        assert f.read(4) == b"KAN1"
        hlen = struct.unpack("<Q", f.read(8))[0]
        import json
        header = json.loads(f.read(hlen))
    assert header["proj.qweight"]["dtype"] == "int8" and header["proj.qweight"]["shape"] == [64, 48]
    assert header["proj.qweight.scale"]["dtype"] == "float64"
    assert header["proj.qweight.scale"]["shape"] == ([48] if per_channel else [])
    serialize.load(b, path)
    qa, qb = a.proj.qweight, b.proj.qweight
    assert qa.q == qb.q
    assert np.array_equal(np.atleast_1d(np.asarray(qa.scale)), np.atleast_1d(np.asarray(qb.scale)))
    assert a.proj.bias.numpy().tobytes() == b.proj.bias.numpy().tobytes()
    # a per-tensor checkpoint does not load into a per-channel model
    if not per_channel:
        with pytest.raises(ValueError, match="shape mismatch"):
            serialize.load(_quantized_module(True, 3), path)


@pytest.mark.gpu
def test_quantized_decoder_checkpoint(tmp_path, cuda_device):
    """Config 3's int8 decoder: save, load into a differently seeded model of
    the same architecture, identical logits."""
    from kansaiml_b200 import serialize, workloads
    a = workloads.Decoder(seed=3, layers=1)
    b = workloads.Decoder(seed=9, layers=1)
    ids = workloads.config3_ids(batch=4, seed=4)
    path = str(tmp_path / "dec.kan")
    serialize.save(a, path)
    assert os.path.getsize(path) < 4 * 1024 * 1024
    serialize.load(b, path)
    assert a(ids).numpy().tobytes() == b(ids).numpy().tobytes()
