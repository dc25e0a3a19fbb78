"""GPU parity: scale finding, quantize and dequantize (libkz) vs the reference.

Codes must be bit-exact and scales the identical double; dequantized values
bit-identical fp32.  Small cases against the reference's own golden outputs,
large and adversarial cases against the pinned C oracle.
"""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kq(cuda_device):
    from kansaiml_b200 import quantize
    return quantize


def dev(a, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def test_golden_quantize_symmetric(kq):
    g = golden("quantize_cases.npz")
    cases = inputs.quantize_case_inputs()
    for name, x in cases.items():
        q, s, shape = kq.quantize_symmetric(dev(x))
        assert shape == list(x.shape)
        assert s == float(g[f"{name}__scale"]), name
        np.testing.assert_array_equal(np.asarray(q, np.int8), g[f"{name}__q"].reshape(-1), err_msg=name)


def test_golden_reference_randn_case(kq):
    """tests/test_quantize.py:66-72 input from the reference's own randn."""
    import kansaiml_b200 as k
    g = golden("quantize_cases.npz")
    t = k.randn([256, 256], std=1.0, seed=1)
    np.testing.assert_array_equal(t.numpy()[0], g["randn256_seed1__first_row"])
    qt = kq.QTensor.from_tensor(t)
    assert qt.scale == float(g["randn256_seed1__scale"])
    np.testing.assert_array_equal(qt.codes.cpu().numpy(), g["randn256_seed1__q"])
    assert 4 * t.numel() / qt.nbytes() == 4.0


def test_golden_dequantize(kq):
    g = golden("quantize_cases.npz")
    for name in [str(n) for n in g["names"]]:
        if f"{name}__deq" not in g:
            continue
        q = g[f"{name}__q"]
        s = float(g[f"{name}__scale"])
        out = kq.dequantize(q.reshape(-1).tolist(), s, list(q.shape))
        assert out.numpy().tobytes() == g[f"{name}__deq"].tobytes(), name


def test_roundtrip_bound_and_zero(kq):
    """tests/test_quantize.py:41-60 on the device."""
    x = inputs.quantize_case_inputs()["uniform1000"]
    q, s, shape = kq.quantize_symmetric(dev(x))
    rec = kq.dequantize(q, s, shape).numpy().astype(np.float64)
    assert np.abs(x.astype(np.float64) - rec).max() <= s / 2 + 1e-6
    q0, _, _ = kq.quantize_symmetric(dev(np.asarray([0.0, 1.0, -1.0], np.float32)))
    assert q0[0] == 0


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_nonfinite_raises(kq, bad):
    x = np.random.RandomState(0).standard_normal(10000).astype(np.float32)
    x[1234] = bad
    with pytest.raises(ValueError):
        kq.quantize_symmetric(dev(x))
    assert kq.device_status(clear=True) == 2   # KZ_ERR_NONFINITE, recorded on the device
    assert kq.device_status(clear=True) == 0


@pytest.mark.parametrize("n", [1, 15, 16, 17, 4095, 1 << 20, (1 << 20) + 7])
def test_quantize_sizes_vs_oracle(kq, n):
    x = (np.random.RandomState(n % 1000).standard_normal(n) * 3.7).astype(np.float32)
    q, s64, s32 = kq.quantize_tensor_device(dev(x))
    qo, so = ocpu.quantize_tensor(x)
    assert float(s64.item()) == so
    assert float(s32.item()) == np.float32(so)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


def test_quantize_unaligned_views(kq):
    """A tensor starting 4 bytes past an allocation takes the scalar path."""
    x = np.random.RandomState(9).standard_normal(100001).astype(np.float32)
    base = dev(x)
    v = base[1:]
    q, s64, _ = kq.quantize_tensor_device(v)
    qo, so = ocpu.quantize_tensor(x[1:])
    assert float(s64.item()) == so
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


def test_near_tie_stress_vs_oracle(kq):
    """Millions of values at / within ulps of half-integer quotients, at many
    scales: the fp32 fast path must hand every one of them to the exact path."""
    rs = np.random.RandomState(2024)
    for trial in range(6):
        amax = float(np.float32(10.0 ** rs.uniform(-30, 30)))
        scale = amax / 127.0
        k = rs.randint(-126, 127, 400000)
        v = ((k + 0.5) * scale).astype(np.float32)
        steps = rs.randint(-2, 3, v.size)
        v = np.where(steps > 0, np.nextafter(v, np.float32(np.inf)), v)
        v = np.where(steps < 0, np.nextafter(v, np.float32(-np.inf)), v).astype(np.float32)
        v = np.clip(v, -np.float32(amax), np.float32(amax))
        v[0] = np.float32(amax)
        q, s64, _ = kq.quantize_tensor_device(dev(v))
        qo, so = ocpu.quantize_tensor(v)
        assert float(s64.item()) == so
        np.testing.assert_array_equal(q.cpu().numpy(), qo, err_msg=f"trial {trial} amax {amax}")


@pytest.mark.parametrize("offset", [0, 1])
def test_guard_band_stress_vs_oracle(kq, offset):
    """Quotients at 2^-18 .. 2^-11 (in code units) from half-integers, on both
    sides of the fast paths' tie guards (2^-16 for the fused multiply-add form,
    2^-15 for the scalar form).  offset=1 makes the view unaligned, which takes
    the scalar form."""
    rs = np.random.RandomState(77 + offset)
    for trial in range(4):
        amax = float(np.float32(10.0 ** rs.uniform(-20, 20)))
        scale = amax / 127.0
        k = rs.randint(-127, 127, 300000)
        delta = rs.choice([1.0, -1.0], k.size) * 2.0 ** rs.uniform(-18, -11, k.size)
        v = ((k + 0.5 + delta) * scale).astype(np.float32)
        v = np.clip(v, -np.float32(amax), np.float32(amax))
        v[0] = np.float32(amax)
        base = dev(np.concatenate([np.zeros(offset, np.float32), v]))
        q, s64, _ = kq.quantize_tensor_device(base[offset:])
        qo, so = ocpu.quantize_tensor(v)
        assert float(s64.item()) == so
        np.testing.assert_array_equal(q.cpu().numpy(), qo, err_msg=f"trial {trial} amax {amax}")


def test_full_config2_activation_vs_oracle(kq):
    """BASELINE config 2 activations [2048, 4096] ~ N(0, 1), full size."""
    x = np.random.RandomState(1).standard_normal((2048, 4096)).astype(np.float32)
    q, s64, _ = kq.quantize_tensor_device(dev(x))
    qo, so = ocpu.quantize_tensor(x)
    assert float(s64.item()) == so
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


def test_golden_per_channel(kq):
    g = golden("percol_cases.npz")
    w = inputs.percol_weight()
    qt = kq.QTensor.from_tensor(dev(w), per_channel=True)
    np.testing.assert_array_equal(qt.codes.cpu().numpy(), g["qT"])
    np.testing.assert_array_equal(np.asarray(qt.scale), g["scales"])
    # q materialises in the weight's own [K, N] layout
    np.testing.assert_array_equal(np.asarray(qt.q, np.int8).reshape(w.shape), g["qT"].T)


@pytest.mark.parametrize("K,N", [(1, 1), (7, 33), (200, 130), (1000, 520), (4096, 4096), (3000, 10)])
def test_per_channel_vs_oracle(kq, K, N):
    w = (np.random.RandomState(K + N).standard_normal((K, N)) * 0.02).astype(np.float32)
    qT, s64, s32 = kq.quantize_cols_device(dev(w))
    qo, so = ocpu.quantize_cols(w)
    np.testing.assert_array_equal(s64.cpu().numpy(), so)
    np.testing.assert_array_equal(s32.cpu().numpy(), so.astype(np.float32))
    np.testing.assert_array_equal(qT.cpu().numpy(), qo)


@pytest.mark.parametrize("M,K", [(1, 1), (5, 300), (64, 4096), (513, 1000)])
def test_per_row_vs_oracle(kq, M, K):
    x = np.random.RandomState(M * K).standard_normal((M, K)).astype(np.float32)
    x[0] = 0.0
    q, s64, _ = kq.quantize_rows_device(dev(x))
    qo, so = ocpu.quantize_rows(x)
    np.testing.assert_array_equal(s64.cpu().numpy(), so)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("n", [1, 17, 1 << 20, 3 * (1 << 20) + 5])
def test_dequantize_vs_oracle(kq, n):
    rs = np.random.RandomState(n % 997)
    q = rs.randint(-127, 128, n).astype(np.int8)
    s = float(rs.uniform(1e-4, 1.0))
    out = kq.dequantize(q.tolist() if n < 100000 else kq.QTensor(q, s, [n]), s, [n])
    assert out.numpy().tobytes() == ocpu.dequantize(q, s).tobytes()


@pytest.mark.parametrize("s", [0.02 / 127, 1.0, 3e-39, 2e-38, 1e-42, -0.5, 1e39])
def test_dequantize_both_forms_bit_exact(kq, s):
    """Every byte value (all 256, -128 included), aligned and at an odd
    offset, at scales that take the table-free split form (0.02/127, 1.0) and
    at scales that do not (subnormal products, a negative scale, one past fp32
    range): the result equals (float)((double)q * scale) bit for bit either
    way."""
    import torch
    from kansaiml_b200 import _lib
    lib = _lib.load()
    assert lib.kz_dequantize_uses_table(s) == (0 if s in (0.02 / 127, 1.0) else 1)
    codes = np.tile(np.arange(-128, 128, dtype=np.int16).astype(np.int8), 4099)
    qd = torch.from_numpy(codes).cuda()
    ref = (codes.astype(np.float64) * s).astype(np.float32)
    for off in (0, 1):
        n = codes.size - off
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        _lib.call("kz_dequantize_i8_f32", qd.data_ptr() + off, n, s, out.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert out.cpu().numpy().tobytes() == ref[off:].tobytes(), (s, off)


def test_dequantize_per_channel_roundtrip(kq):
    w = (np.random.RandomState(3).standard_normal((300, 200)) * 0.05).astype(np.float32)
    qt = kq.QTensor.from_tensor(dev(w), per_channel=True)
    deq = qt.dequantize().numpy()
    qo, so = ocpu.quantize_cols(w)
    ref = (qo.T.astype(np.float64) * so[None, :]).astype(np.float32)
    assert deq.tobytes() == ref.tobytes()
    assert np.all(np.abs(deq - w) <= (so[None, :] / 2 + 1e-7))


def test_fused_single_launch_repeated_calls(kq):
    """Large tensors take the single cooperative launch (absmax, grid barrier,
    quantize); 12000003 elements overflow the shared-memory-resident chunk of
    every block, so each block also reads a remainder from global memory.
    Repeated calls on one partials buffer stay bit-exact; each call leaves the
    barrier word (second-to-last) with zero low bits and bit 31 flipped, and
    the reserved last word at zero."""
    from kansaiml_b200 import _lib
    lib = _lib.load()
    partials = torch.zeros(1024, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    calls = 0
    for seed, n, scale in [(0, 1 << 22, 1.0), (1, (1 << 23) + 13, 1e-3), (2, 3 << 20, 50.0), (3, 12000003, 2.0)]:
        x = (np.random.RandomState(seed).standard_normal(n) * scale).astype(np.float32)
        xd = dev(x)
        q = torch.empty(n, dtype=torch.int8, device="cuda")
        s64 = torch.empty(1, dtype=torch.float64, device="cuda")
        s32 = torch.empty(1, dtype=torch.float32, device="cuda")
        for _ in range(3):
            assert lib.kz_quantize_tensor_f32(xd.data_ptr(), n, q.data_ptr(), s64.data_ptr(), s32.data_ptr(),
                                              partials.data_ptr(), stream) == 0
            calls += 1
        torch.cuda.synchronize()
        qo, so = ocpu.quantize_tensor(x)
        assert float(s64.item()) == so
        np.testing.assert_array_equal(q.cpu().numpy(), qo)
        assert partials[-2:].cpu().numpy().tolist() == [-(1 << 31) if calls % 2 else 0, 0]
    assert kq.device_status() == 0
