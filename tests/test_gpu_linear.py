"""GPU parity: qlinear with the reference's semantics (W8A32) and the W8A8
int8 tensor-core GEMM with its fused epilogue.

W8A32 outputs must be bit-identical to the reference's (golden fixtures) for
act none / relu; gelu goes through CUDA's erff, within 1e-6 absolute.
The int8 GEMM's int32 accumulators must be bit-exact against the oracle; its
fp32 epilogue applies the same fp32 operations in the same order as the
oracle, so it is compared bit-exact too (gelu: 1e-5 relative, the north-star
tolerance for fp32 outputs after dequantization).
"""
import numpy as np
import pytest
import torch

import inputs
from conftest import golden
from oracle import cpu as ocpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def k(cuda_device):
    import kansaiml_b200
    from kansaiml_b200 import nn, quantize
    return kansaiml_b200, nn, quantize


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ----------------------------------------------------------------- W8A32

def test_w8a32_golden_bit_exact(k):
    kz, nn, kq = k
    g = golden("w8a32_cases.npz")
    for i in range(int(g["count"])):
        x, w, b = inputs.w8a32_inputs(i)
        qw = kq.QTensor.from_tensor(dev(w))
        np.testing.assert_array_equal(qw.codes.cpu().numpy(), g[f"c{i}__q"])
        assert qw.scale == float(g[f"c{i}__scale"])
        y = kq.qlinear(dev(x), qw, dev(b)).numpy()
        assert y.tobytes() == g[f"c{i}__y"].tobytes(), i
        y = kq.qlinear(dev(x), qw, dev(b), act="relu").numpy()
        assert y.tobytes() == g[f"c{i}__y_relu"].tobytes(), i
        y = kq.qlinear(dev(x), qw, dev(b), act="gelu").numpy()
        np.testing.assert_allclose(y, g[f"c{i}__y_gelu"], rtol=0, atol=1e-6)


def test_mlp_config1_bit_exact(k):
    """BASELINE config 1 through nn.Sequential(QLinear, ReLU, QLinear)."""
    kz, nn, kq = k
    g = golden("mlp_config1.npz")
    x, b1, b2 = inputs.mlp_config1_inputs()
    l1 = nn.Linear(784, 256, seed=1)
    l2 = nn.Linear(256, 10, seed=2)
    assert inputs.sha(l1.weight.numpy()) == str(g["w1_sha256"])
    assert inputs.sha(l2.weight.numpy()) == str(g["w2_sha256"])
    l1.bias, l2.bias = kz.from_numpy(b1), kz.from_numpy(b2)
    qmodel = nn.Sequential(kq.QLinear(l1), nn.ReLU(), kq.QLinear(l2))
    np.testing.assert_array_equal(qmodel.layers[0].qweight.codes.cpu().numpy(), g["q1"])
    assert qmodel.layers[0].qweight.scale == float(g["s1"])
    y = qmodel(kz.from_numpy(x)).numpy()
    assert y.tobytes() == g["y"].tobytes()
    h = nn.ReLU()(qmodel.layers[0](kz.from_numpy(x))).numpy()    # unfused path
    assert h.tobytes() == g["h"].tobytes()


@pytest.mark.parametrize("M,K,N", [(1, 33, 10), (3, 784, 65), (64, 784, 256), (64, 256, 10), (300, 200, 300),
                                   (2048, 512, 1024), (129, 31, 1), (5, 4000, 70), (7, 1537, 40),
                                   (1537, 520, 1664), (1024, 2048, 2560), (2000, 517, 2048)])
def test_w8a32_shapes_vs_oracle(k, M, K, N):
    """The three W8A32 kernels (one thread per output for small batches, 64 x
    64 tiles, and 128 x 128 tiles with 8 x 8 outputs per thread for large
    aligned batches -- the last three shapes, one of them with K % 4 != 0,
    which falls back) against the oracle's k-ordered fp32 loop, bit-exact, on
    ragged M, K and N, short and long K."""
    kz, nn, kq = k
    rs = np.random.RandomState(M * 7 + K + N)
    x = rs.standard_normal((M, K)).astype(np.float32)
    w = (rs.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    bias = rs.standard_normal(N).astype(np.float32)
    qw = kq.QTensor.from_tensor(dev(w))
    q = qw.codes.cpu().numpy().reshape(K, N)
    for act in (0, 1):
        y = kq.qlinear(dev(x), qw, dev(bias), act=[None, "relu"][act]).numpy()
        yo = ocpu.qlinear_w8a32(x, q, qw.scale, bias, act)
        assert y.tobytes() == yo.tobytes(), (M, K, N, act)


def test_xor_quantized_predictions(k):
    """tests/test_quantize.py:81-125: the trained XOR model, quantized."""
    kz, nn, kq = k
    g = golden("xor_qlinear.npz")

    class L:
        pass
    l1, l2 = L(), L()
    l1.weight, l1.bias = kz.from_numpy(g["w1"]), kz.from_numpy(g["b1"])
    l2.weight, l2.bias = kz.from_numpy(g["w2"]), kz.from_numpy(g["b2"])
    qmodel = nn.Sequential(kq.QLinear(l1), nn.ReLU(), kq.QLinear(l2))
    y = qmodel(kz.from_numpy(g["x"])).numpy()
    assert y.tobytes() == g["quant_preds"].tobytes()
    assert np.abs(y.reshape(-1) - g["float_preds"].reshape(-1)).max() < 0.1
    assert [round(float(v)) for v in y.ravel()] == [0, 1, 1, 0]


def test_reference_tensor_objects_accepted(k):
    """A duck-typed reference Tensor (tolist + shape) quantizes like ours."""
    kz, nn, kq = k

    class RefLike:
        def __init__(self, a):
            self.a = a
            self.shape = list(a.shape)

        def tolist(self):
            return self.a.reshape(-1).tolist()

    x = inputs.quantize_case_inputs()["uniform1000"]
    q, s, shape = kq.quantize_symmetric(RefLike(x))
    qo, so = ocpu.quantize_tensor(x)
    assert s == so and np.array_equal(np.asarray(q, np.int8), qo)


# ------------------------------------------------------------------ W8A8

GEMM_SHAPES = [(1, 1, 16), (128, 256, 128), (37, 53, 208), (64, 10, 784), (300, 700, 1040), (129, 257, 4096),
               (1024, 1024, 1024), (256, 65, 256), (2000, 3000, 48)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_i8_int32_exact(k, M, N, K):
    kz, nn, kq = k
    rs = np.random.RandomState(M * 7 + N * 3 + K)
    a = rs.randint(-127, 128, (M, K)).astype(np.int8)
    b = rs.randint(-127, 128, (N, K)).astype(np.int8)
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    kq.gemm_i8_device(dev(a), dev(b), out_i32=acc)
    np.testing.assert_array_equal(acc.cpu().numpy(), ocpu.gemm_i8(a, b))
    assert kq.device_status() == 0


def test_gemm_i8_extreme_codes(k):
    """All -128 / +127 operands: the accumulator's extreme magnitudes."""
    kz, nn, kq = k
    M, N, K = 256, 256, 8192
    a = np.full((M, K), -128, np.int8)
    b = np.full((N, K), -128, np.int8)
    b[1::2] = 127
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    kq.gemm_i8_device(dev(a), dev(b), out_i32=acc)
    np.testing.assert_array_equal(acc.cpu().numpy(), ocpu.gemm_i8(a, b))


@pytest.mark.parametrize("act", [None, "relu", "gelu"])
@pytest.mark.parametrize("per_row", [False, True])
def test_gemm_epilogue_vs_oracle(k, act, per_row):
    kz, nn, kq = k
    M, N, K = 333, 520, 672
    rs = np.random.RandomState(5)
    a = rs.randint(-127, 128, (M, K)).astype(np.int8)
    b = rs.randint(-127, 128, (N, K)).astype(np.int8)
    rsc = rs.uniform(1e-3, 1e-2, M if per_row else 1).astype(np.float32)
    csc = rs.uniform(1e-3, 1e-2, N).astype(np.float32)
    bias = rs.standard_normal(N).astype(np.float32)
    partials = torch.zeros(1024, dtype=torch.int32, device="cuda")
    y, acc = kq.gemm_i8_device(dev(a), dev(b), row_scale=dev(rsc), col_scale=dev(csc), bias=dev(bias), act=act,
                               out_i32=torch.empty((M, N), dtype=torch.int32, device="cuda"), partials=partials)
    acc_o = ocpu.gemm_i8(a, b)
    np.testing.assert_array_equal(acc.cpu().numpy(), acc_o)
    yo = ocpu.epilogue(acc_o, rsc if per_row else rsc[0], csc, bias, {None: 0, "relu": 1, "gelu": 2}[act])
    yg = y.cpu().numpy()
    if act == "gelu":
        np.testing.assert_allclose(yg, yo, rtol=1e-5, atol=1e-6)
    else:
        assert yg.tobytes() == yo.tobytes()
    # fused absmax of the output
    p = partials.cpu().numpy().view(np.uint32)
    amax = p[1:1 + p[0]].max().view(np.float32) if p[0] else 0.0
    assert amax == np.abs(yg).max()


def test_gemm_blocked_a_layout(k):
    """A stored as G rank-major blocks [G][M][K/G] (an all-gather of column
    shards) gives the same result as the plain [M, K] layout."""
    kz, nn, kq = k
    G, M, N, Kb = 4, 300, 256, 256
    K = G * Kb
    rs = np.random.RandomState(11)
    a = rs.randint(-127, 128, (M, K)).astype(np.int8)
    b = rs.randint(-127, 128, (N, K)).astype(np.int8)
    blocked = np.ascontiguousarray(a.reshape(M, G, Kb).transpose(1, 0, 2))
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    kq.gemm_i8_device(dev(blocked), dev(b), out_i32=acc, a_kblock=Kb, m=M)
    np.testing.assert_array_equal(acc.cpu().numpy(), ocpu.gemm_i8(a, b))


def test_gemm_k0(k):
    kz, nn, kq = k
    M, N = 5, 7
    a = torch.empty((M, 0), dtype=torch.int8, device="cuda")
    b = torch.empty((N, 0), dtype=torch.int8, device="cuda")
    bias = dev(np.arange(N, dtype=np.float32) - 3)
    one = dev(np.ones(1, np.float32))
    y, _ = kq.gemm_i8_device(a, b, row_scale=one, col_scale=one, bias=bias, act="relu")
    np.testing.assert_array_equal(y.cpu().numpy(), np.maximum(np.tile(np.arange(N) - 3.0, (M, 1)), 0))


def test_w8a8_qlinear_config2_vs_oracle(k):
    """per-channel W [4096, 4096] ~ N(0, 0.02), X [2048, 4096]
    ~ N(0, 1), per-tensor activations.  Weight codes, and every one of the
    2048 output rows: the oracle's int8 GEMM (all rows) + epilogue, bit for
    bit."""
    kz, nn, kq = k
    rs = np.random.RandomState(2)
    w = (rs.standard_normal((4096, 4096)) * 0.02).astype(np.float32)
    x = rs.standard_normal((2048, 4096)).astype(np.float32)

    class L:
        pass
    lin = L()
    lin.weight, lin.bias = kz.from_numpy(w), None
    ql = kq.QLinear(lin, per_channel=True)
    y = ql(kz.from_numpy(x)).numpy()
    wq, ws = ocpu.quantize_cols(w)
    np.testing.assert_array_equal(ql.qweight.codes.cpu().numpy(), wq)
    xq, xs = ocpu.quantize_tensor(x)
    yo = ocpu.epilogue(ocpu.gemm_i8(xq, wq), xs, ws)
    assert y.tobytes() == yo.tobytes()
