"""GPU tests of the gated int8 GEMM on one GPU (kz_gemm_i8_gated): its A
operand arrives while it runs, delivered by the copy engines
(kz_copy_and_flag on another stream), and must give the plain GEMM's result
bit for bit.  Failure detection without a GPU fault: a flag that nothing ever
sets makes the kernel's bounded wait (1 s) run out; the kernel records
KZ_ERR_DEVICE_TIMEOUT in the status word and unwinds, and the context stays
usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs(cuda_device):
    from kansaiml_b200 import _lib
    from kansaiml_b200 import quantize as kq
    return _lib, _lib.load(), kq


def _operands(G, M, kb, N, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    src = torch.randint(-127, 128, (G, M, kb), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (N, G * kb), dtype=torch.int8, device="cuda", generator=g)
    rs = torch.full((1,), 0.01, device="cuda")
    cs = torch.rand(N, device="cuda", generator=g) * 0.01 + 1e-3
    return src, b, rs, cs


@pytest.mark.parametrize("flag_rows", [384, 128])
def test_gated_gemm_fed_by_copy_engines(libs, flag_rows):
    _lib, lib, kq = libs
    G, M, kb, N, first = 3, 384, 256, 512, 1
    src, b, rs, cs = _operands(G, M, kb, N, 7)
    K = G * kb
    chunks = -(-M // flag_rows)
    a = torch.zeros_like(src)
    a[first] = src[first]                         # the resident block
    flags = torch.zeros(G * chunks, dtype=torch.int32, device="cuda")
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    torch.cuda.synchronize()
    # the GEMM goes first; the rest of A arrives afterwards from another stream
    assert lib.kz_gemm_i8_gated(a.data_ptr(), b.data_ptr(), M, N, K, kb, rs.data_ptr(), 0, cs.data_ptr(), 1, None,
                                0, out.data_ptr(), None, N, None, flags.data_ptr(), 1, first, flag_rows,
                                main.cuda_stream) == 0
    for h in range(G):
        if h == first:
            continue
        for c in range(chunks):
            r0, r1 = c * flag_rows, min(M, (c + 1) * flag_rows)
            assert lib.kz_copy_and_flag(a[h, r0:r1].data_ptr(), src[h, r0:r1].data_ptr(), (r1 - r0) * kb,
                                        flags.data_ptr() + 4 * (h * chunks + c), 1, side.cuda_stream) == 0
    torch.cuda.synchronize()
    assert kq.device_status(clear=True) == 0
    ref, _ = kq.gemm_i8_device(src, b, row_scale=rs, col_scale=cs, a_kblock=kb, m=M)
    assert torch.equal(out, ref)


def test_gated_gemm_wait_runs_out(libs):
    """Nothing ever sets block 2's flag: the bounded wait expires after about a
    second, the status word says KZ_ERR_DEVICE_TIMEOUT, and the device keeps
    working."""
    _lib, lib, kq = libs
    G, M, kb, N = 3, 256, 128, 256
    src, b, rs, cs = _operands(G, M, kb, N, 9)
    flags = torch.zeros(G, dtype=torch.int32, device="cuda")
    flags[1] = 1                                  # block 1 present, block 2 never
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    assert kq.device_status(clear=True) == 0
    assert lib.kz_gemm_i8_gated(src.data_ptr(), b.data_ptr(), M, N, G * kb, kb, rs.data_ptr(), 0, cs.data_ptr(), 1,
                                None, 0, out.data_ptr(), None, N, None, flags.data_ptr(), 1, 0, M,
                                torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert kq.device_status(clear=True) == _lib.KZ_ERR_DEVICE_TIMEOUT
    # the context is still usable
    y, _ = kq.gemm_i8_device(src, b, row_scale=rs, col_scale=cs, a_kblock=kb, m=M)
    torch.cuda.synchronize()
    assert kq.device_status(clear=True) == 0
    assert torch.isfinite(y).all()
