// qlinear with the reference's exact semantics (W8A32):
//   out = act(x @ dequantize(q, scale) + bias)
// python/kansai/quantize.py:115-122 -> Tensor::matmul (core/src/Tensor.cpp:332-362)
// -> cpu::matmul (backend/cpu/src/Ops.cpp:328-337) -> add_bias_broadcast
// (Ops.cpp:34-38) -> relu_fwd / gelu_fwd (Ops.cpp:197-199, 250-256).
//
// The reference's loop accumulates each output in k order, starting from
// +0.0f, with the product and the sum each rounded to fp32 (no FMA on the
// Linux build).  This kernel keeps that order per output and uses
// __fmul_rn / __fadd_rn so the compiler cannot contract them, which makes
// its results bit-identical to the reference for act none/relu.  Tensor
// cores are deliberately not used: TF32 or any reordering of the k sum would
// change the fp32 rounding.  The weight is dequantized on the fly through a
// 255-entry table table[q + 127] = (float)((double)q * scale)
// (quantize.py:76 + Tensor::from_flat's narrowing).
#include "kz_common.cuh"

namespace kz {

constexpr int kBM = 64, kBN = 64, kBK = 16;

__device__ __forceinline__ float act_apply(float v, int act) {
    if (act == KZ_ACT_RELU) return v > 0.0f ? v : 0.0f;
    if (act == KZ_ACT_GELU) {
        const float cdf = __fmul_rn(0.5f, __fadd_rn(1.0f, erff(__fmul_rn(v, 0.7071067811865476f))));
        return __fmul_rn(v, cdf);
    }
    return v;
}

// 256 threads as 16 x 16; each computes a 4 x 4 block of a 64 x 64 tile.
__global__ void __launch_bounds__(256) qlinear_w8a32_kernel(const float* __restrict__ x, int64_t M, int64_t K,
                                                            const int8_t* __restrict__ q, double scale,
                                                            const float* __restrict__ bias, int64_t N, int act,
                                                            float* __restrict__ out) {
    __shared__ float table[256];
    __shared__ float As[kBK][kBM + 4];
    __shared__ float Bs[kBK][kBN + 4];
    const int tid = threadIdx.x;
    if (tid < 255) table[tid] = __double2float_rn((double)(tid - 127) * scale);
    if (tid == 255) table[255] = __double2float_rn(-128.0 * scale);
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = blockIdx.y * (int64_t)kBM, n0 = blockIdx.x * (int64_t)kBN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    __syncthreads();
    for (int64_t k0 = 0; k0 < K; k0 += kBK) {
        // x tile: 64 rows x 16 k -> As[k][m]
        for (int e = tid; e < kBM * kBK; e += 256) {
            const int mm = e / kBK, kk = e % kBK;
            const int64_t m = m0 + mm, k = k0 + kk;
            As[kk][mm] = (m < M && k < K) ? x[m * K + k] : 0.0f;
        }
        // weight tile: 16 k x 64 n -> Bs[k][n], dequantized
        for (int e = tid; e < kBK * kBN; e += 256) {
            const int kk = e / kBN, nn = e % kBN;
            const int64_t k = k0 + kk, n = n0 + nn;
            Bs[kk][nn] = (k < K && n < N) ? table[(int)q[k * N + n] + 127 & 255] : 0.0f;
        }
        __syncthreads();
        const int kend = (int)min((int64_t)kBK, K - k0);
        for (int kk = 0; kk < kend; ++kk) {   // k order preserved
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tx * 4 + j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (bias) v = __fadd_rn(v, bias[n]);
            out[m * N + n] = act_apply(v, act);
        }
    }
}

// Small-M form: one thread per output, so M x N independent k-ordered chains
// run at once (the 64 x 64 tiles above give a 64-row batch only N / 64
// blocks).  A block is 4 rows (one warp each) x 32 columns (one lane each);
// the weight is staged 32 k x 32 n at a time, dequantized through the table,
// double-buffered in shared memory with the next chunk's codes and x values
// prefetched into registers; x[m, k] reaches every lane of the row's warp by
// shuffle.  Same operations in the same order as the tiled kernel.
constexpr int kRowsR = 4, kColsR = 32, kChunkR = 32;

__global__ void __launch_bounds__(128) qlinear_w8a32_rows_kernel(const float* __restrict__ x, int64_t M, int64_t K,
                                                                 const int8_t* __restrict__ q, double scale,
                                                                 const float* __restrict__ bias, int64_t N, int act,
                                                                 float* __restrict__ out) {
    __shared__ float table[256];
    __shared__ float ws[2][kChunkR][kColsR + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < 256; i += 128)
        table[i] = i < 255 ? __double2float_rn((double)(i - 127) * scale) : __double2float_rn(-128.0 * scale);
    const int64_t m = blockIdx.y * (int64_t)kRowsR + warp;
    const int64_t n0 = blockIdx.x * (int64_t)kColsR;
    const bool row_ok = m < M;
    // staging map: thread t owns chunk row kk = t / 4 and columns 8 (t % 4) .. + 7
    const int skk = tid >> 2, sc0 = (tid & 3) * 8;
    int8_t code[8];
    float xr = 0.0f;
    auto fetch = [&](int64_t k0) {
        const int64_t k = k0 + skk;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t n = n0 + sc0 + j;
            code[j] = (k < K && n < N) ? __ldg(q + k * N + n) : (int8_t)0;
        }
        xr = (row_ok && k0 + lane < K) ? __ldg(x + m * K + k0 + lane) : 0.0f;
    };
    fetch(0);
    __syncthreads();   // table ready
    float acc = 0.0f;
    int buf = 0;
    for (int64_t k0 = 0; k0 < K; k0 += kChunkR) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ws[buf][skk][sc0 + j] = table[((int)code[j] + 127) & 255];
        const float xc = xr;
        if (k0 + kChunkR < K) fetch(k0 + kChunkR);
        __syncthreads();
        const int kend = (int)min((int64_t)kChunkR, K - k0);
        if (kend == kChunkR) {
#pragma unroll
            for (int kk = 0; kk < kChunkR; ++kk)   // k order preserved
                acc = __fadd_rn(acc, __fmul_rn(__shfl_sync(0xffffffffu, xc, kk), ws[buf][kk][lane]));
        } else {
            for (int kk = 0; kk < kend; ++kk)
                acc = __fadd_rn(acc, __fmul_rn(__shfl_sync(0xffffffffu, xc, kk), ws[buf][kk][lane]));
        }
        buf ^= 1;
    }
    const int64_t n = n0 + lane;
    if (row_ok && n < N) {
        float v = acc;
        if (bias) v = __fadd_rn(v, bias[n]);
        out[m * N + n] = act_apply(v, act);
    }
}

}  // namespace kz

using namespace kz;

extern "C" int kz_qlinear_w8a32_f32(const float* x, int64_t M, int64_t K, const int8_t* q, double scale,
                                    const float* bias, int64_t N, int act, float* out, kz_stream_t stream) {
    KZ_REQUIRE(M >= 0 && K >= 0 && N >= 0, "kz_qlinear_w8a32_f32: negative dimension");
    KZ_REQUIRE(act >= KZ_ACT_NONE && act <= KZ_ACT_GELU, "kz_qlinear_w8a32_f32: unknown activation");
    if (M == 0 || N == 0) return KZ_OK;
    KZ_REQUIRE(out != nullptr, "kz_qlinear_w8a32_f32: out is NULL");
    KZ_REQUIRE(K == 0 || (x && q), "kz_qlinear_w8a32_f32: x or q is NULL");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // Few 64 x 64 tiles (small batches) leave most SMs idle: one thread per
    // output instead.  Both kernels round identically.
    const int64_t tiles = ((N + kBN - 1) / kBN) * ((M + kBM - 1) / kBM);
    if (tiles < 2 * (int64_t)sm_count()) {
        KZ_REQUIRE((M + kRowsR - 1) / kRowsR < 65536, "kz_qlinear_w8a32_f32: M too large");
        dim3 grid((unsigned)((N + kColsR - 1) / kColsR), (unsigned)((M + kRowsR - 1) / kRowsR));
        qlinear_w8a32_rows_kernel<<<grid, 128, 0, s>>>(x, M, K, q, scale, bias, N, act, out);
        return launch_status("qlinear_w8a32_rows_kernel");
    }
    KZ_REQUIRE((M + kBM - 1) / kBM < 65536, "kz_qlinear_w8a32_f32: M too large");
    dim3 grid((unsigned)((N + kBN - 1) / kBN), (unsigned)((M + kBM - 1) / kBM));
    qlinear_w8a32_kernel<<<grid, 256, 0, s>>>(x, M, K, q, scale, bias, N, act, out);
    return launch_status("qlinear_w8a32_kernel");
}
