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

// Large-batch form for aligned shapes (K % 4 == 0, N % 4 == 0, 16-byte
// aligned x and out, 4-byte aligned q): 128 x 128 tiles, 256 threads, 8 x 8
// outputs per thread -- rows {4 ty .. +3, 64 + 4 ty .. +3} and the same for
// columns, so the 16-byte shared loads of a quarter-warp never conflict --
// giving 128 multiplies and adds per four 16-byte shared loads.  The k tile
// (8 deep) is double-buffered: the next tile's x (one float4) and codes (one
// word) are in registers while the current one is consumed.  Same operations
// in the same k order as the other two kernels.
constexpr int kTM = 128, kTN = 128, kTK = 8, kTP = kTM + 4;

__global__ void __launch_bounds__(256, 2) qlinear_w8a32_tile128_kernel(const float* __restrict__ x, int64_t M,
                                                                       int64_t K, const int8_t* __restrict__ q,
                                                                       double scale, const float* __restrict__ bias,
                                                                       int64_t N, int act, float* __restrict__ out) {
    __shared__ float table[256];
    __shared__ __align__(16) float As[2][kTK][kTP];
    __shared__ __align__(16) float Bs[2][kTK][kTP];
    const int tid = threadIdx.x;
    // entry u: the value of the code whose byte is u (quantize.py:76 + from_flat)
    table[tid] = __double2float_rn((double)(int)(int8_t)(uint8_t)tid * scale);
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = blockIdx.y * (int64_t)kTM, n0 = blockIdx.x * (int64_t)kTN;
    // staging maps: x row xr, k half xh (one float4); code row wk, columns wc .. wc + 3 (one word)
    const int xr = tid >> 1, xh = tid & 1;
    const int wk = tid >> 5, wc = (tid & 31) * 4;
    const bool x_row_ok = m0 + xr < M, w_col_ok = n0 + wc < N;
    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t wv = 0;
    auto fetch = [&](int64_t k0) {
        const int64_t kx = k0 + 4 * xh, kw = k0 + wk;
        xv = (x_row_ok && kx < K) ? __ldg(reinterpret_cast<const float4*>(x + (m0 + xr) * K + kx))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        wv = (w_col_ok && kw < K) ? __ldg(reinterpret_cast<const uint32_t*>(q + kw * N + n0 + wc)) : 0u;
    };
    auto stage = [&](int b) {
        As[b][4 * xh + 0][xr] = xv.x;
        As[b][4 * xh + 1][xr] = xv.y;
        As[b][4 * xh + 2][xr] = xv.z;
        As[b][4 * xh + 3][xr] = xv.w;
        *reinterpret_cast<float4*>(&Bs[b][wk][wc]) =
            make_float4(table[wv & 0xFFu], table[(wv >> 8) & 0xFFu], table[(wv >> 16) & 0xFFu], table[wv >> 24]);
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    fetch(0);
    __syncthreads();   // table ready
    stage(0);
    __syncthreads();
    int buf = 0;
    for (int64_t k0 = 0; k0 < K; k0 += kTK) {
        const bool more = k0 + kTK < K;
        if (more) fetch(k0 + kTK);
        const int kend = (int)min((int64_t)kTK, K - k0);
        for (int kk = 0; kk < kend; ++kk) {   // k order preserved
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][4 * ty]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + 4 * ty]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][4 * tx]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + 4 * tx]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        if (more) {
            stage(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
        if (m >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t n = n0 + h * 64 + 4 * tx;
            if (n >= N) continue;   // N % 4 == 0: the four columns are in or out together
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float t = acc[i][4 * h + j];
                if (bias) t = __fadd_rn(t, __ldg(bias + n + j));
                v[j] = act_apply(t, act);
            }
            *reinterpret_cast<float4*>(out + m * N + n) = make_float4(v[0], v[1], v[2], v[3]);
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
    // Enough 128 x 128 tiles for every SM, aligned shapes: the 8 x 8 per
    // thread kernel.
    const int64_t tiles128 = ((N + kTN - 1) / kTN) * ((M + kTM - 1) / kTM);
    const bool aligned = K % 4 == 0 && N % 4 == 0 && K > 0 &&
                         ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(q) & 3u) == 0;
    if (aligned && tiles128 >= (int64_t)sm_count() && (M + kTM - 1) / kTM < 65536) {
        dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
        qlinear_w8a32_tile128_kernel<<<grid, 256, 0, s>>>(x, M, K, q, scale, bias, N, act, out);
        return launch_status("qlinear_w8a32_tile128_kernel");
    }
    // Few 64 x 64 tiles (small batches) leave most SMs idle: one thread per
    // output instead.  All three kernels round identically.
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
