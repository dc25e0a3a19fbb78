// Scaled dot-product attention in the reference's own operation order.
//
// The reference composes MultiHeadAttention.forward (python/kansai/nn.py:
// 410-427) from Tensor ops, each a plain fp32 loop:
//   scores = q.matmul(k^T)        Ops.cpp:322-339  out += a*b, reduction index ascending
//   scores = scores.mul(scale)    fp32 multiply by fl(1/sqrt(d_k))
//   scores = scores.add(mask)     optional additive mask, broadcast
//   softmax(3)                    Tensor.cpp:906-913: max (Ops.cpp:275-292), sub,
//                                 exp (std::exp), sum (reduce_to_shape, Ops.cpp:
//                                 177-190, index ascending from 0), div = mul by
//                                 the reciprocal 1/x (Tensor.cpp:677-679, Ops.cpp:213-215)
//   attended = weights.matmul(v)  key index ascending
// This kernel computes the same values with the same roundings: every
// product and every sum is a separately rounded fp32 operation (__fmul_rn /
// __fadd_rn, never contracted into an FMA) taken in the reference's index
// order.  The one operation it cannot take from the reference is exp: the
// reference calls the host libm's expf; here exp is rounded correctly from a
// double-precision exp (CUDA's exp(double), error below 1 ulp of double), which
// equals the host's expf wherever that one is correctly rounded.
//
// A causal flag replaces causal_mask()'s additive -1e9 entries without
// reading them: those keys get an exponential of exactly 0, so leaving them
// out of the max, the sum and the weighted sum of v changes no bit (adding
// +-0 to a non-zero fp32 sum is exact, and the diagonal key keeps every row's
// sum non-zero).
//
// Work decomposition: one CTA per (batch, head, block of 64 query rows), the
// blocks with the most keys (causal) first.  The CTA stages its query rows,
// then 64-key tiles of K, in shared memory (row pitch d_k + 4 floats, so the
// 16-byte reads of 8 consecutive lanes fall in distinct bank groups), keeps
// the block's whole score rows on chip, runs the softmax there and streams
// 64-key tiles of V for the weighted sum.  Thread tile 8 query rows x 4 keys
// (rows ty + 8a, keys tx + 16b): per 4 reduction steps 12 shared 16-byte
// loads feed 256 fp32 operations.  The next tile's global loads are issued
// into registers before the current tile's arithmetic.  The output is written
// head-merged ([batch, seq_q, heads * d_k], the layout the output projection
// reads) with the absmax partials of every value, so the projection's
// per-tensor quantize needs no extra pass.
#include <math.h>

#include <algorithm>
#include <atomic>

#include "kz_common.cuh"

namespace kz {
namespace {

constexpr int kAttRows = 64;      // query rows per CTA
constexpr int kAttKeys = 64;      // keys per staged K / V tile
constexpr int kAttThreads = 128;  // 8 x 16 threads
constexpr int kAttMaxDk = 128;
constexpr int kAttMaxBlocks = KZ_PARTIALS_WORDS - 3;
// opt-in dynamic shared memory ceiling: 227 KB per CTA less room for the
// kernel's static arrays (the two count together against the limit)
constexpr size_t kAttMaxSmem = 226 * 1024;

struct AttArgs {
    const float* q;
    const float* k;
    const float* v;
    const float* mask;
    float* out;
    uint32_t* partials;
    int64_t q_rs, k_rs, v_rs, o_rs;       // row strides (floats)
    int64_t m_bs, m_hs, m_rs;             // mask strides (floats); key stride 1
    int batch, heads, seq_q, seq_k, d_k;
    int q_blocks, items, s_pitch;
    int causal;
    float scale;
};

__device__ __forceinline__ uint32_t abs_bits_f(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// exp(x) rounded to nearest fp32 from a double-precision exp.
__device__ __forceinline__ float exp_rn(float x) { return __double2float_rn(exp((double)x)); }

// Loads rows [r0, r0 + 64) x d_k of one head (row stride rs) as float4s into
// registers: thread t takes float4 index t + 128 u.  Rows >= nrows read as 0.
template <int DK>
struct TileRegs {
    static constexpr int F4 = kAttRows * DK / 4 / kAttThreads;   // float4 per thread
    float4 r[F4];

    __device__ __forceinline__ void load(const float* base, int64_t rs, int r0, int nrows) {
#pragma unroll
        for (int u = 0; u < F4; ++u) {
            const int f = threadIdx.x + u * kAttThreads;
            const int row = f / (DK / 4), c4 = f % (DK / 4);
            if (r0 + row < nrows)
                r[u] = __ldg(reinterpret_cast<const float4*>(base + (int64_t)(r0 + row) * rs) + c4);
            else
                r[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __device__ __forceinline__ void store(float* tile) const {
#pragma unroll
        for (int u = 0; u < F4; ++u) {
            const int f = threadIdx.x + u * kAttThreads;
            const int row = f / (DK / 4), c4 = f % (DK / 4);
            *reinterpret_cast<float4*>(tile + row * (DK + 4) + 4 * c4) = r[u];
        }
    }
};

template <int DK>
__global__ void __launch_bounds__(kAttThreads, 2) attention_ref_kernel(AttArgs a) {
    constexpr int P = DK + 4;                   // Q / K / V tile pitch
    constexpr int NC = (DK + 63) / 64;          // output column groups per thread
    extern __shared__ __align__(16) float att_smem[];
    float* qs = att_smem;                       // [64][P]
    float* ks = qs + kAttRows * P;              // [64][P], K tiles then V tiles
    float* ss = ks + kAttKeys * P;              // [64][s_pitch] scores -> weights
    __shared__ float s_max[kAttRows];
    __shared__ float s_rinv[kAttRows];
    __shared__ uint32_t red[kAttThreads / 32];
    griddep_launch_dependents();
    griddep_wait();
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;     // keys tx + 16b, rows ty + 8a
    const int sp = a.s_pitch;
    uint32_t amax = 0;

    for (int item = blockIdx.x; item < a.items; item += gridDim.x) {
        const int bh = item % (a.batch * a.heads);
        const int qb = a.q_blocks - 1 - item / (a.batch * a.heads);   // most keys first
        const int b = bh / a.heads, h = bh % a.heads;
        const int i0 = qb * kAttRows;
        const int rows = min(kAttRows, a.seq_q - i0);
        // keys this block needs: all of them, or (causal) up to its last row
        const int kend = a.causal ? min(a.seq_k, i0 + rows) : a.seq_k;
        const int ntiles = (kend + kAttKeys - 1) / kAttKeys;
        const float* qg = a.q + (int64_t)b * a.seq_q * a.q_rs + (int64_t)h * DK;
        const float* kg = a.k + (int64_t)b * a.seq_k * a.k_rs + (int64_t)h * DK;
        const float* vg = a.v + (int64_t)b * a.seq_k * a.v_rs + (int64_t)h * DK;
        const float* mg = a.mask ? a.mask + (int64_t)b * a.m_bs + (int64_t)h * a.m_hs : nullptr;

        TileRegs<DK> pre;
        pre.load(qg, a.q_rs, i0, a.seq_q);
        __syncthreads();                        // the previous item is done with every buffer
        pre.store(qs);
        pre.load(kg, a.k_rs, 0, kend);

        // ---- scores: s[i][j] = ((sum_t q[i][t] * k[j][t]) * scale) (+ mask)
        for (int kt = 0; kt < ntiles; ++kt) {
            __syncthreads();                    // ks free (previous tile consumed)
            pre.store(ks);
            __syncthreads();
            if (kt + 1 < ntiles) pre.load(kg, a.k_rs, (kt + 1) * kAttKeys, kend);
            float acc[8][4];
#pragma unroll
            for (int r = 0; r < 8; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
#pragma unroll 2
            for (int t4 = 0; t4 < DK / 4; ++t4) {
                float4 qv[8], kv[4];
#pragma unroll
                for (int r = 0; r < 8; ++r) qv[r] = *reinterpret_cast<const float4*>(qs + (ty + 8 * r) * P + 4 * t4);
#pragma unroll
                for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(ks + (tx + 16 * c) * P + 4 * t4);
#pragma unroll
                for (int r = 0; r < 8; ++r)
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float s = acc[r][c];
                        s = __fadd_rn(s, __fmul_rn(qv[r].x, kv[c].x));
                        s = __fadd_rn(s, __fmul_rn(qv[r].y, kv[c].y));
                        s = __fadd_rn(s, __fmul_rn(qv[r].z, kv[c].z));
                        s = __fadd_rn(s, __fmul_rn(qv[r].w, kv[c].w));
                        acc[r][c] = s;
                    }
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const int i = ty + 8 * r;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j = kt * kAttKeys + tx + 16 * c;
                    float s = __fmul_rn(acc[r][c], a.scale);
                    if (mg && i < rows && j < kend) s = __fadd_rn(s, __ldg(mg + (int64_t)(i0 + i) * a.m_rs + j));
                    ss[i * sp + j] = s;
                }
            }
        }
        // the first V tile loads while the softmax runs
        pre.load(vg, a.v_rs, 0, kend);
        __syncthreads();

        // ---- softmax over each row's keys j < lim(i): max, exp(s - max), ordered sum, * 1/sum
        const int kpad = ntiles * kAttKeys;
        {
            // row max, two threads per row (order-free)
            const int i = tid >> 1, half = tid & 1;
            const int lim = a.causal ? min(kend, i0 + i + 1) : kend;
            float m = -INFINITY;
            bool any = false;
            for (int j = half; j < lim; j += 2) {
                const float s = ss[i * sp + j];
                if (!any || s > m) m = s;
                any = true;
            }
            const float other = __shfl_xor_sync(0xffffffffu, m, 1);
            const int other_any = __shfl_xor_sync(0xffffffffu, (int)any, 1);
            if (other_any && (!any || other > m)) m = other;
            if (half == 0) s_max[i] = m;
        }
        __syncthreads();
        for (int e = tid; e < kAttRows * (kpad / 4); e += kAttThreads) {
            const int i = e / (kpad / 4), j4 = e % (kpad / 4);
            const int lim = i < rows ? (a.causal ? min(kend, i0 + i + 1) : kend) : 0;
            float4* p = reinterpret_cast<float4*>(ss + i * sp + 4 * j4);
            float4 s = *p;
            const float m = s_max[i];
            const int j = 4 * j4;
            s.x = j + 0 < lim ? exp_rn(__fsub_rn(s.x, m)) : 0.0f;
            s.y = j + 1 < lim ? exp_rn(__fsub_rn(s.y, m)) : 0.0f;
            s.z = j + 2 < lim ? exp_rn(__fsub_rn(s.z, m)) : 0.0f;
            s.w = j + 3 < lim ? exp_rn(__fsub_rn(s.w, m)) : 0.0f;
            *p = s;
        }
        __syncthreads();
        if (tid < kAttRows) {
            // the denominator: one thread per row, keys in ascending order
            const int i = tid;
            const int lim = i < rows ? (a.causal ? min(kend, i0 + i + 1) : kend) : 0;
            const int l4 = (lim + 3) / 4;       // entries past lim are 0: adding them changes nothing
            float d = 0.0f;
            for (int j4 = 0; j4 < l4; ++j4) {
                const float4 e = *reinterpret_cast<const float4*>(ss + i * sp + 4 * j4);
                d = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(d, e.x), e.y), e.z), e.w);
            }
            s_rinv[i] = lim > 0 ? __frcp_rn(d) : 0.0f;
        }
        __syncthreads();
        for (int e = tid; e < kAttRows * (kpad / 4); e += kAttThreads) {
            const int i = e / (kpad / 4), j4 = e % (kpad / 4);
            float4* p = reinterpret_cast<float4*>(ss + i * sp + 4 * j4);
            float4 w = *p;
            const float r = s_rinv[i];
            w.x = __fmul_rn(w.x, r);
            w.y = __fmul_rn(w.y, r);
            w.z = __fmul_rn(w.z, r);
            w.w = __fmul_rn(w.w, r);
            *p = w;
        }

        // ---- attended[i][t] = sum_j w[i][j] * v[j][t], j ascending
        float o[8][NC][4];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int g = 0; g < NC; ++g)
#pragma unroll
                for (int c = 0; c < 4; ++c) o[r][g][c] = 0.0f;
        for (int kt = 0; kt < ntiles; ++kt) {
            __syncthreads();                    // weights final / ks free
            pre.store(ks);
            __syncthreads();
            if (kt + 1 < ntiles) pre.load(vg, a.v_rs, (kt + 1) * kAttKeys, kend);
#pragma unroll 2
            for (int j4 = 0; j4 < kAttKeys / 4; ++j4) {
                float4 wv[8];
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    wv[r] = *reinterpret_cast<const float4*>(ss + (ty + 8 * r) * sp + kt * kAttKeys + 4 * j4);
#pragma unroll
                for (int g = 0; g < NC; ++g) {
                    const int t = 4 * tx + 64 * g;
                    if (t < DK) {
                        float4 vv[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) vv[u] = *reinterpret_cast<const float4*>(ks + (4 * j4 + u) * P + t);
#pragma unroll
                        for (int r = 0; r < 8; ++r) {
                            const float wr[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                o[r][g][0] = __fadd_rn(o[r][g][0], __fmul_rn(wr[u], vv[u].x));
                                o[r][g][1] = __fadd_rn(o[r][g][1], __fmul_rn(wr[u], vv[u].y));
                                o[r][g][2] = __fadd_rn(o[r][g][2], __fmul_rn(wr[u], vv[u].z));
                                o[r][g][3] = __fadd_rn(o[r][g][3], __fmul_rn(wr[u], vv[u].w));
                            }
                        }
                    }
                }
            }
        }
        // ---- head-merged output and its absmax
        float* og = a.out + (int64_t)b * a.seq_q * a.o_rs + (int64_t)h * DK;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int i = ty + 8 * r;
            if (i < rows) {
#pragma unroll
                for (int g = 0; g < NC; ++g) {
                    const int t = 4 * tx + 64 * g;
                    if (t < DK) {
                        const float4 val = make_float4(o[r][g][0], o[r][g][1], o[r][g][2], o[r][g][3]);
                        *reinterpret_cast<float4*>(og + (int64_t)(i0 + i) * a.o_rs + t) = val;
                        amax = max(amax, max(max(abs_bits_f(val.x), abs_bits_f(val.y)),
                                             max(abs_bits_f(val.z), abs_bits_f(val.w))));
                    }
                }
            }
        }
    }
    if (a.partials) {
        amax = warp_max_u32(amax);
        if ((tid & 31) == 0) red[tid >> 5] = amax;
        __syncthreads();
        if (tid == 0) {
            uint32_t m = 0;
            for (int w = 0; w < kAttThreads / 32; ++w) m = max(m, red[w]);
            a.partials[1 + blockIdx.x] = m;
            if (blockIdx.x == 0) a.partials[0] = gridDim.x;
        }
    }
}

template <int DK>
int launch_attention(const AttArgs& a, size_t smem, int grid, cudaStream_t s) {
    static std::atomic<int> attr_set[64];
    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        KZ_CHECK_CUDA(cudaFuncSetAttribute(attention_ref_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kAttMaxSmem));
        if (dev >= 0 && dev < 64) attr_set[dev] = 1;
    }
    KZ_CHECK_CUDA(launch_pdl(attention_ref_kernel<DK>, dim3(grid), dim3(kAttThreads), smem, s, a));
    return KZ_OK;
}

}  // namespace
}  // namespace kz

using namespace kz;

extern "C" int kz_attention_smem_bytes(int64_t seq_k, int64_t d_k) {
    if (seq_k <= 0 || d_k <= 0 || d_k > kAttMaxDk) return 0;
    const int64_t kpad = (seq_k + kAttKeys - 1) / kAttKeys * kAttKeys;
    const int64_t bytes = (int64_t)sizeof(float) * (2 * 64 * (d_k + 4) + kAttRows * (kpad + 4));
    return bytes <= (int64_t)kAttMaxSmem ? (int)bytes : 0;
}

extern "C" int kz_attention_f32(const float* q, const float* k, const float* v, int64_t batch, int64_t heads,
                                int64_t seq_q, int64_t seq_k, int64_t d_k, int64_t q_row_stride,
                                int64_t k_row_stride, int64_t v_row_stride, const float* mask,
                                int64_t mask_batch_stride, int64_t mask_head_stride, int64_t mask_row_stride,
                                int causal, float scale, float* out, int64_t out_row_stride,
                                uint32_t* absmax_partials, kz_stream_t stream) {
    KZ_REQUIRE(batch >= 0 && heads > 0 && seq_q >= 0 && seq_k >= 0, "kz_attention_f32: negative size");
    KZ_REQUIRE(d_k == 32 || d_k == 64 || d_k == 128, "kz_attention_f32: d_k must be 32, 64 or 128");
    KZ_REQUIRE(!causal || seq_q == seq_k, "kz_attention_f32: causal attention needs seq_q == seq_k");
    KZ_REQUIRE(batch * heads * seq_q == 0 || seq_k > 0, "kz_attention_f32: no keys");
    KZ_REQUIRE(batch < (1 << 20) && heads < (1 << 16) && seq_q < (1 << 24) && seq_k < (1 << 24),
               "kz_attention_f32: size out of range");
    if (batch * heads * seq_q == 0) {
        // no values: zero partials (an absmax of 0)
        if (absmax_partials)
            KZ_CHECK_CUDA(cudaMemsetAsync(absmax_partials, 0, sizeof(uint32_t), reinterpret_cast<cudaStream_t>(stream)));
        return KZ_OK;
    }
    KZ_REQUIRE(q && k && v && out, "kz_attention_f32: NULL operand");
    const uintptr_t bits = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                           reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
    KZ_REQUIRE((bits & 15u) == 0, "kz_attention_f32: q, k, v and out must be 16-byte aligned");
    KZ_REQUIRE(q_row_stride % 4 == 0 && k_row_stride % 4 == 0 && v_row_stride % 4 == 0 && out_row_stride % 4 == 0,
               "kz_attention_f32: row strides must be multiples of 4 floats");
    KZ_REQUIRE(q_row_stride >= heads * d_k && k_row_stride >= heads * d_k && v_row_stride >= heads * d_k &&
                   out_row_stride >= heads * d_k,
               "kz_attention_f32: a row stride is shorter than heads * d_k");
    const int smem = kz_attention_smem_bytes(seq_k, d_k);
    KZ_REQUIRE(smem > 0, "kz_attention_f32: seq_k too long for on-chip score rows");
    int st = check_device();
    if (st) return st;
    AttArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.mask = causal ? nullptr : mask;
    a.out = out;
    a.partials = absmax_partials;
    a.q_rs = q_row_stride;
    a.k_rs = k_row_stride;
    a.v_rs = v_row_stride;
    a.o_rs = out_row_stride;
    a.m_bs = mask_batch_stride;
    a.m_hs = mask_head_stride;
    a.m_rs = mask_row_stride;
    a.batch = (int)batch;
    a.heads = (int)heads;
    a.seq_q = (int)seq_q;
    a.seq_k = (int)seq_k;
    a.d_k = (int)d_k;
    a.q_blocks = (int)((seq_q + kAttRows - 1) / kAttRows);
    a.items = (int)(batch * heads) * a.q_blocks;
    a.s_pitch = (int)((seq_k + kAttKeys - 1) / kAttKeys * kAttKeys + 4);
    a.causal = causal ? 1 : 0;
    a.scale = scale;
    const int grid = (int)std::min<int64_t>(a.items, kAttMaxBlocks);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (d_k == 32) return launch_attention<32>(a, smem, grid, s);
    if (d_k == 64) return launch_attention<64>(a, smem, grid, s);
    return launch_attention<128>(a, smem, grid, s);
}
