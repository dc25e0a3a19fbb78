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
// product and every sum is a separately rounded fp32 operation (scalar .rn
// multiplies, packed .rn adds; the file is built with --fmad=false and no
// multiply feeds an add it could be fused with) taken in the reference's
// index order.  The one operation it cannot take from the reference is exp:
// the reference calls the host libm's expf; here exp is rounded correctly
// from a double-precision exp (CUDA's exp(double), error below 1 ulp of
// double), which equals the host's expf wherever that one is correctly
// rounded.
//
// A causal flag replaces causal_mask()'s additive -1e9 entries without
// reading them: those keys get an exponential of exactly 0, so leaving them
// out of the max, the sum and the weighted sum of v changes no bit (adding
// +-0 to a non-zero fp32 sum is exact, and the diagonal key keeps every row's
// sum non-zero).  For the same reason the diagonal tile skips, in both
// products, the groups of 16 rows that lie wholly before a group of keys.
//
// Work decomposition: one CTA per (batch, head, block of 64 query rows), the
// blocks with the most keys (causal) first.  The CTA stages its query rows,
// then 64-key tiles of K, in shared memory (K / V rows at a pitch of d_k + 4
// floats, so the 16-byte reads of 8 consecutive lanes fall in distinct bank
// groups), keeps the block's whole score rows on chip, runs the softmax there
// and streams 64-key tiles of V for the weighted sum.  256 threads, thread
// tile 4 query rows x 4 keys (row pairs ty + 16 rp of rows i, i + 8; keys
// tx + 16 c).  The sums run on sm_100's packed f32x2 add, one instruction per
// two rows, each half rounded as the scalar instruction would (the products
// are scalar multiplies): query rows and score rows are stored
// pair-interleaved so their 16-byte loads give both rows' operands, and per 4
// reduction steps 8 shared loads feed 96 instructions (128 fp32 operations).
// The next tile's global loads are issued into registers before the current
// tile's arithmetic.  The output is written head-merged ([batch, seq_q,
// heads * d_k], the layout the output projection reads) with the absmax
// partials of every value, so the projection's per-tensor quantize needs no
// extra pass.
#include <math.h>

#include <algorithm>
#include <atomic>

#include "kz_common.cuh"

namespace kz {
namespace {

constexpr int kAttRows = 64;      // query rows per CTA
constexpr int kAttKeys = 64;      // keys per staged K / V tile
constexpr int kAttThreads = 256;  // 16 x 16 threads
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
// Below -104 the exponential is under half the smallest subnormal and rounds
// to 0 either way; those inputs (masked scores) skip the double exp.
__device__ __forceinline__ float exp_rn(float x) {
    return x < -104.0f ? 0.0f : __double2float_rn(exp((double)x));
}

// Packed fp32 pairs: sm_100's f32x2 add rounds each half exactly like the
// scalar instruction (round to nearest, subnormals kept), so two separately
// rounded sums cost one instruction.  The products stay scalar multiplies: a
// packed multiply whose only use is a packed add is fused into one packed FMA
// by the code generator (single rounding, even with --fmad=false), while a
// pair of scalar .rn products feeding the packed add is not.
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk(uint64_t r, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
// d = {d.lo + lo * b, d.hi + hi * b}, each product rounded before its sum
__device__ __forceinline__ void mul_add2(uint64_t& d, float lo, float hi, float b) {
    const float p0 = __fmul_rn(lo, b), p1 = __fmul_rn(hi, b);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(d), "l"(pk(p0, p1)));
}

// Row pairs.  Query rows i and i + 8 (i = 16 g + o, o < 8) are one pair, id
// pid = o + 8 g; the pair's values are interleaved in shared memory
// (element (i, x) at pair[2 x + (i / 8) % 2]) so one 16-byte load yields the
// two rows' values at two consecutive x -- ready-made f32x2 operands.
__device__ __forceinline__ int pair_id(int i) { return (i & 7) + 8 * (i >> 4); }
__device__ __forceinline__ int pair_slot(int i) { return (i >> 3) & 1; }
__device__ __forceinline__ int pair_row(int pid, int slot) { return (pid & 7) + 16 * (pid >> 3) + 8 * slot; }

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
    // row-major tile [64][DK + 4] (K and V)
    __device__ __forceinline__ void store(float* tile) const {
#pragma unroll
        for (int u = 0; u < F4; ++u) {
            const int f = threadIdx.x + u * kAttThreads;
            const int row = f / (DK / 4), c4 = f % (DK / 4);
            *reinterpret_cast<float4*>(tile + row * (DK + 4) + 4 * c4) = r[u];
        }
    }
    // row-pair interleaved tile [32][2 DK + 4] (Q)
    __device__ __forceinline__ void store_pairs(float* tile) const {
#pragma unroll
        for (int u = 0; u < F4; ++u) {
            const int f = threadIdx.x + u * kAttThreads;
            const int row = f / (DK / 4), c4 = f % (DK / 4);
            float* d = tile + pair_id(row) * (2 * DK + 4) + 8 * c4 + pair_slot(row);
            d[0] = r[u].x;
            d[2] = r[u].y;
            d[4] = r[u].z;
            d[6] = r[u].w;
        }
    }
};

// A[rp][c] = {s[i][j], s[i + 8][j]} += q[.][t] * k[j][t] for t ascending
// (row pair ty + 16 rp, whose rows lie in the 16-row group 2 rp + ty / 8;
// key j = tx + 16 c of the tile), each product and sum rounded on its own.
// DIAG (causal diagonal tile) skips the pairs whose row group precedes the
// key group (every row before every key; the test is uniform per warp).
template <int DK, bool DIAG>
__device__ __forceinline__ void score_tile(const float* qp, const float* ks, int ty, int tx, uint64_t (&A)[2][4]) {
    constexpr int P = DK + 4, PQ = 2 * DK + 4;
    const int hb = ty >> 3;
#pragma unroll 2
    for (int t4 = 0; t4 < DK / 4; ++t4) {
        float4 qa[2], qb[2], kv[4];
#pragma unroll
        for (int rp = 0; rp < 2; ++rp) {
            const float* row = qp + (ty + 16 * rp) * PQ + 8 * t4;
            qa[rp] = *reinterpret_cast<const float4*>(row);        // t, t + 1
            qb[rp] = *reinterpret_cast<const float4*>(row + 4);    // t + 2, t + 3
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(ks + (tx + 16 * c) * P + 4 * t4);
#define KZ_QK_STEP(QV, LO, HI, KC)                                                   \
        _Pragma("unroll") for (int c = 0; c < 4; ++c)                                \
            _Pragma("unroll") for (int rp = 0; rp < 2; ++rp)                         \
                if (!DIAG || 2 * rp + hb >= c) mul_add2(A[rp][c], QV[rp].LO, QV[rp].HI, kv[c].KC);
        KZ_QK_STEP(qa, x, y, x)
        KZ_QK_STEP(qa, z, w, y)
        KZ_QK_STEP(qb, x, y, z)
        KZ_QK_STEP(qb, z, w, w)
#undef KZ_QK_STEP
    }
}

// O[rp][g][c] = {o[i][t + c], o[i + 8][t + c]} += w[.][j + u] * v[j + u][t + c]
// for u = 0..3 (row pairs ty + 16 rp with rp >= RP0; t = 4 tx + 64 g), each
// product and sum rounded on its own, keys in ascending order.
template <int DK, int RP0>
__device__ __forceinline__ void pv_step(const float* ss, const float* ks, int sp, int ty, int tx, int j, int j4,
                                        uint64_t (&O)[2][(DK + 63) / 64][4]) {
    constexpr int P = DK + 4, NC = (DK + 63) / 64;
    float4 wa[2], wb[2];
#pragma unroll
    for (int rp = RP0; rp < 2; ++rp) {
        const float* w = ss + (ty + 16 * rp) * sp + 2 * j;
        wa[rp] = *reinterpret_cast<const float4*>(w);       // keys j, j + 1
        wb[rp] = *reinterpret_cast<const float4*>(w + 4);   // keys j + 2, j + 3
    }
#pragma unroll
    for (int g = 0; g < NC; ++g) {
        const int t = 4 * tx + 64 * g;
        if (t < DK) {
            float4 vv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) vv[u] = *reinterpret_cast<const float4*>(ks + (4 * j4 + u) * P + t);
#define KZ_PV_STEP(WV, LO, HI, U)                                             \
            _Pragma("unroll") for (int rp = RP0; rp < 2; ++rp) {              \
                mul_add2(O[rp][g][0], WV[rp].LO, WV[rp].HI, vv[U].x);         \
                mul_add2(O[rp][g][1], WV[rp].LO, WV[rp].HI, vv[U].y);         \
                mul_add2(O[rp][g][2], WV[rp].LO, WV[rp].HI, vv[U].z);         \
                mul_add2(O[rp][g][3], WV[rp].LO, WV[rp].HI, vv[U].w);         \
            }
            KZ_PV_STEP(wa, x, y, 0)
            KZ_PV_STEP(wa, z, w, 1)
            KZ_PV_STEP(wb, x, y, 2)
            KZ_PV_STEP(wb, z, w, 3)
#undef KZ_PV_STEP
        }
    }
}

template <int DK>
__global__ void __launch_bounds__(kAttThreads, DK <= 64 ? 2 : 1) attention_ref_kernel(AttArgs a) {
    constexpr int P = DK + 4;                   // K / V tile pitch
    constexpr int PQ = 2 * DK + 4;              // Q row-pair pitch
    constexpr int NC = (DK + 63) / 64;          // output column groups per thread
    extern __shared__ __align__(16) float att_smem[];
    float* qp = att_smem;                       // [32][PQ] query row pairs
    float* ks = qp + (kAttRows / 2) * PQ;       // [64][P], K tiles then V tiles
    float* ss = ks + kAttKeys * P;              // [32][s_pitch] score row pairs -> weights
    __shared__ float s_max[kAttRows];
    __shared__ float s_rinv[kAttRows];
    __shared__ uint32_t red[kAttThreads / 32];
    griddep_launch_dependents();
    griddep_wait();
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;     // keys tx + 16c, row pairs ty + 16rp
    const int sp = a.s_pitch;                   // floats per row pair: 2 x keys + 4
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
        const int kpad = ntiles * kAttKeys;
        const float* qg = a.q + (int64_t)b * a.seq_q * a.q_rs + (int64_t)h * DK;
        const float* kg = a.k + (int64_t)b * a.seq_k * a.k_rs + (int64_t)h * DK;
        const float* vg = a.v + (int64_t)b * a.seq_k * a.v_rs + (int64_t)h * DK;
        const float* mg = a.mask ? a.mask + (int64_t)b * a.m_bs + (int64_t)h * a.m_hs : nullptr;
        // keys row i (of this block) attends to: [0, lim)
        auto row_lim = [&](int i) { return i < rows ? (a.causal ? min(kend, i0 + i + 1) : kend) : 0; };

        TileRegs<DK> pre;
        pre.load(qg, a.q_rs, i0, a.seq_q);
        __syncthreads();                        // the previous item is done with every buffer
        pre.store_pairs(qp);
        pre.load(kg, a.k_rs, 0, kend);

        // ---- scores: s[i][j] = ((sum_t q[i][t] * k[j][t]) * scale) (+ mask)
        for (int kt = 0; kt < ntiles; ++kt) {
            __syncthreads();                    // ks free (previous tile consumed)
            pre.store(ks);
            __syncthreads();
            if (kt + 1 < ntiles) pre.load(kg, a.k_rs, (kt + 1) * kAttKeys, kend);
            uint64_t A[2][4];
#pragma unroll
            for (int rp = 0; rp < 2; ++rp)
#pragma unroll
                for (int c = 0; c < 4; ++c) A[rp][c] = 0ull;    // +0.0f, +0.0f
            if (a.causal && kt == ntiles - 1)
                score_tile<DK, true>(qp, ks, ty, tx, A);
            else
                score_tile<DK, false>(qp, ks, ty, tx, A);
#pragma unroll
            for (int rp = 0; rp < 2; ++rp) {
                const int pid = ty + 16 * rp, il = pair_row(pid, 0), ih = il + 8;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j = kt * kAttKeys + tx + 16 * c;
                    float lo, hi;
                    upk(A[rp][c], lo, hi);
                    lo = __fmul_rn(lo, a.scale);
                    hi = __fmul_rn(hi, a.scale);
                    if (mg && j < kend) {
                        if (il < rows) lo = __fadd_rn(lo, __ldg(mg + (int64_t)(i0 + il) * a.m_rs + j));
                        if (ih < rows) hi = __fadd_rn(hi, __ldg(mg + (int64_t)(i0 + ih) * a.m_rs + j));
                    }
                    *reinterpret_cast<float2*>(ss + pid * sp + 2 * j) = make_float2(lo, hi);
                }
            }
        }
        // the first V tile loads while the softmax runs
        pre.load(vg, a.v_rs, 0, kend);
        __syncthreads();

        // ---- softmax of each row over its keys [0, lim): max, exp(s - max), ordered sum, * 1/sum
        {
            // row-pair max, eight threads per pair (order-free)
            const int pid = tid >> 3, part = tid & 7;
            const int il = pair_row(pid, 0), ih = il + 8;
            const int ll = row_lim(il), lh = row_lim(ih);
            float ml = -INFINITY, mh = -INFINITY;
            for (int j = part; j < max(ll, lh); j += 8) {
                const float2 v = *reinterpret_cast<const float2*>(ss + pid * sp + 2 * j);
                if (j < ll) ml = fmaxf(ml, v.x);
                if (j < lh) mh = fmaxf(mh, v.y);
            }
#pragma unroll
            for (int o = 1; o <= 4; o <<= 1) {
                ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, o));
                mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
            }
            if (part == 0) {
                s_max[il] = ml;
                s_max[ih] = mh;
            }
        }
        __syncthreads();
        // exponentials, keys at or past a row's limit set to exactly 0
        for (int e = tid; e < (kAttRows / 2) * (kpad / 2); e += kAttThreads) {
            const int pid = e / (kpad / 2), j = 2 * (e % (kpad / 2));
            const int il = pair_row(pid, 0), ih = il + 8;
            const int ll = row_lim(il), lh = row_lim(ih);
            const float ml = s_max[il], mh = s_max[ih];
            float4* p = reinterpret_cast<float4*>(ss + pid * sp + 2 * j);
            float4 v = *p;                      // (j, lo) (j, hi) (j + 1, lo) (j + 1, hi)
            v.x = j < ll ? exp_rn(__fsub_rn(v.x, ml)) : 0.0f;
            v.y = j < lh ? exp_rn(__fsub_rn(v.y, mh)) : 0.0f;
            v.z = j + 1 < ll ? exp_rn(__fsub_rn(v.z, ml)) : 0.0f;
            v.w = j + 1 < lh ? exp_rn(__fsub_rn(v.w, mh)) : 0.0f;
            *p = v;
        }
        __syncthreads();
        if (tid < kAttRows / 2) {
            // the denominators: one thread per row pair, each row's keys in ascending order
            const int pid = tid, il = pair_row(pid, 0), ih = il + 8;
            const int lim = max(row_lim(il), row_lim(ih));  // entries past a row's own limit are 0
            float dl = 0.0f, dh = 0.0f;
            for (int j = 0; j < lim; j += 2) {
                const float4 v = *reinterpret_cast<const float4*>(ss + pid * sp + 2 * j);
                dl = __fadd_rn(__fadd_rn(dl, v.x), v.z);
                dh = __fadd_rn(__fadd_rn(dh, v.y), v.w);
            }
            s_rinv[il] = row_lim(il) > 0 ? __frcp_rn(dl) : 0.0f;
            s_rinv[ih] = row_lim(ih) > 0 ? __frcp_rn(dh) : 0.0f;
        }
        __syncthreads();
        for (int e = tid; e < (kAttRows / 2) * (kpad / 2); e += kAttThreads) {
            const int pid = e / (kpad / 2), j = 2 * (e % (kpad / 2));
            const int il = pair_row(pid, 0);
            const float rl = s_rinv[il], rh = s_rinv[il + 8];
            float4* p = reinterpret_cast<float4*>(ss + pid * sp + 2 * j);
            float4 v = *p;
            v.x = __fmul_rn(v.x, rl);
            v.y = __fmul_rn(v.y, rh);
            v.z = __fmul_rn(v.z, rl);
            v.w = __fmul_rn(v.w, rh);
            *p = v;
        }

        // ---- attended[i][t] = sum_j w[i][j] * v[j][t], j ascending
        uint64_t O[2][NC][4];                   // {o[i][t + c], o[i + 8][t + c]}
#pragma unroll
        for (int rp = 0; rp < 2; ++rp)
#pragma unroll
            for (int g = 0; g < NC; ++g)
#pragma unroll
                for (int c = 0; c < 4; ++c) O[rp][g][c] = 0ull;
        for (int kt = 0; kt < ntiles; ++kt) {
            __syncthreads();                    // weights final / ks free
            pre.store(ks);
            __syncthreads();
            if (kt + 1 < ntiles) pre.load(vg, a.v_rs, (kt + 1) * kAttKeys, kend);
            // causal diagonal tile: key segment s (keys 16 s .. 16 s + 15) needs
            // only the row groups g >= s (g = 2 rp + ty / 8); the pairs of an
            // earlier group have weight 0 there (keys after the row), and
            // adding their +-0 products would change no sum
            const bool diag = a.causal && kt == ntiles - 1;
#pragma unroll 2
            for (int j4 = 0; j4 < kAttKeys / 4; ++j4) {
                const int j = kt * kAttKeys + 4 * j4;
                const int rp0 = diag ? max(0, ((j4 >> 2) - (ty >> 3) + 1) >> 1) : 0;   // uniform per warp
                if (rp0 == 0)
                    pv_step<DK, 0>(ss, ks, sp, ty, tx, j, j4, O);
                else if (rp0 == 1)
                    pv_step<DK, 1>(ss, ks, sp, ty, tx, j, j4, O);
            }
        }
        // ---- head-merged output and its absmax
        float* og = a.out + (int64_t)b * a.seq_q * a.o_rs + (int64_t)h * DK;
#pragma unroll
        for (int rp = 0; rp < 2; ++rp) {
            const int il = pair_row(ty + 16 * rp, 0);
#pragma unroll
            for (int g = 0; g < NC; ++g) {
                const int t = 4 * tx + 64 * g;
                if (t < DK) {
                    float lo[4], hi[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) upk(O[rp][g][c], lo[c], hi[c]);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int i = il + 8 * half;
                        if (i < rows) {
                            const float* o = half ? hi : lo;
                            const float4 val = make_float4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<float4*>(og + (int64_t)(i0 + i) * a.o_rs + t) = val;
                            amax = max(amax, max(max(abs_bits_f(val.x), abs_bits_f(val.y)),
                                                 max(abs_bits_f(val.z), abs_bits_f(val.w))));
                        }
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
    // query row pairs [32][2 d_k + 4], one K / V tile [64][d_k + 4], score row pairs [32][2 kpad + 4]
    const int64_t bytes = (int64_t)sizeof(float) * (32 * (2 * d_k + 4) + 64 * (d_k + 4) + 32 * (2 * kpad + 4));
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
    KZ_REQUIRE(batch < (1 << 20) && heads < (1 << 16) && seq_q < (1 << 24) && seq_k < (1 << 24) &&
                   batch * heads * ((seq_q + kAttRows - 1) / kAttRows) < (int64_t)INT32_MAX,
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
    a.s_pitch = (int)(2 * ((seq_k + kAttKeys - 1) / kAttKeys * kAttKeys) + 4);
    a.causal = causal ? 1 : 0;
    a.scale = scale;
    const int grid = (int)std::min<int64_t>(a.items, kAttMaxBlocks);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (d_k == 32) return launch_attention<32>(a, smem, grid, s);
    if (d_k == 64) return launch_attention<64>(a, smem, grid, s);
    return launch_attention<128>(a, smem, grid, s);
}
