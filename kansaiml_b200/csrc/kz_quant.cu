// Scale finding, quantize and dequantize for Kansai's int8 path
// (python/kansai/quantize.py:50-77), as HBM-bound sm_100a kernels.
//
// Rounding contract (bit-exact with the reference): every fp32 element is
// widened to double, scale = (double)max|x| / 127.0 (1.0 if max|x| == 0),
// q = clamp(rint((double)x / scale), -127, 127) with rint rounding half to
// even on the correctly rounded double quotient.
//
// Fast path.  The exact double division per element is replaced by an fp32
// estimate t = fl32(x * r), r = fl32(fl64(1 / scale)).  With |x / scale| <= 127:
//   |r - 1/scale| <= (2^-53 + 2^-24 + 2^-77) / scale
//   |t - x*r|     <= 2^-24 |x*r|   (+2^-149 if t is subnormal)
// so |t - x/scale| < 127 * 2^-22.9 < 2^-16, and the double quotient differs
// from x/scale by at most 128 * 2^-53.  Hence |t - fl64(x/scale)| < 2^-15.
// Whenever t lies at least 2^-15 away from every half-integer
// (|t - rint(t)| <= 1/2 - 2^-15), fl64(x/scale) lies in the same open interval
// (k - 1/2, k + 1/2) and rounds to the same k = rint(t).  The remaining
// elements (about 1 in 2000 for smooth data) take the exact double division.
// t - rint(t) is computed exactly (Sterbenz).  When 1/scale does not fit fp32
// (max|x| < 2^-100) every element takes the exact path.
//
// The fast path rounds with one fp32 add: y = t + 1.5 * 2^23 lies in
// [2^23, 2^24) where floats are the integers, so the add itself rounds t half
// to even, y - 1.5 * 2^23 = rint(t) exactly, and y's bit pattern is
// 0x4B400000 + rint(t), whose low byte is the two's-complement int8 code.  No
// clamp is needed: |t| <= 127 * (1 + 2^-23) * (1 + 2^-24) < 127.5 - 2^-12, so
// rint(t) is in [-127, 127] and never near the 127.5 tie.
//
// The vector form (pack4) folds the multiply into fused multiply-adds:
// y = fl32(x*r + 1.5 * 2^23) gives k = y - 1.5 * 2^23, the integer nearest to
// the exact product x*r, and d = fl32(x*r - k) its residual with one rounding
// (|fl32(d) - d| <= 2^-25).  |x*r - x/scale| <= 127 (1 + 2^-52)(2^-24 + 2^-53
// + 2^-77) < 2^-17.01, so |fl64(x/scale) - k| <= |fl32(d)| + 2^-25 + 2^-17.01
// + 2^-46 < |fl32(d)| + 2^-16.9, and |fl32(d)| <= 1/2 - 2^-16 proves
// k = rint(fl64(x/scale)).  Only the elements that fail the bound (about one in
// 16000 for smooth data) take the exact division.
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <mutex>

#include <cmath>
#include <cstring>

#include "kz_common.cuh"

namespace kz {

constexpr float kTieGuard = 0.5f - 1.0f / 32768.0f;       // scalar form: |t - rint(t)| bound
constexpr float kTieGuardFma = 0.5f - 1.0f / 65536.0f;    // fused-multiply-add form: |d| bound
constexpr uint32_t kInfBits = 0x7F800000u;

__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// ---------------------------------------------------------------- absmax

// Grid-stride max of |x| bits; block b writes partials[1 + b], block 0 writes
// the count.  NaN bit patterns exceed +Inf's, so they survive the max.
__global__ void __launch_bounds__(256) absmax_kernel(const float* __restrict__ x, int64_t n,
                                                     uint32_t* __restrict__ partials) {
    griddep_launch_dependents();
    griddep_wait();
    uint32_t m = 0;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    if (aligned) {
        const int64_t nv = n >> 2;
        const float4* xv = reinterpret_cast<const float4*>(x);
        int64_t i = tid;
        // eight independent 16-byte loads in flight per thread; default caching
        // keeps x in L2 for the quantize pass that follows
        for (; i + 7 * nthreads < nv; i += 8 * nthreads) {
            float4 a[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) a[u] = __ldg(xv + i + u * nthreads);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                m = max(m, max(max(abs_bits(a[u].x), abs_bits(a[u].y)), max(abs_bits(a[u].z), abs_bits(a[u].w))));
        }
        for (; i < nv; i += nthreads) {
            float4 a = __ldg(xv + i);
            m = max(m, max(max(abs_bits(a.x), abs_bits(a.y)), max(abs_bits(a.z), abs_bits(a.w))));
        }
        for (int64_t j = (nv << 2) + tid; j < n; j += nthreads) m = max(m, abs_bits(x[j]));
    } else {
        for (int64_t j = tid; j < n; j += nthreads) m = max(m, abs_bits(x[j]));
    }
    m = warp_max_u32(m);
    __shared__ uint32_t red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) {
            partials[1 + blockIdx.x] = v;
            if (blockIdx.x == 0) partials[0] = gridDim.x;
        }
    }
}

// ------------------------------------------------------- scale + quantize

struct ScaleInfo {
    double scale;   // the reference's double scale
    float rcp;      // fl32(fl64(1 / scale)), fast-path multiplier
    bool fast;      // fast path valid (1/scale representable in fp32)
    bool finite;    // absmax finite
};

__device__ __forceinline__ ScaleInfo scale_from_absmax_bits(uint32_t bits) {
    ScaleInfo si;
    si.finite = bits < kInfBits;
    const float a = __uint_as_float(bits);
    si.scale = a > 0.0f ? (double)a / 127.0 : 1.0;   // quantize.py:68
    si.rcp = __double2float_rn(1.0 / si.scale);
    si.fast = a >= 7.8886090522101181e-31f;           // 2^-100
    return si;
}

__device__ __forceinline__ int8_t quant_exact(float v, double scale) {
    double t = rint((double)v / scale);               // quantize.py:69, IEEE division
    t = fmin(fmax(t, -127.0), 127.0);
    return (int8_t)(int)t;
}

__device__ __forceinline__ int8_t quant_one(float v, const ScaleInfo& si) {
    if (si.fast) {
        const float t = __fmul_rn(v, si.rcp);
        const float tr = rintf(t);
        if (fabsf(t - tr) <= kTieGuard) return (int8_t)(int)fminf(fmaxf(tr, -127.0f), 127.0f);
    }
    return quant_exact(v, si.scale);
}

constexpr float kRoundMagic = 12582912.0f;   // 1.5 * 2^23

// Code of one element by the fused-multiply-add form (see the file header);
// *near is set when the element needs the exact path.
__device__ __forceinline__ uint32_t fma_code(float v, float rcp, bool* near) {
    const float y = __fmaf_rn(v, rcp, kRoundMagic);
    const float d = __fmaf_rn(v, rcp, -__fsub_rn(y, kRoundMagic));
    *near = fabsf(d) > kTieGuardFma;
    return __float_as_uint(y) & 0xFFu;
}

// Exact-path repair of a packed word: only the near-tie bytes are recomputed,
// so a warp with one such element pays for one division.
__device__ __forceinline__ uint32_t pack4_repair(float4 v, uint32_t w, double scale, float rcp, bool fast) {
    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        bool near = true;
        if (fast) fma_code(e[j], rcp, &near);
        if (near) w = (w & ~(0xFFu << (8 * j))) | ((uint32_t)(uint8_t)quant_exact(e[j], scale) << (8 * j));
    }
    return w;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: each lane rounds exactly like
// the scalar instruction, so results are bit-identical).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Fast-path word of four codes (little-endian) and the largest |residual| of
// the four; residuals above kTieGuardFma mark elements for pack4_repair.
// Per pair: y = fl(x*r + M), -k = M - y (exact), d = fl(x*r - k).
__device__ __forceinline__ uint32_t pack4_fast(const float4& v, float rcp, float& dmax) {
    const uint64_t R = pk2(rcp, rcp), Mg = pk2(kRoundMagic, kRoundMagic);
    const uint64_t v01 = pk2(v.x, v.y), v23 = pk2(v.z, v.w);
    const uint64_t y01 = fma2(v01, R, Mg), y23 = fma2(v23, R, Mg);
    const uint64_t d01 = fma2(v01, R, sub2(Mg, y01)), d23 = fma2(v23, R, sub2(Mg, y23));
    float y0, y1, y2, y3, d0, d1, d2, d3;
    upk2(y01, y0, y1);
    upk2(y23, y2, y3);
    upk2(d01, d0, d1);
    upk2(d23, d2, d3);
    const uint32_t lo01 = __byte_perm(__float_as_uint(y0), __float_as_uint(y1), 0x0040);
    const uint32_t lo23 = __byte_perm(__float_as_uint(y2), __float_as_uint(y3), 0x0040);
    dmax = fmaxf(fmaxf(fabsf(d0), fabsf(d1)), fmaxf(fabsf(d2), fabsf(d3)));
    return __byte_perm(lo01, lo23, 0x5410);
}

// Sixteen codes from four float4: one tie check (one branch) for all of them,
// so the four independent chains interleave.
__device__ __forceinline__ uint4 pack16(const float4& a, const float4& b, const float4& c, const float4& d,
                                        const ScaleInfo& si) {
    float m0, m1, m2, m3;
    uint4 w;
    w.x = pack4_fast(a, si.rcp, m0);
    w.y = pack4_fast(b, si.rcp, m1);
    w.z = pack4_fast(c, si.rcp, m2);
    w.w = pack4_fast(d, si.rcp, m3);
    if (!si.fast || fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) > kTieGuardFma) {
        if (!si.fast || m0 > kTieGuardFma) w.x = pack4_repair(a, w.x, si.scale, si.rcp, si.fast);
        if (!si.fast || m1 > kTieGuardFma) w.y = pack4_repair(b, w.y, si.scale, si.rcp, si.fast);
        if (!si.fast || m2 > kTieGuardFma) w.z = pack4_repair(c, w.z, si.scale, si.rcp, si.fast);
        if (!si.fast || m3 > kTieGuardFma) w.w = pack4_repair(d, w.w, si.scale, si.rcp, si.fast);
    }
    return w;
}

// Four codes packed little-endian into one word: three fp32 operations per
// element and one tie check per four; a word with a near-tie element is
// repaired per element.
__device__ __forceinline__ uint32_t pack4(const float4& v, const ScaleInfo& si) {
    float dm;
    const uint32_t w = pack4_fast(v, si.rcp, dm);
    if (si.fast && dm <= kTieGuardFma) return w;
    return pack4_repair(v, w, si.scale, si.rcp, si.fast);
}

// Reduce a partials buffer inside one block and derive the scale once (the
// double divisions run on one thread); every thread gets the result.
__device__ __forceinline__ ScaleInfo block_scale_from_partials(const uint32_t* __restrict__ partials) {
    __shared__ uint32_t red[32];
    __shared__ ScaleInfo result;
    const uint32_t count = min(partials[0], (uint32_t)(KZ_PARTIALS_WORDS - 3));
    uint32_t m = 0;
    for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) m = max(m, partials[1 + i]);
    m = warp_max_u32(m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) result = scale_from_absmax_bits(v);
    }
    __syncthreads();
    return result;
}

__global__ void __launch_bounds__(256) quantize_partials_kernel(const float* __restrict__ x, int64_t n,
                                                                const uint32_t* __restrict__ partials,
                                                                int8_t* __restrict__ q, double* scale_out,
                                                                float* scale_f32_out, int* status) {
    griddep_launch_dependents();
    griddep_wait();
    const ScaleInfo si = block_scale_from_partials(partials);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (si.finite) {
            *scale_out = si.scale;
            if (scale_f32_out) *scale_f32_out = __double2float_rn(si.scale);
        } else {
            *scale_out = __longlong_as_double(0x7FF8000000000000ll);
            if (scale_f32_out) *scale_f32_out = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15u) == 0;
    if (!si.finite) {
        for (int64_t j = tid; j < n; j += nthreads) q[j] = 0;
        return;
    }
    if (aligned) {
        // 16 elements per thread per step: 64 B in, one 16 B store out.
        const int64_t n16 = n >> 4;
        const float4* xv = reinterpret_cast<const float4*>(x);
        uint4* qv = reinterpret_cast<uint4*>(q);
        for (int64_t i = tid; i < n16; i += nthreads) {
            const float4 a = __ldcs(xv + 4 * i), b = __ldcs(xv + 4 * i + 1);
            const float4 c = __ldcs(xv + 4 * i + 2), d = __ldcs(xv + 4 * i + 3);
            qv[i] = pack16(a, b, c, d, si);   // default policy: the int8 GEMM reads the codes next
        }
        for (int64_t j = (n16 << 4) + tid; j < n; j += nthreads) q[j] = quant_one(x[j], si);
    } else {
        for (int64_t j = tid; j < n; j += nthreads) q[j] = quant_one(x[j], si);
    }
}

// ----------------------------------------- fused absmax + quantize (1 launch)

// Word of the partials buffer the fused kernels use as their grid barrier.
// It must be zero before the first use of a buffer; every completed launch
// leaves its low 31 bits at zero and flips bit 31.
constexpr int kBarrierWord = KZ_PARTIALS_WORDS - 2;
constexpr int kFusedMaxBlocks = KZ_PARTIALS_WORDS - 3;

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded sense-reversal grid barrier for a cooperative launch (all blocks
// co-resident), one atomic per block: block 0 adds 2^31 - (G - 1), every other
// block adds 1.  Whatever the arrival order, bit 31 of the word keeps its old
// value until the G-th arrival and flips with it, and the low 31 bits end where
// they started (zero).  Each block waits until bit 31 differs from the value
// it saw on arrival.  Returns false after recording KZ_ERR_DEVICE_TIMEOUT when
// the wait runs out.
__device__ __forceinline__ bool grid_barrier(uint32_t* partials, int* status) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t* word = partials + kBarrierWord;
        const uint32_t add = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
        uint32_t old;   // release: this block's partial is visible before the arrival
        asm volatile("atom.release.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(word), "r"(add) : "memory");
        ok = 1;
        const uint64_t t0 = globaltimer_ns();
        uint32_t it = 0;
        while (((ld_acquire_gpu(word) ^ old) & 0x80000000u) == 0) {
            if ((++it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
                record_status(status, KZ_ERR_DEVICE_TIMEOUT);
                ok = 0;
                break;
            }
        }
        // the acquire load that saw the flip orders this block's later reads
        // (the other threads' through the __syncthreads below)
    }
    __syncthreads();
    return ok != 0;
}

// One launch: phase 1 writes each block's partial absmax, a grid barrier, then
// phase 2 reduces the partials, derives the scale and quantizes (x is re-read
// while still in L2).  Same arithmetic as absmax_kernel + quantize_partials_kernel.
__global__ void __launch_bounds__(1024, 1) quantize_fused_kernel(const float* __restrict__ x, int64_t n,
                                                             uint32_t* __restrict__ partials, int8_t* __restrict__ q,
                                                             double* scale_out, float* scale_f32_out, int* status) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15u) == 0;
    const float4* xv = reinterpret_cast<const float4*>(x);
    // phase 1: block absmax
    uint32_t m = 0;
    if (aligned) {
        const int64_t nv = n >> 2;
        int64_t i = tid;
        for (; i + 7 * nthreads < nv; i += 8 * nthreads) {
            float4 a[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) a[u] = __ldg(xv + i + u * nthreads);
#pragma unroll
            for (int u = 0; u < 8; ++u)
                m = max(m, max(max(abs_bits(a[u].x), abs_bits(a[u].y)), max(abs_bits(a[u].z), abs_bits(a[u].w))));
        }
        for (; i < nv; i += nthreads) {
            const float4 a = __ldg(xv + i);
            m = max(m, max(max(abs_bits(a.x), abs_bits(a.y)), max(abs_bits(a.z), abs_bits(a.w))));
        }
        for (int64_t j = (nv << 2) + tid; j < n; j += nthreads) m = max(m, abs_bits(x[j]));
    } else {
        for (int64_t j = tid; j < n; j += nthreads) m = max(m, abs_bits(x[j]));
    }
    m = warp_max_u32(m);
    __shared__ uint32_t red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) {
            partials[1 + blockIdx.x] = v;
            if (blockIdx.x == 0) partials[0] = gridDim.x;
        }
    }
    if (!grid_barrier(partials, status)) return;
    // phase 2: global absmax -> scale -> codes
    uint32_t bits = 0;
    for (uint32_t i = threadIdx.x; i < gridDim.x; i += blockDim.x) bits = max(bits, __ldcg(partials + 1 + i));
    bits = warp_max_u32(bits);
    __syncthreads();
    if (lane == 0) red[warp] = bits;
    __syncthreads();
    __shared__ ScaleInfo s_si;
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) s_si = scale_from_absmax_bits(v);
    }
    __syncthreads();
    const ScaleInfo si = s_si;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (si.finite) {
            *scale_out = si.scale;
            if (scale_f32_out) *scale_f32_out = __double2float_rn(si.scale);
        } else {
            *scale_out = __longlong_as_double(0x7FF8000000000000ll);
            if (scale_f32_out) *scale_f32_out = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    if (!si.finite) {
        for (int64_t j = tid; j < n; j += nthreads) q[j] = 0;
        return;
    }
    if (aligned) {
        const int64_t n16 = n >> 4;
        uint4* qv = reinterpret_cast<uint4*>(q);
        for (int64_t i = tid; i < n16; i += nthreads) {
            const float4 a = __ldcs(xv + 4 * i), b = __ldcs(xv + 4 * i + 1);
            const float4 c = __ldcs(xv + 4 * i + 2), d = __ldcs(xv + 4 * i + 3);
            qv[i] = pack16(a, b, c, d, si);
        }
        for (int64_t j = (n16 << 4) + tid; j < n; j += nthreads) q[j] = quant_one(x[j], si);
    } else {
        for (int64_t j = tid; j < n; j += nthreads) q[j] = quant_one(x[j], si);
    }
}

// Shared-memory-resident variant of the fused quantize: block b owns the
// contiguous chunk [b * chunk, (b + 1) * chunk) of x; the first `cap` bytes of
// it arrive by bulk copy into shared memory (one HBM read at full bandwidth)
// in 32 KB pieces, each with its own mbarrier so that its absmax is taken
// while the later pieces are still in flight, and stay there for both passes;
// any remainder beyond `cap` is read from global memory in both passes.  x and
// q must be 16-byte aligned and chunk a multiple of 16 elements.
constexpr int kResidentBlock = 1024;
constexpr uint32_t kBulkPiece = 32768;
constexpr int kMaxPieces = 8;   // 8 x 32 KB covers the largest resident chunk (< 227 KB)

__global__ void __launch_bounds__(kResidentBlock, 1)
    quantize_resident_kernel(const float* __restrict__ x, int64_t n, int64_t chunk, uint32_t cap_floats,
                             uint32_t* __restrict__ partials, int8_t* __restrict__ q, double* scale_out,
                             float* scale_f32_out, int* status) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);
    __shared__ uint64_t bars[kMaxPieces];   // one per bulk piece, so each piece is reduced as it lands
    __shared__ uint32_t red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t e0 = blockIdx.x * chunk;
    const int64_t e1 = min(n, e0 + chunk);
    const int64_t len = max((int64_t)0, e1 - e0);
    // resident floats (x4; at most kMaxPieces pieces, checked on the host)
    const uint32_t res = (uint32_t)min((int64_t)cap_floats, len & ~(int64_t)3);
    const uint32_t pieces = (res * 4u + kBulkPiece - 1) / kBulkPiece;
    const uint32_t bar0 = smem_u32(bars);
    if (threadIdx.x < pieces) mbar_init(bar0 + 8 * threadIdx.x, 1);
    if (threadIdx.x == 0) fence_mbarrier_init();
    __syncthreads();
    griddep_launch_dependents();
    griddep_wait();
    if (threadIdx.x == 0) {
        const char* src = reinterpret_cast<const char*>(x + e0);
        for (uint32_t k = 0; k < pieces; ++k) {
            const uint32_t off = k * kBulkPiece, bytes = min(kBulkPiece, res * 4u - off);
            mbar_arrive_expect_tx(bar0 + 8 * k, bytes);
            bulk_load(smem_u32(smem_raw) + off, src + off, bytes, bar0 + 8 * k);
        }
    }
    // phase 1: absmax of the non-resident remainder while the copy is in flight.
    // When res < len the remainder starts at e0 + cap, a multiple of 16 elements.
    uint32_t m = 0;
    const int64_t r0 = e0 + res;
    const int64_t rem4 = (e1 - r0) >> 2;
    const float4* xr4 = reinterpret_cast<const float4*>(x + r0);
    for (int64_t i = threadIdx.x; i < rem4; i += blockDim.x) {
        const float4 a = __ldg(xr4 + i);
        m = max(m, max(max(abs_bits(a.x), abs_bits(a.y)), max(abs_bits(a.z), abs_bits(a.w))));
    }
    for (int64_t j = r0 + 4 * rem4 + threadIdx.x; j < e1; j += blockDim.x) m = max(m, abs_bits(x[j]));
    // then each resident piece as soon as it has landed
    bool ok = true;
    const float4* xs4 = reinterpret_cast<const float4*>(xs);
    constexpr uint32_t kPieceVec = kBulkPiece / 16;   // float4 per piece
    for (uint32_t k = 0; ok && k < pieces; ++k) {
        ok = mbar_wait(bar0 + 8 * k, 0, status, nullptr);
        if (!ok) break;
        const uint32_t end = min(res / 4, (k + 1) * kPieceVec);
        for (uint32_t i = k * kPieceVec + threadIdx.x; i < end; i += blockDim.x) {
            const float4 a = xs4[i];
            m = max(m, max(max(abs_bits(a.x), abs_bits(a.y)), max(abs_bits(a.z), abs_bits(a.w))));
        }
    }
    m = warp_max_u32(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) {
            partials[1 + blockIdx.x] = v;
            if (blockIdx.x == 0) partials[0] = gridDim.x;
        }
    }
    if (!grid_barrier(partials, status) || !ok) return;
    // phase 2: global absmax (one partial per thread) -> scale -> codes
    uint32_t bits = 0;
    for (uint32_t i = threadIdx.x; i < gridDim.x; i += blockDim.x) bits = max(bits, __ldcg(partials + 1 + i));
    bits = warp_max_u32(bits);
    __syncthreads();
    if (lane == 0) red[warp] = bits;
    __syncthreads();
    __shared__ ScaleInfo s_si;
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) s_si = scale_from_absmax_bits(v);
    }
    __syncthreads();
    const ScaleInfo si = s_si;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (si.finite) {
            *scale_out = si.scale;
            if (scale_f32_out) *scale_f32_out = __double2float_rn(si.scale);
        } else {
            *scale_out = __longlong_as_double(0x7FF8000000000000ll);
            if (scale_f32_out) *scale_f32_out = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    if (!si.finite) {
        for (int64_t j = e0 + threadIdx.x; j < e1; j += blockDim.x) q[j] = 0;
        return;
    }
    // resident part: consecutive threads read consecutive 16 B of shared memory
    // (no bank conflicts) and store 4 codes each (128 B per warp).
    uint32_t* qw = reinterpret_cast<uint32_t*>(q + e0);
    constexpr uint32_t B = kResidentBlock;
    uint32_t i = threadIdx.x;
    for (; i + 3 * B < res / 4; i += 4 * B) {
        const uint4 w = pack16(xs4[i], xs4[i + B], xs4[i + 2 * B], xs4[i + 3 * B], si);
        qw[i] = w.x;
        qw[i + B] = w.y;
        qw[i + 2 * B] = w.z;
        qw[i + 3 * B] = w.w;
    }
    for (; i < res / 4; i += B) qw[i] = pack4(xs4[i], si);
    uint32_t* qr = reinterpret_cast<uint32_t*>(q + r0);
    for (int64_t i = threadIdx.x; i < rem4; i += blockDim.x) qr[i] = pack4(__ldcs(xr4 + i), si);
    for (int64_t j = r0 + 4 * rem4 + threadIdx.x; j < e1; j += blockDim.x) q[j] = quant_one(x[j], si);
}

// ------------------------------------------- LayerNorm with absmax partials

// LayerNorm over the last axis in the reference's operation order
// (nn.py:323-331):
//   mean = sum(dim) * fl32(1/D)          sum(dim): Ops.cpp:157-190 reduce_to_shape
//                                        adds the row's elements one at a time
//                                        in index order, from 0.0f; the scale is
//                                        a broadcast fp32 mul (Tensor.cpp:864-880)
//   centered = x - mean
//   var = sum(dim)(centered * centered) * fl32(1/D)
//   y = centered * fl32(1 / sqrt(var + eps)) * gamma + beta
//                                        (Tensor::div is mul by reciprocal,
//                                        Tensor.cpp:677-679)
// every step one fp32 operation rounded to nearest (the reference's x86-64
// build has no fused multiply-add), so y equals the reference's LayerNorm bit
// for bit.  NULL gamma / beta act as the reference's initial ones / zeros
// (the + 0.0f still turns a -0.0 into +0.0, as the reference's add does).
//
// A block owns kLnRows rows.  Staged form (D % 4 == 0, 16-byte aligned rows,
// kLnRows rows fit in shared memory): all threads copy the rows in with
// coalesced 16-byte loads (adding the residual and writing the sum when there
// is one), then lane r of warp 0 walks row r serially from shared memory --
// the sums must run in index order, and one thread per row keeps the order
// without a cross-lane combine -- reading 16 bytes at a time (the row pitch
// is 16 bytes times an odd number modulo 128, so the eight lanes of each
// quarter-warp hit distinct bank groups), and finally all threads write y with
// coalesced 16-byte stores and take its absmax.  Otherwise the same
// arithmetic reads global memory directly.
constexpr int kLnRows = 16;
constexpr int kLnThreads = 128;
constexpr int kLnBatch = 8;   // 16-byte loads in flight per thread while staging rows

__global__ void __launch_bounds__(kLnThreads) layernorm_partials_kernel(
    const float* __restrict__ x, int64_t M, int64_t D, const float* __restrict__ gamma,
    const float* __restrict__ beta, float eps, float* __restrict__ y, uint32_t* __restrict__ partials,
    const float* __restrict__ res, float* __restrict__ sum_out, int staged, int stride) {
    extern __shared__ __align__(16) float ln_rows[];
    __shared__ float s_mean[kLnRows], s_rden[kLnRows];
    __shared__ uint32_t red[kLnThreads / 32];
    griddep_launch_dependents();
    griddep_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float inv_d = __frcp_rn((float)D);
    const int64_t D4 = D >> 2;
    uint32_t m = 0;
    for (int64_t r0 = (int64_t)blockIdx.x * kLnRows; r0 < M; r0 += (int64_t)gridDim.x * kLnRows) {
        const int rows = (int)min((int64_t)kLnRows, M - r0);
        if (staged) {
            // rows in: ln_rows[r * stride + j] = x (+ res); batches of kLnBatch
            // 16-byte loads per thread are issued before any is used
            const int d4 = (int)D4;
            const int total = rows * d4;
            const float4* x4 = reinterpret_cast<const float4*>(x) + r0 * D4;
            const float4* res4 = res ? reinterpret_cast<const float4*>(res) + r0 * D4 : nullptr;
            for (int t0 = threadIdx.x; t0 < total; t0 += kLnThreads * kLnBatch) {
                float4 v[kLnBatch], w[kLnBatch];
#pragma unroll
                for (int u = 0; u < kLnBatch; ++u) {
                    const int t = t0 + u * kLnThreads;
                    if (t < total) {
                        v[u] = __ldg(x4 + t);
                        if (res4) w[u] = __ldg(res4 + t);
                    }
                }
#pragma unroll
                for (int u = 0; u < kLnBatch; ++u) {
                    const int t = t0 + u * kLnThreads;
                    if (t < total) {
                        const int r = t / d4;
                        const int c = t - r * d4;
                        float4 a = v[u];
                        if (res4) {
                            a.x = __fadd_rn(a.x, w[u].x);
                            a.y = __fadd_rn(a.y, w[u].y);
                            a.z = __fadd_rn(a.z, w[u].z);
                            a.w = __fadd_rn(a.w, w[u].w);
                            reinterpret_cast<float4*>(sum_out)[r0 * D4 + t] = a;
                        }
                        *reinterpret_cast<float4*>(ln_rows + (int64_t)r * stride + 4 * c) = a;
                    }
                }
            }
            __syncthreads();
            if (warp == 0 && lane < rows) {
                const float4* row = reinterpret_cast<const float4*>(ln_rows + (int64_t)lane * stride);
                float s = 0.0f;
#pragma unroll 8
                for (int c = 0; c < d4; ++c) {
                    const float4 v = row[c];
                    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
                }
                const float mean = __fmul_rn(s, inv_d);
                float q = 0.0f;
#pragma unroll 8
                for (int c = 0; c < d4; ++c) {
                    const float4 v = row[c];
                    const float a = __fsub_rn(v.x, mean), b = __fsub_rn(v.y, mean);
                    const float e = __fsub_rn(v.z, mean), f = __fsub_rn(v.w, mean);
                    q = __fadd_rn(q, __fmul_rn(a, a));
                    q = __fadd_rn(q, __fmul_rn(b, b));
                    q = __fadd_rn(q, __fmul_rn(e, e));
                    q = __fadd_rn(q, __fmul_rn(f, f));
                }
                s_mean[lane] = mean;
                s_rden[lane] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(q, inv_d), eps)));
            }
            __syncthreads();
            for (int t = threadIdx.x; t < rows * d4; t += kLnThreads) {
                const int r = t / d4;
                const int c = t - r * d4;
                const float mean = s_mean[r], rden = s_rden[r];
                const float4 v = *reinterpret_cast<const float4*>(ln_rows + (int64_t)r * stride + 4 * c);
                const float4 gm = gamma ? __ldg(reinterpret_cast<const float4*>(gamma) + c) : make_float4(1.f, 1.f, 1.f, 1.f);
                const float4 bt = beta ? __ldg(reinterpret_cast<const float4*>(beta) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                float4 o;
                o.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mean), rden), gm.x), bt.x);
                o.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mean), rden), gm.y), bt.y);
                o.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mean), rden), gm.z), bt.z);
                o.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mean), rden), gm.w), bt.w);
                reinterpret_cast<float4*>(y)[(r0 + r) * D4 + c] = o;
                m = max(m, max(max(abs_bits(o.x), abs_bits(o.y)), max(abs_bits(o.z), abs_bits(o.w))));
            }
            __syncthreads();   // ln_rows and the row statistics are reused by the next row group
        } else {
            auto val = [&](int64_t i) { return res ? __fadd_rn(x[i], res[i]) : x[i]; };
            if (warp == 0 && lane < rows) {
                const int64_t base = (r0 + lane) * D;
                float s = 0.0f;
                for (int64_t j = 0; j < D; ++j) s = __fadd_rn(s, val(base + j));
                const float mean = __fmul_rn(s, inv_d);
                float q = 0.0f;
                for (int64_t j = 0; j < D; ++j) {
                    const float a = __fsub_rn(val(base + j), mean);
                    q = __fadd_rn(q, __fmul_rn(a, a));
                }
                s_mean[lane] = mean;
                s_rden[lane] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(q, inv_d), eps)));
            }
            __syncthreads();
            for (int64_t t = threadIdx.x; t < rows * D; t += kLnThreads) {
                const int r = (int)(t / D);
                const int64_t j = t - r * D;
                const int64_t i = (r0 + r) * D + j;
                const float v = val(i);
                if (res) sum_out[i] = v;
                const float gm = gamma ? gamma[j] : 1.0f, bt = beta ? beta[j] : 0.0f;
                const float o = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, s_mean[r]), s_rden[r]), gm), bt);
                y[i] = o;
                m = max(m, abs_bits(o));
            }
            __syncthreads();
        }
    }
    m = warp_max_u32(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t v = 0;
        for (int w = 0; w < kLnThreads / 32; ++w) v = max(v, red[w]);
        partials[1 + blockIdx.x] = v;
        if (blockIdx.x == 0) partials[0] = gridDim.x;
    }
}

// ------------------------------------------------------ per-column (weights)

// Column absmax partials: partial[r][n] = max over rows of split r of |w[k][n]|.
// Block (32, 8): threadIdx.x walks 32 adjacent columns (128 B coalesced rows),
// threadIdx.y strides rows.
__global__ void __launch_bounds__(256) absmax_cols_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                                          int64_t rows_per_split, uint32_t* __restrict__ partial) {
    const int64_t n = blockIdx.x * 32 + threadIdx.x;
    const int64_t k0 = blockIdx.y * rows_per_split;
    const int64_t k1 = min(K, k0 + rows_per_split);
    uint32_t m = 0;
    if (n < N)
        for (int64_t k = k0 + threadIdx.y; k < k1; k += 8) m = max(m, abs_bits(__ldg(w + k * N + n)));
    __shared__ uint32_t red[8][33];
    red[threadIdx.y][threadIdx.x] = m;
    __syncthreads();
    if (threadIdx.y == 0 && n < N) {
#pragma unroll
        for (int i = 1; i < 8; ++i) m = max(m, red[i][threadIdx.x]);
        partial[blockIdx.y * N + n] = m;
    }
}

// Transposing quantize: tile of 128 rows (k) x 32 columns (n) of w[K, N] ->
// qT[n][k0 .. k0 + 128).  Thread x owns column n0 + x for the whole tile, so it
// derives that column's scale once from the split partials.
__global__ void __launch_bounds__(256) quantize_cols_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                                            const uint32_t* __restrict__ partial, int splits,
                                                            int8_t* __restrict__ qT, double* scales,
                                                            float* scales_f32, int* status) {
    __shared__ __align__(16) int8_t tile[32][128 + 16];
    const int64_t n0 = blockIdx.x * 32;
    const int64_t k0 = blockIdx.y * 128;
    const int64_t n = n0 + threadIdx.x;
    uint32_t bits = 0;
    if (n < N)
        for (int r = 0; r < splits; ++r) bits = max(bits, partial[r * N + n]);
    const ScaleInfo si = scale_from_absmax_bits(bits);
    if (blockIdx.y == 0 && threadIdx.y == 0 && n < N) {
        if (si.finite) {
            scales[n] = si.scale;
            if (scales_f32) scales_f32[n] = __double2float_rn(si.scale);
        } else {
            scales[n] = __longlong_as_double(0x7FF8000000000000ll);
            if (scales_f32) scales_f32[n] = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    for (int kk = threadIdx.y; kk < 128; kk += 8) {
        const int64_t k = k0 + kk;
        int8_t v = 0;
        if (n < N && k < K && si.finite) v = quant_one(__ldg(w + k * N + n), si);
        tile[threadIdx.x][kk] = v;
    }
    __syncthreads();
    // write out: 32 rows of qT x 128 bytes; thread t -> row t / 8, 16-byte chunk t % 8
    const int t = threadIdx.y * 32 + threadIdx.x;
    const int row = t >> 3, chunk = t & 7;
    const int64_t nn = n0 + row;
    const int64_t kb = k0 + chunk * 16;
    if (nn < N && kb < K) {
        int8_t* dst = qT + nn * K + kb;
        if (kb + 16 <= K && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&tile[row][chunk * 16]);
        } else {
            for (int j = 0; j < 16 && kb + j < K; ++j) dst[j] = tile[row][chunk * 16 + j];
        }
    }
}

// Vectorised forms for the common case (N % 4 == 0, K % 16 == 0, 16-byte
// aligned w and qT).  A block is 256 threads over a tile of 64 columns: thread
// t owns columns n0 + 4 (t % 16) .. + 3 (one 16-byte load per row) and 16
// consecutive rows starting at 16 (t / 16), so a warp reads two 256-byte row
// segments per load and every thread has 16 independent 16-byte loads in
// flight.
constexpr int kColTile = 64;
constexpr int kColRowsPerThread = 16;
constexpr int kColRowsPerPass = 16 * kColRowsPerThread;   // 256 rows per block pass

// partial[split][n] = max |w[k][n]| over the split's rows (bit patterns).
__global__ void __launch_bounds__(256) absmax_cols4_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                                           int64_t rows_per_split, uint32_t* __restrict__ partial) {
    __shared__ uint32_t red[16][kColTile + 1];
    const int cg = threadIdx.x & 15, rg = threadIdx.x >> 4;
    const int64_t n = (int64_t)blockIdx.x * kColTile + 4 * cg;
    const int64_t k0 = blockIdx.y * rows_per_split;
    const int64_t k1 = min(K, k0 + rows_per_split);
    uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
    if (n < N) {
        for (int64_t kb = k0 + rg * kColRowsPerThread; kb < k1; kb += kColRowsPerPass) {
            float4 v[kColRowsPerThread];
#pragma unroll
            for (int i = 0; i < kColRowsPerThread; ++i)
                v[i] = kb + i < k1 ? __ldg(reinterpret_cast<const float4*>(w + (kb + i) * N + n))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < kColRowsPerThread; ++i) {
                m0 = max(m0, abs_bits(v[i].x));
                m1 = max(m1, abs_bits(v[i].y));
                m2 = max(m2, abs_bits(v[i].z));
                m3 = max(m3, abs_bits(v[i].w));
            }
        }
    }
    red[rg][4 * cg] = m0;
    red[rg][4 * cg + 1] = m1;
    red[rg][4 * cg + 2] = m2;
    red[rg][4 * cg + 3] = m3;
    __syncthreads();
    if (threadIdx.x < kColTile) {
        const int64_t c = (int64_t)blockIdx.x * kColTile + threadIdx.x;
        uint32_t m = 0;
#pragma unroll
        for (int r = 0; r < 16; ++r) m = max(m, red[r][threadIdx.x]);
        if (c < N) partial[blockIdx.y * N + c] = m;
    }
}

// Transposing quantize of 64 columns x 256 rows: each thread turns its 16
// rows x 4 columns into four 16-byte runs of K-major codes, one per column,
// each quantized with that column's scale (pack16: fast path + exact repair).
__global__ void __launch_bounds__(256) quantize_cols4_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                                             const uint32_t* __restrict__ partial, int splits,
                                                             int8_t* __restrict__ qT, double* scales,
                                                             float* scales_f32, int* status) {
    __shared__ ScaleInfo s_si[kColTile];
    const int64_t n0 = (int64_t)blockIdx.x * kColTile;
    if (threadIdx.x < kColTile) {
        const int64_t n = n0 + threadIdx.x;
        uint32_t bits = 0;
        if (n < N)
            for (int r = 0; r < splits; ++r) bits = max(bits, partial[r * N + n]);
        const ScaleInfo si = scale_from_absmax_bits(bits);
        s_si[threadIdx.x] = si;
        if (blockIdx.y == 0 && n < N) {
            if (si.finite) {
                scales[n] = si.scale;
                if (scales_f32) scales_f32[n] = __double2float_rn(si.scale);
            } else {
                scales[n] = __longlong_as_double(0x7FF8000000000000ll);
                if (scales_f32) scales_f32[n] = __uint_as_float(0x7FC00000u);
                record_status(status, KZ_ERR_NONFINITE);
            }
        }
    }
    __syncthreads();
    const int cg = threadIdx.x & 15, rg = threadIdx.x >> 4;
    const int64_t n = n0 + 4 * cg;
    const int64_t k = (int64_t)blockIdx.y * kColRowsPerPass + rg * kColRowsPerThread;
    if (n >= N || k >= K) return;
    float4 v[kColRowsPerThread];
#pragma unroll
    for (int i = 0; i < kColRowsPerThread; ++i) v[i] = __ldcs(reinterpret_cast<const float4*>(w + (k + i) * N + n));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const ScaleInfo si = s_si[4 * cg + j];
        auto col = [&](int i) { return j == 0 ? v[i].x : j == 1 ? v[i].y : j == 2 ? v[i].z : v[i].w; };
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (si.finite)
            out = pack16(make_float4(col(0), col(1), col(2), col(3)), make_float4(col(4), col(5), col(6), col(7)),
                         make_float4(col(8), col(9), col(10), col(11)),
                         make_float4(col(12), col(13), col(14), col(15)), si);
        *reinterpret_cast<uint4*>(qT + (n + j) * K + k) = out;
    }
}

// One pass over a strip of 8 whole columns (K <= 4096 rows): the strip is
// read once into registers (each thread 16 consecutive rows x 4 columns, one
// 16-byte load per row; a warp's loads cover 16 rows x 32 bytes, whole
// sectors), the 8 column maxima are reduced in the block, and each thread
// quantizes its 16 values per column from registers into one 16-byte run of
// K-major codes (pack16: fast path + exact repair).  4 B read + 1 B written
// per element, nothing read twice.
constexpr int kStripCols = 8;
constexpr int kStripThreads = 512;
constexpr int kStripMaxK = 16 * (kStripThreads / 2);   // 4096

__global__ void __launch_bounds__(kStripThreads, 1) quantize_cols_strip_kernel(const float* __restrict__ w, int64_t K,
                                                                           int64_t N, int8_t* __restrict__ qT,
                                                                           double* scales, float* scales_f32,
                                                                           int* status) {
    __shared__ uint32_t red[kStripThreads / 32][kStripCols];
    __shared__ ScaleInfo s_si[kStripCols];
    const int t = threadIdx.x, half = t & 1, lane = t & 31, warp = t >> 5;
    const int64_t n = (int64_t)blockIdx.x * kStripCols + 4 * half;
    const int64_t k0 = 16 * (int64_t)(t >> 1);
    const bool rows_ok = k0 < K;   // K % 16 == 0: all 16 rows or none
    float4 v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
        v[i] = rows_ok ? __ldcs(reinterpret_cast<const float4*>(w + (k0 + i) * N + n)) : make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        m0 = max(m0, abs_bits(v[i].x));
        m1 = max(m1, abs_bits(v[i].y));
        m2 = max(m2, abs_bits(v[i].z));
        m3 = max(m3, abs_bits(v[i].w));
    }
    // lanes of one parity hold the same four columns
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) {
        m0 = max(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = max(m1, __shfl_xor_sync(0xffffffffu, m1, o));
        m2 = max(m2, __shfl_xor_sync(0xffffffffu, m2, o));
        m3 = max(m3, __shfl_xor_sync(0xffffffffu, m3, o));
    }
    if (lane < 2) {
        red[warp][4 * lane + 0] = m0;
        red[warp][4 * lane + 1] = m1;
        red[warp][4 * lane + 2] = m2;
        red[warp][4 * lane + 3] = m3;
    }
    __syncthreads();
    if (t < kStripCols) {
        uint32_t bits = 0;
#pragma unroll
        for (int r = 0; r < kStripThreads / 32; ++r) bits = max(bits, red[r][t]);
        const ScaleInfo si = scale_from_absmax_bits(bits);
        s_si[t] = si;
        const int64_t c = (int64_t)blockIdx.x * kStripCols + t;
        if (si.finite) {
            scales[c] = si.scale;
            if (scales_f32) scales_f32[c] = __double2float_rn(si.scale);
        } else {
            scales[c] = __longlong_as_double(0x7FF8000000000000ll);
            if (scales_f32) scales_f32[c] = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    __syncthreads();
    if (!rows_ok) return;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const ScaleInfo si = s_si[4 * half + j];
        auto col = [&](int i) { return j == 0 ? v[i].x : j == 1 ? v[i].y : j == 2 ? v[i].z : v[i].w; };
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (si.finite)
            out = pack16(make_float4(col(0), col(1), col(2), col(3)), make_float4(col(4), col(5), col(6), col(7)),
                         make_float4(col(8), col(9), col(10), col(11)),
                         make_float4(col(12), col(13), col(14), col(15)), si);
        *reinterpret_cast<uint4*>(qT + (n + j) * K + k0) = out;
    }
}

// --------------------------------------------------------- per-row (tokens)

// One block per row: absmax then quantize of that row.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, int64_t M, int64_t K,
                                                            int8_t* __restrict__ q, double* scales,
                                                            float* scales_f32, int* status) {
    const int64_t row = blockIdx.x;
    const float* xr = x + row * K;
    int8_t* qr = q + row * K;
    uint32_t m = 0;
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) m = max(m, abs_bits(xr[j]));
    m = warp_max_u32(m);
    __shared__ uint32_t red[32];
    __shared__ ScaleInfo res;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
        v = warp_max_u32(v);
        if (lane == 0) res = scale_from_absmax_bits(v);
    }
    __syncthreads();
    const ScaleInfo si = res;
    if (threadIdx.x == 0) {
        if (si.finite) {
            scales[row] = si.scale;
            if (scales_f32) scales_f32[row] = __double2float_rn(si.scale);
        } else {
            scales[row] = __longlong_as_double(0x7FF8000000000000ll);
            if (scales_f32) scales_f32[row] = __uint_as_float(0x7FC00000u);
            record_status(status, KZ_ERR_NONFINITE);
        }
    }
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) qr[j] = si.finite ? quant_one(xr[j], si) : (int8_t)0;
}

// -------------------------------------------------------------- dequantize

// Per-tensor dequantize, two exact forms.  The value of a code q is
// (float)((double)q * scale) (quantize.py:76-77, from_flat).  Form 1 (no
// table): with s_hi = (float)scale and s_lo = (float)(scale - s_hi),
// fma(q, s_hi, q * s_lo) in fp32 is within about 2^-47 of q * scale and so
// rounds to the same fp32 value for almost every scale; the host checks all
// 256 byte values for the call's scale (dequant_split_exact) and takes this
// form only when every one matches bit for bit.  Each code then costs a byte
// permute that places it in the mantissa of 2^23 (offset binary), one exact
// subtraction, one multiply and one FMA -- no shared memory and no per-block
// set-up.  Form 2 (any other scale):
// a lookup table: entry u holds
// (float)((double)q * scale) for the code q whose byte is u -- every value the
// reference can produce, indexed by the raw byte so that a lookup costs one
// byte permute, one address computation and one shared load -- so
// the per-element work is one shared-memory load (1 B in, 4 B out).  The
// table is replicated once per bank (entry u of copy b at word u * 32 + b) and
// lane b reads copy b, so a warp's 32 lookups never conflict however the codes
// fall.  Thread t turns one 4-byte word of codes into one 16-byte store, so
// warps read and write contiguous runs; each thread loads kDeqBatch words
// before converting any.
constexpr int kDeqTable = 256;
constexpr int kDeqBatch = 8;   // 4-byte code words in flight per thread
__global__ void __launch_bounds__(256) dequantize_kernel(const int8_t* __restrict__ q, int64_t n, double scale,
                                                         float* __restrict__ out) {
    __shared__ float table[kDeqTable * 32];
    __shared__ float values[kDeqTable];
    if (threadIdx.x < kDeqTable) {
        const int u = threadIdx.x;   // entry u: the code whose two's-complement byte is u
        values[u] = __double2float_rn((double)(int)(int8_t)(uint8_t)u * scale);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kDeqTable * 32; i += blockDim.x) table[i] = values[i >> 5];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    const float* tlane = table + lane;
    // byte k of a word, zero-extended by one byte permute, scaled to its row of the table
    auto lutw = [&](uint32_t w, int k) { return tlane[__byte_perm(w, 0u, 0x4440u | (uint32_t)k) << 5]; };
    auto lut = [&](uint32_t byte) { return tlane[(byte & 0xFFu) << 5]; };
    const bool aligned = (reinterpret_cast<uintptr_t>(q) & 3u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    if (aligned) {
        // thread t converts word t of 4 codes into one 16-byte store, so a
        // warp reads 128 contiguous bytes and writes 512; kDeqBatch words
        // per thread are loaded before any is converted
        const int64_t n4 = n >> 2;
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(q);
        float4* ov = reinterpret_cast<float4*>(out);
        for (int64_t i0 = tid; i0 < n4; i0 += kDeqBatch * nthreads) {
            uint32_t w[kDeqBatch];
#pragma unroll
            for (int u = 0; u < kDeqBatch; ++u) {
                const int64_t i = i0 + u * nthreads;
                w[u] = i < n4 ? __ldcs(qw + i) : 0u;
            }
#pragma unroll
            for (int u = 0; u < kDeqBatch; ++u) {
                const int64_t i = i0 + u * nthreads;
                if (i < n4)
                    __stcs(ov + i, make_float4(lutw(w[u], 0), lutw(w[u], 1), lutw(w[u], 2), lutw(w[u], 3)));
            }
        }
        for (int64_t j = (n4 << 2) + tid; j < n; j += nthreads) out[j] = lut((uint8_t)q[j]);
    } else {
        for (int64_t j = tid; j < n; j += nthreads) out[j] = lut((uint8_t)q[j]);
    }
}

// Form 1 (see above): thread t turns one word of four codes into one 16-byte
// store; kDeqBatch words in flight per thread.
__global__ void __launch_bounds__(256) dequantize_split_kernel(const int8_t* __restrict__ q, int64_t n, float s_hi,
                                                               float s_lo, float* __restrict__ out) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    // byte k of wx (the code + 128) as the mantissa of 2^23: 2^23 + q + 128 exactly
    auto val = [&](uint32_t wx, int k) {
        const float f = __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7440u | (uint32_t)k));
        const float qf = __fsub_rn(f, 8388736.0f);
        return __fmaf_rn(qf, s_hi, __fmul_rn(qf, s_lo));
    };
    auto val1 = [&](int8_t c) {
        const float qf = (float)(int)c;
        return __fmaf_rn(qf, s_hi, __fmul_rn(qf, s_lo));
    };
    const bool aligned = (reinterpret_cast<uintptr_t>(q) & 3u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    if (aligned) {
        const int64_t n4 = n >> 2;
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(q);
        float4* ov = reinterpret_cast<float4*>(out);
        for (int64_t i0 = tid; i0 < n4; i0 += kDeqBatch * nthreads) {
            uint32_t w[kDeqBatch];
#pragma unroll
            for (int u = 0; u < kDeqBatch; ++u) {
                const int64_t i = i0 + u * nthreads;
                w[u] = i < n4 ? __ldcs(qw + i) ^ 0x80808080u : 0u;
            }
#pragma unroll
            for (int u = 0; u < kDeqBatch; ++u) {
                const int64_t i = i0 + u * nthreads;
                if (i < n4) __stcs(ov + i, make_float4(val(w[u], 0), val(w[u], 1), val(w[u], 2), val(w[u], 3)));
            }
        }
        for (int64_t j = (n4 << 2) + tid; j < n; j += nthreads) out[j] = val1(q[j]);
    } else {
        for (int64_t j = tid; j < n; j += nthreads) out[j] = val1(q[j]);
    }
}

// out[k][n] = (float)((double)qT[n][k] * scales[n]); 32x32 tiles through smem.
__global__ void __launch_bounds__(256) dequantize_cols_kernel(const int8_t* __restrict__ qT, int64_t K, int64_t N,
                                                              const double* __restrict__ scales,
                                                              float* __restrict__ out) {
    __shared__ int8_t tile[32][33];
    const int64_t n0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int64_t n = n0 + r, k = k0 + threadIdx.x;
        tile[r][threadIdx.x] = (n < N && k < K) ? qT[n * K + k] : (int8_t)0;
    }
    __syncthreads();
    const int64_t n = n0 + threadIdx.x;
    const double s = n < N ? scales[n] : 0.0;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int64_t k = k0 + r;
        if (n < N && k < K) out[k * N + n] = __double2float_rn((double)tile[threadIdx.x][r] * s);
    }
}

static int elementwise_grid(int64_t work_items) {
    const int64_t cap = (int64_t)sm_count() * 8;   // 8 resident 256-thread blocks per SM
    int64_t g = (work_items + 255) / 256;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (int)g;
}

}  // namespace kz

using namespace kz;

extern "C" {

int kz_absmax_f32(const float* x, int64_t n, uint32_t* partials, kz_stream_t stream) {
    KZ_REQUIRE(n >= 0, "kz_absmax_f32: n must be >= 0");
    KZ_REQUIRE(partials != nullptr, "kz_absmax_f32: partials is NULL");
    KZ_REQUIRE(n == 0 || x != nullptr, "kz_absmax_f32: x is NULL");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int grid = (int)std::min<int64_t>((n + 32 * 256 - 1) / (32 * 256), 6 * (int64_t)sm_count());
    if (grid < 1) grid = 1;
    if (grid > KZ_PARTIALS_WORDS - 3) grid = KZ_PARTIALS_WORDS - 3;
    KZ_CHECK_CUDA(launch_pdl(absmax_kernel, dim3(grid), dim3(256), 0, s, x, n, partials));
    return KZ_OK;
}

int kz_quantize_partials_f32(const float* x, int64_t n, const uint32_t* partials, int8_t* q, double* scale,
                             float* scale_f32, kz_stream_t stream) {
    KZ_REQUIRE(n >= 0, "kz_quantize_partials_f32: n must be >= 0");
    KZ_REQUIRE(partials && scale, "kz_quantize_partials_f32: partials and scale must be non-NULL");
    KZ_REQUIRE(n == 0 || (x && q), "kz_quantize_partials_f32: x or q is NULL");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    KZ_CHECK_CUDA(launch_pdl(quantize_partials_kernel, dim3(elementwise_grid((n + 15) / 16)), dim3(256), 0, s, x, n,
                             partials, q, scale, scale_f32, device_status_ptr()));
    return KZ_OK;
}

static int fused_grid(int dev) {
    static std::atomic<int> cached[64];   // per device; first calls may race (the value is the same)
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_fused_kernel, 1024, 0) != cudaSuccess)
        per_sm = 0;
    int g = std::min(per_sm, 1) * sm_count();   // one 1024-thread block per SM: few barrier arrivals
    if (g > kFusedMaxBlocks) g = kFusedMaxBlocks;
    if (dev >= 0 && dev < 64) cached[dev] = g;
    return g;
}

// Row pitch (floats) of the staged LayerNorm: D rounded up so that the pitch
// in bytes is 16 times an odd number modulo 128 (conflict-free 16-byte reads
// by one lane per row).
static int layernorm_stride(int64_t D) {
    int64_t s = (D + 3) / 4 * 4;
    while ((s % 32) % 8 != 4) s += 4;
    return (int)s;
}

constexpr int kLnMaxSmem = 96 * 1024;

static int layernorm_partials_impl(const float* x, const float* res, int64_t M, int64_t D, const float* gamma,
                                   const float* beta, float eps, float* sum_out, float* y, uint32_t* partials,
                                   kz_stream_t stream) {
    KZ_REQUIRE(M >= 0 && D > 0, "kz_layernorm_partials_f32: need M >= 0 and D > 0");
    KZ_REQUIRE(partials, "kz_layernorm_partials_f32: partials is NULL");
    KZ_REQUIRE(M == 0 || (x && y), "kz_layernorm_partials_f32: x or y is NULL");
    int st = check_device();
    if (st) return st;
    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    const uintptr_t bits = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                           reinterpret_cast<uintptr_t>(res) | reinterpret_cast<uintptr_t>(sum_out) |
                           reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta);
    const int stride = layernorm_stride(D);
    const size_t smem = (size_t)kLnRows * stride * sizeof(float);
    const int staged = (D % 4 == 0) && (bits & 15u) == 0 && smem <= (size_t)kLnMaxSmem;
    if (staged && smem > 48 * 1024) {
        static std::atomic<int> attr_set[64];
        if (dev < 0 || dev >= 64 || !attr_set[dev]) {
            KZ_CHECK_CUDA(cudaFuncSetAttribute(layernorm_partials_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kLnMaxSmem));
            if (dev >= 0 && dev < 64) attr_set[dev] = 1;
        }
    }
    const int64_t cap = std::min<int64_t>(4 * (int64_t)sm_count(), kFusedMaxBlocks);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((M + kLnRows - 1) / kLnRows, cap));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    KZ_CHECK_CUDA(launch_pdl(layernorm_partials_kernel, dim3(grid), dim3(kLnThreads), staged ? smem : 0, s, x, M, D,
                             gamma, beta, eps, y, partials, res, sum_out, staged, stride));
    return KZ_OK;
}

int kz_layernorm_partials_f32(const float* x, int64_t M, int64_t D, const float* gamma, const float* beta, float eps,
                              float* y, uint32_t* partials, kz_stream_t stream) {
    return layernorm_partials_impl(x, nullptr, M, D, gamma, beta, eps, nullptr, y, partials, stream);
}

int kz_add_layernorm_partials_f32(const float* x, const float* res, int64_t M, int64_t D, const float* gamma,
                                  const float* beta, float eps, float* sum_out, float* y, uint32_t* partials,
                                  kz_stream_t stream) {
    KZ_REQUIRE(M == 0 || (res && sum_out), "kz_add_layernorm_partials_f32: res or sum_out is NULL");
    KZ_REQUIRE(M == 0 || (sum_out != x && sum_out != res && sum_out != y),
               "kz_add_layernorm_partials_f32: sum_out must not alias x, res or y");
    return layernorm_partials_impl(x, res, M, D, gamma, beta, eps, sum_out, y, partials, stream);
}

int kz_quantize_tensor_f32(const float* x, int64_t n, int8_t* q, double* scale, float* scale_f32,
                           uint32_t* partials, kz_stream_t stream) {
    KZ_REQUIRE(n >= 0, "kz_quantize_tensor_f32: n must be >= 0");
    KZ_REQUIRE(partials && scale, "kz_quantize_tensor_f32: partials and scale must be non-NULL");
    KZ_REQUIRE(n == 0 || (x && q), "kz_quantize_tensor_f32: x or q is NULL");
    int st = check_device();
    if (st) return st;
    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    const int grid = fused_grid(dev);
    if (grid < 1 || n < (int64_t)1 << 16) {
        // small tensors: the two-kernel form (no grid barrier needed)
        st = kz_absmax_f32(x, n, partials, stream);
        if (st) return st;
        return kz_quantize_partials_f32(x, n, partials, q, scale, scale_f32, stream);
    }
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15u) == 0;
    if (aligned) {
        // one block per SM, its chunk resident in shared memory
        static std::atomic<int> smem_set[64];
        int max_smem = 0;
        KZ_CHECK_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        const int dyn = max_smem - 1024;   // leave room for the kernel's static shared memory
        if (dev >= 0 && dev < 64 && !smem_set[dev]) {
            KZ_CHECK_CUDA(cudaFuncSetAttribute(quantize_resident_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
            smem_set[dev] = 1;
        }
        const int G = std::min(sm_count(), kFusedMaxBlocks);
        int64_t chunk = (n + G - 1) / G;
        chunk = (chunk + 15) / 16 * 16;
        const uint32_t cap = (uint32_t)((dyn / 4) & ~15);
        KZ_REQUIRE((uint64_t)cap * 4 <= (uint64_t)kMaxPieces * kBulkPiece, "quantize: resident chunk over the piece count");
        cudaLaunchConfig_t rcfg = {};
        rcfg.gridDim = dim3((unsigned)G);
        rcfg.blockDim = dim3(kResidentBlock);
        rcfg.dynamicSmemBytes = (size_t)dyn;
        rcfg.stream = reinterpret_cast<cudaStream_t>(stream);
        // Programmatic dependent launch as well: every block waits for the
        // preceding grid (griddepcontrol.wait) before it touches x or the
        // partials, so all blocks are resident before the grid barrier.
        cudaLaunchAttribute rattr[2] = {};
        rattr[0].id = cudaLaunchAttributeCooperative;
        rattr[0].val.cooperative = 1;
        rattr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        rattr[1].val.programmaticStreamSerializationAllowed = 1;
        rcfg.attrs = rattr;
        rcfg.numAttrs = 2;
        KZ_CHECK_CUDA(cudaLaunchKernelEx(&rcfg, quantize_resident_kernel, x, n, chunk, cap, partials, q, scale,
                                         scale_f32, device_status_ptr()));
        return KZ_OK;
    }
    const int g = (int)std::min<int64_t>(grid, (n + 16383) / 16384);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)g);
    cfg.blockDim = dim3(1024);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1] = {};
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KZ_CHECK_CUDA(cudaLaunchKernelEx(&cfg, quantize_fused_kernel, x, n, partials, q, scale, scale_f32,
                                     device_status_ptr()));
    return KZ_OK;
}

static bool cols_vectorised(const float* w, int64_t K, int64_t N, const int8_t* qT) {
    return K > 0 && N % 4 == 0 && K % 16 == 0 &&
           ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(qT)) & 15u) == 0;
}

static int64_t col_splits(int64_t K, int64_t N, bool vec) {
    if (vec) {
        // one 256-row pass per block where that fits in 64 splits
        int64_t want = (K + kColRowsPerPass - 1) / kColRowsPerPass;
        return std::max<int64_t>(1, std::min<int64_t>(want, 64));
    }
    // enough blocks to fill the GPU: ~4 waves of (N / 32) x splits
    const int64_t col_tiles = (N + 31) / 32;
    int64_t want = (4 * (int64_t)sm_count() + col_tiles - 1) / col_tiles;
    int64_t max_splits = (K + 63) / 64;   // at least 64 rows per split
    if (want > max_splits) want = max_splits;
    if (want < 1) want = 1;
    if (want > 64) want = 64;
    return want;
}

// Both per-channel quantize entry points: `partial` holds at least
// max_words words of scratch (splits x N are used).
static int quantize_cols_launch(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales, float* scales_f32,
                                uint32_t* partial, int64_t max_words, cudaStream_t s, const char* who,
                                bool allow_strip = false) {
    const bool vec = cols_vectorised(w, K, N, qT);
    if (allow_strip && vec && K > kStripMaxK / 2 && K <= kStripMaxK && N % kStripCols == 0) {
        // whole columns fit one block's registers (and fill most of its
        // threads): a single pass, no workspace
        KZ_REQUIRE(N / kStripCols < INT32_MAX, "quantize_cols: N too large");
        quantize_cols_strip_kernel<<<(unsigned)(N / kStripCols), kStripThreads, 0, s>>>(w, K, N, qT, scales,
                                                                                     scales_f32, device_status_ptr());
        return launch_status(who);
    }
    int64_t splits = K == 0 ? 1 : col_splits(K, N, vec);
    if (splits * N > max_words) splits = std::max<int64_t>(1, max_words / N);
    KZ_REQUIRE(splits * N <= max_words, "quantize_cols: scratch smaller than N words");
    if (K == 0) {
        KZ_CHECK_CUDA(cudaMemsetAsync(partial, 0, (size_t)N * sizeof(uint32_t), s));
    } else if (vec) {
        const int64_t rows_per_split = (K + splits - 1) / splits;
        KZ_REQUIRE((N + kColTile - 1) / kColTile < INT32_MAX, "quantize_cols: N too large");
        absmax_cols4_kernel<<<dim3((unsigned)((N + kColTile - 1) / kColTile), (unsigned)splits), 256, 0, s>>>(
            w, K, N, rows_per_split, partial);
        int st = launch_status(who);
        if (st) return st;
        const int64_t ktiles = (K + kColRowsPerPass - 1) / kColRowsPerPass;
        KZ_REQUIRE(ktiles < 65536, "quantize_cols: K too large");
        quantize_cols4_kernel<<<dim3((unsigned)((N + kColTile - 1) / kColTile), (unsigned)ktiles), 256, 0, s>>>(
            w, K, N, partial, (int)splits, qT, scales, scales_f32, device_status_ptr());
        return launch_status(who);
    } else {
        const int64_t rows_per_split = (K + splits - 1) / splits;
        absmax_cols_kernel<<<dim3((unsigned)((N + 31) / 32), (unsigned)splits), dim3(32, 8), 0, s>>>(
            w, K, N, rows_per_split, partial);
        int st = launch_status(who);
        if (st) return st;
    }
    const int64_t ktiles = K == 0 ? 1 : (K + 127) / 128;
    KZ_REQUIRE(ktiles < 65536, "quantize_cols: K too large");
    quantize_cols_kernel<<<dim3((unsigned)((N + 31) / 32), (unsigned)ktiles), dim3(32, 8), 0, s>>>(
        w, K, N, partial, (int)splits, qT, scales, scales_f32, device_status_ptr());
    return launch_status(who);
}

size_t kz_quantize_cols_workspace_bytes(int64_t K, int64_t N) {
    if (K < 0 || N <= 0) return 0;   // K == 0 still clears N words of partials
    return (size_t)64 * (size_t)N * sizeof(uint32_t);
}

int kz_quantize_cols_f32(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales, float* scales_f32,
                         void* workspace, size_t workspace_bytes, kz_stream_t stream) {
    KZ_REQUIRE(K >= 0 && N >= 0, "kz_quantize_cols_f32: K and N must be >= 0");
    if (K == 0 || N == 0) {
        KZ_REQUIRE(N == 0 || scales, "kz_quantize_cols_f32: scales is NULL");
        if (N == 0) return KZ_OK;
    }
    KZ_REQUIRE(scales != nullptr, "kz_quantize_cols_f32: scales is NULL");
    KZ_REQUIRE(K == 0 || (w && qT), "kz_quantize_cols_f32: w or qT is NULL");
    int st = check_device();
    if (st) return st;
    const int64_t splits = K == 0 ? 1 : col_splits(K, N, cols_vectorised(w, K, N, qT));
    KZ_REQUIRE(workspace != nullptr && workspace_bytes >= (size_t)splits * (size_t)N * sizeof(uint32_t),
               "kz_quantize_cols_f32: workspace smaller than kz_quantize_cols_workspace_bytes(K, N)");
    return quantize_cols_launch(w, K, N, qT, scales, scales_f32, static_cast<uint32_t*>(workspace),
                                (int64_t)(workspace_bytes / sizeof(uint32_t)), reinterpret_cast<cudaStream_t>(stream),
                                "kz_quantize_cols_f32", /*allow_strip=*/true);
}

int kz_quantize_rows_f32(const float* x, int64_t M, int64_t K, int8_t* q, double* scales, float* scales_f32,
                         kz_stream_t stream) {
    KZ_REQUIRE(M >= 0 && K >= 0, "kz_quantize_rows_f32: M and K must be >= 0");
    if (M == 0) return KZ_OK;
    KZ_REQUIRE(scales != nullptr, "kz_quantize_rows_f32: scales is NULL");
    KZ_REQUIRE(K == 0 || (x && q), "kz_quantize_rows_f32: x or q is NULL");
    KZ_REQUIRE(M < (int64_t)INT32_MAX, "kz_quantize_rows_f32: M too large");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    quantize_rows_kernel<<<(unsigned)M, 256, 0, s>>>(x, M, K, q, scales, scales_f32, device_status_ptr());
    return launch_status("quantize_rows_kernel");
}

// True when fma(q, s_hi, q * s_lo) in fp32 equals (float)((double)q * scale)
// for all 256 byte values q (the split form of the device kernel; the host's
// fmaf and multiply are IEEE operations like the device's).
static bool dequant_split_exact(double scale, float* s_hi, float* s_lo) {
    const float hi = (float)scale;
    const float lo = (float)(scale - (double)hi);
    if (!std::isfinite(hi) || !std::isfinite(lo)) return false;
    for (int c = -128; c <= 127; ++c) {
        const float exact = (float)((double)c * scale);
        const float qf = (float)c;
        volatile float p = qf * lo;            // rounded on its own, as on the device
        const float cand = std::fma(qf, hi, (float)p);
        uint32_t a, b;
        std::memcpy(&a, &exact, 4);
        std::memcpy(&b, &cand, 4);
        if (a != b) return false;
    }
    *s_hi = hi;
    *s_lo = lo;
    return true;
}

int kz_dequantize_uses_table(double scale) {
    float hi, lo;
    return dequant_split_exact(scale, &hi, &lo) ? 0 : 1;
}

int kz_dequantize_i8_f32(const int8_t* q, int64_t n, double scale, float* out, kz_stream_t stream) {
    KZ_REQUIRE(n >= 0, "kz_dequantize_i8_f32: n must be >= 0");
    if (n == 0) return KZ_OK;
    KZ_REQUIRE(q && out, "kz_dequantize_i8_f32: q or out is NULL");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t per_block = 256 * 4 * kDeqBatch;
    float s_hi, s_lo;
    if (dequant_split_exact(scale, &s_hi, &s_lo)) {
        // one wave of resident blocks (the grid-stride loop spreads the tail
        // over every thread) instead of a partial second wave
        static std::atomic<int> resident[64];
        int dev = 0;
        KZ_CHECK_CUDA(cudaGetDevice(&dev));
        int per_sm = (dev >= 0 && dev < 64) ? resident[dev].load() : 0;
        if (per_sm == 0) {
            KZ_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dequantize_split_kernel, 256, 0));
            per_sm = std::max(per_sm, 1);
            if (dev >= 0 && dev < 64) resident[dev] = per_sm;
        }
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + per_block - 1) / per_block,
                                                                     (int64_t)per_sm * sm_count()));
        dequantize_split_kernel<<<grid, 256, 0, s>>>(q, n, s_hi, s_lo, out);
        return launch_status("dequantize_split_kernel");
    }
    // up to six resident blocks per SM (each builds its own 33 KB table once)
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + per_block - 1) / per_block, 6 * (int64_t)sm_count()));
    dequantize_kernel<<<grid, 256, 0, s>>>(q, n, scale, out);
    return launch_status("dequantize_kernel");
}

int kz_dequantize_cols_i8_f32(const int8_t* qT, int64_t K, int64_t N, const double* scales, float* out,
                              kz_stream_t stream) {
    KZ_REQUIRE(K >= 0 && N >= 0, "kz_dequantize_cols_i8_f32: K and N must be >= 0");
    if (K == 0 || N == 0) return KZ_OK;
    KZ_REQUIRE(qT && scales && out, "kz_dequantize_cols_i8_f32: NULL pointer");
    KZ_REQUIRE((N + 31) / 32 < 65536, "kz_dequantize_cols_i8_f32: N too large");
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    dequantize_cols_kernel<<<dim3((unsigned)((K + 31) / 32), (unsigned)((N + 31) / 32)), dim3(32, 8), 0, s>>>(
        qT, K, N, scales, out);
    return launch_status("dequantize_cols_kernel");
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Per-channel weight quantize that allocates nothing.
//
// Some callers of this library cannot call cudaMalloc: a host runtime that
// owns all of the GPU's memory through its own allocator or fixed arena (a
// JVM, Go or game-engine host binding this C ABI, an inference server that
// must not allocate after start-up), where an unplanned cudaMalloc would
// fragment or exceed the memory that host reserved.  For them,
// kz_quantize_cols_f32_noalloc takes no workspace argument: its scratch (the
// column-absmax partial maxima) lives in the file-scope device array below.
//
// The array is 65536 words (256 KB).  Every GPU that loads libkz holds it until
// the process exits.  N is limited to 65536 output channels; larger N is
// rejected with KZ_ERR_INVALID_ARGUMENT.
//
// All calls share this one array.  Each call overwrites every entry it later
// reads (and zeroes the entries it reads when K == 0), so nothing from an
// earlier call leaks into a result.  Calls whose kernels overlap on the GPU --
// two streams, or two host threads -- race on the array: order them on one
// stream or serialise them.
//
// Host code must not use the array's name as a device pointer: on the host it
// is only a stand-in.  The first call on each device, with that device
// current, resolves the device address with cudaGetSymbolAddress (checked) and
// caches it; that set-up runs once per device, so make the first call on a
// device before any stream capture.
// ----------------------------------------------------------------------------

namespace kz {
constexpr int64_t kNoAllocScratchWords = 65536;
static __device__ __align__(256) uint32_t g_noalloc_cols_scratch[kNoAllocScratchWords];

static std::mutex g_noalloc_mu;
static uint32_t* g_noalloc_ptr[64] = {};

static int noalloc_scratch(uint32_t** out) {
    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(KZ_ERR_UNSUPPORTED_DEVICE, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_cols_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_cols_scratch)");
        g_noalloc_ptr[dev] = static_cast<uint32_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return KZ_OK;
}
}  // namespace kz

extern "C" int kz_quantize_cols_f32_noalloc(const float* w, int64_t K, int64_t N, int8_t* qT, double* scales,
                                            float* scales_f32, kz_stream_t stream) {
    KZ_REQUIRE(K >= 0 && N >= 0, "kz_quantize_cols_f32_noalloc: K and N must be >= 0");
    KZ_REQUIRE(N <= kz::kNoAllocScratchWords,
               "kz_quantize_cols_f32_noalloc: N exceeds 65536 output channels, the size of its static scratch; "
               "use kz_quantize_cols_f32 with a workspace");
    if (N == 0) return KZ_OK;
    KZ_REQUIRE(scales != nullptr, "kz_quantize_cols_f32_noalloc: scales is NULL");
    KZ_REQUIRE(K == 0 || (w && qT), "kz_quantize_cols_f32_noalloc: w or qT is NULL");
    const int64_t ktiles = K == 0 ? 1 : (K + 127) / 128;
    KZ_REQUIRE(ktiles < 65536, "kz_quantize_cols_f32_noalloc: K too large");
    int st = check_device();
    if (st) return st;
    uint32_t* partial = nullptr;
    st = kz::noalloc_scratch(&partial);
    if (st) return st;
    return quantize_cols_launch(w, K, N, qT, scales, scales_f32, partial, kz::kNoAllocScratchWords,
                                reinterpret_cast<cudaStream_t>(stream), "kz_quantize_cols_f32_noalloc");
}
