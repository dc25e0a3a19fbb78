// int8 x int8 -> int32 GEMM on the sm_100a tensor cores, with the rescale,
// bias and activation fused into the epilogue.
//
// This is the contraction inside qlinear (python/kansai/quantize.py:121,
// x.matmul(w)) once both operands are int8; the reference itself has no int8
// GEMM (quantize.py:35-44) and runs an fp32 loop (backend/cpu/src/Ops.cpp:328-337).
//
// Design (one CTA per SM, persistent over output tiles):
//   tile 128 x 256 (M x N), k-block 128 bytes = one 128-byte swizzle atom;
//   warp 0      TMA producer: A[128 x 128] and B[256 x 128] per k-block into a
//               4-stage shared-memory ring (48 KB per stage), no multicast;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 int32 accumulators)
//               and one thread issues tcgen05.mma.kind::i8 (M128 N256 K32, four
//               per k-block), committing each stage back to the producer and
//               each finished accumulator to the epilogue;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (each warp owns the
//               32 TMEM lanes = tile rows of its sub-partition), rescale, bias,
//               activation, store; the second accumulator lets the next tile's
//               main loop run while this tile drains.
// Every mbarrier wait is bounded (kz_common.cuh); on expiry the CTA records
// KZ_ERR_DEVICE_TIMEOUT, unwinds, drains its in-flight copies and MMAs with
// bounded waits and frees its TMEM.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kz_common.cuh"

namespace kz {

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;   // 16 KB
constexpr int B_STAGE = BN * BK;   // 32 KB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;        // tile rasterisation: 16 tile-rows per group
constexpr int EPI_WARPS = 4;
constexpr int EPI_BUF = 32 * 32 * 4;                 // one warp's 32 x 32 fp32/int32 sub-tile
constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF;       // one staging buffer per warp: 16 KB
constexpr int NUM_BARS = 2 * STAGES + 2 * NUM_ACC + 1;
constexpr int COLV_BYTES = EPI_WARPS * 2 * BN * 4;      // per warp: the tile's column scales and bias
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + EPI_BYTES + COLV_BYTES + 256;
constexpr uint32_t IDESC = idesc_i8(BM, BN);
}  // namespace gemm

struct GemmParams {
    int M, N, K;
    int a_kblock;
    int num_kb;
    int tiles_m, tiles_n, num_tiles;
    const float* row_scale;
    int64_t rs_stride;
    const float* col_scale;
    int64_t cs_stride;
    const float* bias;
    int act;
    float* out_f32;
    int32_t* out_i32;
    int64_t ldo;
    int tma_out;        // 1: the single output goes through the TMA-store tensor map
    uint32_t* partials;
    int* status;
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& tm, int& tn) {
    const int group_size = gemm::GROUP_M * p.tiles_n;
    const int group = t / group_size;
    const int first_m = group * gemm::GROUP_M;
    const int gm = min(gemm::GROUP_M, p.tiles_m - first_m);
    const int r = t - group * group_size;
    tm = first_m + r % gm;
    tn = r / gm;
}

template <int ACT>
__device__ __forceinline__ float epi_act_t(float v) {
    if constexpr (ACT == KZ_ACT_RELU) return v > 0.0f ? v : 0.0f;
    if constexpr (ACT == KZ_ACT_GELU) {
        const float cdf = __fmul_rn(0.5f, __fadd_rn(1.0f, erff(__fmul_rn(v, 0.7071067811865476f))));
        return __fmul_rn(v, cdf);
    }
    return v;
}

__device__ __forceinline__ float epi_act(float v, int act) {
    if (act == KZ_ACT_RELU) return v > 0.0f ? v : 0.0f;
    if (act == KZ_ACT_GELU) {
        const float cdf = __fmul_rn(0.5f, __fadd_rn(1.0f, erff(__fmul_rn(v, 0.7071067811865476f))));
        return __fmul_rn(v, cdf);
    }
    return v;
}

// Whole-warp bounded wait: every lane polls, then the warp agrees.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* status, volatile int* abort_flag) {
    const bool got = mbar_wait(bar, parity, status, abort_flag);
    return __all_sync(0xffffffffu, got);
}

template <int ACT>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const GemmParams p) {
    using namespace gemm;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE;
    uint8_t* sEpi = sB + STAGES * B_STAGE;
    float* sColv = reinterpret_cast<float*>(sEpi + EPI_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + EPI_BYTES + COLV_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* red = tmem_slot + 2;   // 4 words: epilogue absmax per warp

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + NUM_ACC);
    const uint32_t drain = smem_u32(bars + 2 * STAGES + 2 * NUM_ACC);
    const uint32_t sA0 = smem_u32(sA), sB0 = smem_u32(sB);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, EPI_WARPS);   // one arrive per epilogue warp
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (p.tma_out) tma_prefetch_desc(&tmOut);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (whole warp, lane 0 issues)
        int stage = 0;
        uint32_t phase = 0;
        uint32_t armed_mask = 0, armed_phase = 0;   // per stage: armed at least once / parity of last arm
        bool ok = true;
        for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
            int tm, tn;
            tile_coords(t, p, tm, tn);
            const int m0 = tm * BM, n0 = tn * BN;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!warp_wait(empty0 + 8 * stage, phase ^ 1, p.status, abort_flag)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(full0 + 8 * stage, STAGE_BYTES);
                    const int kbyte = kb * BK;
                    int ax = kbyte, ay = m0;
                    if (p.a_kblock != p.K) {
                        const int g = kbyte / p.a_kblock;
                        ax = kbyte - g * p.a_kblock;
                        ay = g * p.M + m0;
                    }
                    tma_load_2d(sA0 + stage * A_STAGE, &tmA, full0 + 8 * stage, ax, ay);
                    tma_load_2d(sB0 + stage * B_STAGE, &tmB, full0 + 8 * stage, kbyte, n0);
                }
                __syncwarp();
                armed_mask |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (!ok) {
            // unwinding: let every armed copy land before the CTA exits
            for (int s = 0; s < STAGES; ++s)
                if (armed_mask >> s & 1u) mbar_wait(full0 + 8 * s, armed_phase >> s & 1u, nullptr, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (whole warp, lane 0 issues)
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        bool issued = false;
        for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
            if (!warp_wait(tempty0 + 8 * acc, acc_phase ^ 1, p.status, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(acc * BN);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!warp_wait(full0 + 8 * stage, phase, p.status, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_addr = sA0 + stage * A_STAGE, b_addr = sB0 + stage * B_STAGE;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk)
                        tc_mma_i8(d, smem_desc_k_sw128(a_addr + kk * 32), smem_desc_k_sw128(b_addr + kk * 32),
                                  IDESC, (kb | kk) != 0);
                    tc_commit(empty0 + 8 * stage);
                }
                __syncwarp();
                issued = true;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(tfull0 + 8 * acc);
            __syncwarp();
            if (++acc == NUM_ACC) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (!ok && issued) {
            // unwinding: wait for every MMA issued so far before TMEM is freed
            if (lane == 0) {
                tc_commit(drain);
                mbar_wait(drain, 0, nullptr, nullptr);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int sub = warp & 3;                  // TMEM sub-partition this warp may access
        const int row_in_tile = sub * 32 + lane;
        const uint32_t epi0 = smem_u32(sEpi) + (uint32_t)((warp - 2) * EPI_BUF);
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t amax = 0;
        uint32_t qchunk = 0;                       // chunks this warp has staged so far
        const bool vec_ok_f32 = p.out_f32 && (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out_f32) & 15u) == 0);
        const bool vec_ok_i32 = p.out_i32 && (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out_i32) & 15u) == 0);
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
            int tm, tn;
            tile_coords(t, p, tm, tn);
            const int m0 = tm * BM, n0 = tn * BN;
            if (!warp_wait(tfull0 + 8 * acc, acc_phase, p.status, abort_flag)) break;
            tc_fence_after();
            const int m = m0 + row_in_tile;
            const bool row_ok = m < p.M;
            float rs = 0.0f;
            const int nchunks = min(BN / 32, (p.N - n0 + 31) / 32);
            // the tile's column scales and bias, staged once per tile in this
            // warp's own shared-memory slice (read back as broadcasts)
            float* wcs = sColv + (warp - 2) * 2 * BN;
            float* wb = wcs + BN;
            if (p.out_f32) {
                rs = __ldg(p.row_scale + (int64_t)min(m, p.M - 1) * p.rs_stride);
                __syncwarp();
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) {
                    const int nl = min(n0 + c * 32 + lane, p.N - 1);
                    wcs[c * 32 + lane] = __ldg(p.col_scale + (int64_t)nl * p.cs_stride);
                    wb[c * 32 + lane] = p.bias ? __ldg(p.bias + nl) : 0.0f;
                }
                __syncwarp();
            }
            for (int c = 0; c < nchunks; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
                tc_wait_ld();
                if (c == nchunks - 1) {
                    // last read of this accumulator: hand it back to the MMA warp now
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
                }
                const int nb = n0 + c * 32;
                uint32_t v[32];
                if (p.out_f32) {
                    const float4* cs4 = reinterpret_cast<const float4*>(wcs + c * 32);
                    const float4* b4 = reinterpret_cast<const float4*>(wb + c * 32);
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 cs = cs4[j4];
                        const float csv[4] = {cs.x, cs.y, cs.z, cs.w};
                        float bv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        if (p.bias) {
                            const float4 bb = b4[j4];
                            bv[0] = bb.x; bv[1] = bb.y; bv[2] = bb.z; bv[3] = bb.w;
                        }
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int j = 4 * j4 + e;
                            float y = __fmul_rn(__int2float_rn((int)r[j]), rs);
                            y = __fmul_rn(y, csv[e]);
                            if (p.bias) y = __fadd_rn(y, bv[e]);
                            v[j] = __float_as_uint(epi_act_t<ACT>(y));
                        }
                    }
                    if (p.partials && row_ok) {
                        const int valid = min(32, p.N - nb);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < valid) amax = max(amax, v[j] & 0x7FFFFFFFu);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = r[j];
                }
                if (p.tma_out) {
                    // stage the warp's 32 x 32 sub-tile (128-byte rows, 128B-swizzled) and TMA-store it
                    const uint32_t buf = epi0;
                    if (qchunk >= 1) {
                        if (lane == 0) bulk_wait_group_read<0>();   // previous store has read the buffer
                        __syncwarp();
                    }
                    const uint32_t row_addr = buf + (uint32_t)lane * 128u;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_shared_v4(row_addr + (uint32_t)((j ^ (lane & 7)) * 16), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                     v[4 * j + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmOut, buf, nb, m0 + sub * 32);
                        bulk_commit_group();
                    }
                    ++qchunk;
                } else if (row_ok) {
                    // direct stores: ragged or unaligned outputs, or both outputs requested
                    const bool full_chunk = nb + 32 <= p.N;
                    if (p.out_i32) {
                        int32_t* dst = p.out_i32 + (int64_t)m * p.ldo + nb;
                        if (full_chunk && vec_ok_i32) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<int4*>(dst + j) =
                                    make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (nb + j < p.N) dst[j] = (int)r[j];
                        }
                    }
                    if (p.out_f32) {
                        float* dst = p.out_f32 + (int64_t)m * p.ldo + nb;
                        if (full_chunk && vec_ok_f32) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<float4*>(dst + j) =
                                    make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (nb + j < p.N) dst[j] = __uint_as_float(v[j]);
                        }
                    }
                }
            }
            if (++acc == NUM_ACC) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (p.tma_out && lane == 0) bulk_wait_group_all();   // every store landed before exit
        __syncwarp();
        if (p.partials) {
            amax = warp_max_u32(amax);
            if (lane == 0) red[sub] = amax;
            asm volatile("bar.sync 1, 128;" ::: "memory");   // epilogue warps only
            if (warp == 2 && lane == 0) {
                p.partials[1 + blockIdx.x] = max(max(red[0], red[1]), max(red[2], red[3]));
                if (blockIdx.x == 0) p.partials[0] = gridDim.x;
            }
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// K == 0: every accumulator is zero; only the epilogue runs.
__global__ void gemm_i8_k0_kernel(const GemmParams p) {
    const int64_t total = (int64_t)p.M * p.N;
    uint32_t amax = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / p.N, n = i % p.N;
        if (p.out_i32) p.out_i32[m * p.ldo + n] = 0;
        if (p.out_f32) {
            float v = __fmul_rn(__fmul_rn(0.0f, p.row_scale[m * p.rs_stride]), p.col_scale[n * p.cs_stride]);
            if (p.bias) v = __fadd_rn(v, p.bias[n]);
            v = epi_act(v, p.act);
            p.out_f32[m * p.ldo + n] = v;
            amax = max(amax, __float_as_uint(v) & 0x7FFFFFFFu);
        }
    }
    if (p.partials) {
        amax = warp_max_u32(amax);
        __shared__ uint32_t red[32];
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t v = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = max(v, red[w]);
            p.partials[1 + blockIdx.x] = v;
            if (blockIdx.x == 0) p.partials[0] = gridDim.x;
        }
    }
}

// ------------------------------------------------------------------ host

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D tensor map over rows x cols (cols contiguous, row pitch `pitch_bytes`), 128-byte swizzle.
static int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t cols, uint64_t rows,
                        uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(KZ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(KZ_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return KZ_OK;
}

static int make_tmap_i8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                        uint32_t box_rows) {
    return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, cols, rows, cols, box_cols, box_rows);
}

static int ensure_gemm_attrs(int dev) {
    static int done[64] = {};
    if (dev >= 0 && dev < 64 && done[dev]) return KZ_OK;
    KZ_CHECK_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<KZ_ACT_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::SMEM_BYTES));
    KZ_CHECK_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<KZ_ACT_RELU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::SMEM_BYTES));
    KZ_CHECK_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<KZ_ACT_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::SMEM_BYTES));
    if (dev >= 0 && dev < 64) done[dev] = 1;
    return KZ_OK;
}

// Tensor maps are encoded on the host; a call that reuses the same buffers and
// shapes (every step of a serving loop) reuses its maps.  Small per-thread
// cache keyed by everything the maps encode.
struct TmapKey {
    const void* a;
    const void* b;
    const void* out;
    int64_t M, N, K, a_kblock, ldo;
    int out_kind;
    int dev;
    bool operator==(const TmapKey& o) const {
        return a == o.a && b == o.b && out == o.out && M == o.M && N == o.N && K == o.K && a_kblock == o.a_kblock &&
               ldo == o.ldo && out_kind == o.out_kind && dev == o.dev;
    }
};
struct TmapEntry {
    TmapKey key;
    CUtensorMap a, b, out;
    bool valid;
};
constexpr int kTmapCache = 16;
thread_local TmapEntry t_tmap_cache[kTmapCache];
thread_local int t_tmap_next = 0;

}  // namespace kz

using namespace kz;

extern "C" int kz_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
                          const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
                          const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
                          uint32_t* absmax_partials, kz_stream_t stream) {
    KZ_REQUIRE(M >= 0 && N >= 0 && K >= 0, "kz_gemm_i8: negative dimension");
    KZ_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "kz_gemm_i8: dimension too large");
    KZ_REQUIRE(K <= 131072, "kz_gemm_i8: K > 131072 could overflow the int32 accumulator");
    KZ_REQUIRE(out_f32 || out_i32, "kz_gemm_i8: no output (out_f32 and out_i32 are both NULL)");
    KZ_REQUIRE(!out_f32 || (row_scale && col_scale), "kz_gemm_i8: fp32 output needs row_scale and col_scale");
    KZ_REQUIRE(rs_stride == 0 || rs_stride == 1, "kz_gemm_i8: rs_stride must be 0 or 1");
    KZ_REQUIRE(cs_stride == 0 || cs_stride == 1, "kz_gemm_i8: cs_stride must be 0 or 1");
    KZ_REQUIRE(act >= KZ_ACT_NONE && act <= KZ_ACT_GELU, "kz_gemm_i8: unknown activation");
    KZ_REQUIRE(ldo >= N, "kz_gemm_i8: ldo < N");
    if (M == 0 || N == 0) {
        if (absmax_partials) {
            int st = check_device();
            if (st) return st;
            static const uint32_t zero_count[2] = {1, 0};
            KZ_CHECK_CUDA(cudaMemcpyAsync(absmax_partials, zero_count, sizeof(zero_count), cudaMemcpyHostToDevice,
                                          reinterpret_cast<cudaStream_t>(stream)));
        }
        return KZ_OK;
    }
    int st = check_device();
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

    GemmParams p{};
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.a_kblock = (int)(a_kblock ? a_kblock : K);
    p.row_scale = row_scale;
    p.rs_stride = rs_stride;
    p.col_scale = col_scale;
    p.cs_stride = cs_stride;
    p.bias = bias;
    p.act = act;
    p.out_f32 = out_f32;
    p.out_i32 = out_i32;
    p.ldo = ldo;
    p.partials = absmax_partials;
    p.status = device_status_ptr();

    if (K == 0) {
        int grid = (int)std::min<int64_t>((M * N + 255) / 256, (int64_t)sm_count() * 4);
        if (grid > KZ_PARTIALS_WORDS - 1) grid = KZ_PARTIALS_WORDS - 1;
        gemm_i8_k0_kernel<<<grid, 256, 0, s>>>(p);
        return launch_status("gemm_i8_k0_kernel");
    }
    KZ_REQUIRE(A && B, "kz_gemm_i8: A or B is NULL");
    KZ_REQUIRE(K % 16 == 0, "kz_gemm_i8: K must be a multiple of 16 (TMA row pitch)");
    KZ_REQUIRE(K % p.a_kblock == 0, "kz_gemm_i8: a_kblock must divide K");
    KZ_REQUIRE(p.a_kblock == K || p.a_kblock % 128 == 0, "kz_gemm_i8: a_kblock must be K or a multiple of 128");
    KZ_REQUIRE((reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0,
               "kz_gemm_i8: A and B must be 16-byte aligned");
    p.num_kb = (int)((K + gemm::BK - 1) / gemm::BK);
    p.tiles_m = (int)((M + gemm::BM - 1) / gemm::BM);
    p.tiles_n = (int)((N + gemm::BN - 1) / gemm::BN);
    const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
    KZ_REQUIRE(tiles < (1ll << 31), "kz_gemm_i8: too many tiles");
    p.num_tiles = (int)tiles;

    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    // TMA-store epilogue when exactly one output is requested and its rows are 16-byte pitched
    void* out_ptr = out_f32 ? static_cast<void*>(out_f32) : static_cast<void*>(out_i32);
    p.tma_out = (out_f32 == nullptr) != (out_i32 == nullptr) && (ldo * 4) % 16 == 0 &&
                (reinterpret_cast<uintptr_t>(out_ptr) & 15u) == 0;
    const TmapKey key{A, B, out_ptr, M, N, K, p.a_kblock, ldo, p.tma_out ? (out_f32 ? 1 : 2) : 0, dev};
    TmapEntry* ent = nullptr;
    for (int i = 0; i < kTmapCache; ++i)
        if (t_tmap_cache[i].valid && t_tmap_cache[i].key == key) ent = &t_tmap_cache[i];
    if (!ent) {
        TmapEntry fresh;
        memset(&fresh, 0, sizeof(fresh));
        fresh.key = key;
        const uint64_t a_rows = (uint64_t)M * (uint64_t)(K / p.a_kblock);
        st = make_tmap_i8(&fresh.a, A, (uint64_t)p.a_kblock, a_rows, gemm::BK, gemm::BM);
        if (st) return st;
        st = make_tmap_i8(&fresh.b, B, (uint64_t)K, (uint64_t)N, gemm::BK, gemm::BN);
        if (st) return st;
        if (p.tma_out) {
            st = make_tmap_2d(&fresh.out, out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_INT32,
                              out_ptr, (uint64_t)N, (uint64_t)M, (uint64_t)ldo * 4, 32, 32);
            if (st) return st;
        }
        fresh.valid = true;
        ent = &t_tmap_cache[t_tmap_next];
        *ent = fresh;
        t_tmap_next = (t_tmap_next + 1) % kTmapCache;
    }
    st = ensure_gemm_attrs(dev);
    if (st) return st;

    int grid = std::min(p.num_tiles, sm_count());
    if (grid > KZ_PARTIALS_WORDS - 1) grid = KZ_PARTIALS_WORDS - 1;
    if (act == KZ_ACT_RELU)
        gemm_i8_kernel<KZ_ACT_RELU><<<grid, gemm::THREADS, gemm::SMEM_BYTES, s>>>(ent->a, ent->b, ent->out, p);
    else if (act == KZ_ACT_GELU)
        gemm_i8_kernel<KZ_ACT_GELU><<<grid, gemm::THREADS, gemm::SMEM_BYTES, s>>>(ent->a, ent->b, ent->out, p);
    else
        gemm_i8_kernel<KZ_ACT_NONE><<<grid, gemm::THREADS, gemm::SMEM_BYTES, s>>>(ent->a, ent->b, ent->out, p);
    return launch_status("gemm_i8_kernel");
}
