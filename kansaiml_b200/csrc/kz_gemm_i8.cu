// int8 x int8 -> int32 GEMM on the sm_100a tensor cores, with the rescale,
// bias and activation fused into the epilogue.
//
// This is the contraction inside qlinear (python/kansai/quantize.py:121,
// x.matmul(w)) once both operands are int8; the reference itself has no int8
// GEMM (quantize.py:35-44) and runs an fp32 loop (backend/cpu/src/Ops.cpp:328-337).
//
// Two forms of one persistent, warp-specialised kernel (one CTA per SM):
//   PAIR   a CTA pair (cluster of 2) owns a 256 x 256 output tile: each CTA
//          loads 128 rows of A and 128 rows of B per 128-byte k-block (32 KB,
//          6-stage ring), the leader issues tcgen05.mma.cta_group::2.kind::i8
//          (M256 N256 K32) that reads both CTAs' shared memory, and each CTA's
//          TMEM holds its own 128 x 256 int32 accumulator rows.  Per SM this
//          needs 64 B/cycle of TMA fill for 8192 MAC/cycle.
//   single one CTA owns a 128 x 256 tile (A 16 KB + B 32 KB per k-block, 4
//          stages, tcgen05.mma.cta_group::1 M128 N256 K32); used when M <= 128.
// Roles: warp 0 TMA producer; warp 1 TMEM allocation (512 columns = two
// accumulators) and, in the leader, the MMA issue (one lane) with commits back
// to both CTAs' stage barriers and accumulator barriers; warps 2..9 epilogue
// (two warps per TMEM lane quarter, each draining half of the tile's columns):
// tcgen05.ld 32 columns at a time (each warp reads the 32 TMEM lanes of its
// sub-partition), fp32 rescale / bias / activation with the tile's column
// scales staged in shared memory, 128B-swizzled staging and a
// cp.async.bulk.tensor store per 32 x 32 sub-tile.  The second accumulator
// lets tile i+1's main loop run under tile i's epilogue.  No TMA multicast.
// Every mbarrier wait is bounded (kz_common.cuh); on expiry the CTA records
// KZ_ERR_DEVICE_TIMEOUT and unwinds.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kz_common.cuh"

namespace kz {

namespace gemm {
constexpr int BN = 256, BK = 128;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 8;                         // two per TMEM sub-partition, one per column half
constexpr int THREADS = 64 + 32 * EPI_WARPS;
#ifndef KZ_EPI_DIRECT
#define KZ_EPI_DIRECT 0   // 1: epilogue stores straight from registers (32-byte stores) instead of TMA
#endif
#ifndef KZ_GROUP_M
#define KZ_GROUP_M 16   // tile rasterisation: tile-rows per group
#endif
constexpr int GROUP_M = KZ_GROUP_M;
constexpr int EPI_BUF = 32 * 32 * 4;                 // one warp's 32 x 32 fp32/int32 sub-tile
constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF;       // one staging buffer per warp: 32 KB
constexpr int COLV_BYTES = 2 * BN * 4;               // the tile's column scales and bias (shared by the epilogue)

template <bool PAIR>
struct Cfg {
    static constexpr int BM_CTA = 128;                 // accumulator / A rows per CTA
    static constexpr int BM_TILE = PAIR ? 256 : 128;   // output rows per tile
    static constexpr int BN_CTA = PAIR ? 128 : 256;    // B rows loaded per CTA
    static constexpr int A_STAGE = BM_CTA * BK;        // 16 KB
    static constexpr int B_STAGE = BN_CTA * BK;        // 16 / 32 KB
    static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
    static constexpr int STAGES = PAIR ? 6 : 4;
    static constexpr int NUM_BARS = 2 * STAGES + 2 * NUM_ACC + 1;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + COLV_BYTES + 256;   // base 1024-aligned
    static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
    static constexpr uint32_t IDESC = idesc_i8(BM_TILE, BN);
};
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
    // Gated A (kz_gemm_i8_gated): rows [c * flag_rows, (c + 1) * flag_rows) of
    // block g of the [G][M][a_kblock] A layout may be loaded once
    // a_ready[g * flag_chunks + c] == ready_token; block first_block is
    // resident from the start and every tile walks the blocks from it.
    // NULL: no gating.
    const uint32_t* a_ready;
    uint32_t ready_token;
    int first_block;
    int flag_rows, flag_chunks;
    // Fused all-gather (kz_gemm_i8_allgather): CTAs [0, copy_ctas) copy the
    // other ranks' A blocks from their memory into the local [G][M][a_kblock]
    // buffer, chunk by chunk, and publish ready_token in copy_flags (== a_ready)
    // for the computing CTAs.  0: no copy role.
    int copy_ctas;
    uint32_t* copy_flags;
    int group_m;        // tile rasterisation: tile-rows per group
};

// The other ranks' gather buffers ([G][M][a_kblock] bytes in their memory,
// mapped into this process) as TMA store targets, and their flag arrays;
// entry `rank` unused.
constexpr int kMaxPeers = 8;
struct PeerMaps {
    int8_t* peer_a[kMaxPeers];
    uint32_t* flags[kMaxPeers];
};
struct NoPeerMaps {
    int unused;
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& tm, int& tn) {
    const int group_size = p.group_m * p.tiles_n;
    const int group = t / group_size;
    const int first_m = group * p.group_m;
    const int gm = min(p.group_m, p.tiles_m - first_m);
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

// Whole-warp bounded wait: every lane polls, then the warp agrees.  Pair mode
// waits with cluster-scope acquire (arrivals released by the other CTA).
template <bool CLUSTER>
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* status, volatile int* abort_flag) {
    const bool got = CLUSTER ? mbar_wait_cluster(bar, parity, status, abort_flag)
                             : mbar_wait(bar, parity, status, abort_flag);
    return __all_sync(0xffffffffu, got);
}

__device__ __forceinline__ void st_release_gpu_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Copy role of the fused all-gather GEMM (push), run by every thread of a copy
// CTA: thread 0 streams 128-row x 128-byte tiles of this rank's own A block
// from local memory into shared memory (TMA loads, 12 stages in flight); all
// threads then write each tile into every other rank's gather buffer with
// 16-byte stores into peer memory over NVLink (posted writes, many in flight;
// the tile is read back from the 128B-swizzled stage).  Row chunks go in
// order, so the rows the first GEMM tiles need land first; every chunk's
// tiles are dealt round-robin over all copy CTAs.  After a CTA's last tile of a
// chunk, every thread fences its stores at system scope, and the last copy CTA
// to report the chunk resets the chunk's counter and writes ready_token into
// every other rank's flags[rank * C + c].  Waits are bounded; on expiry the
// CTA stops issuing, waits (bounded) for its loads in flight and returns.
__device__ __forceinline__ void gemm_copy_role(const CUtensorMap& tmA, const PeerMaps& pm, const GemmParams& p,
                                               uint8_t* smem) {
    constexpr int S = 12;
    constexpr uint32_t TILE = 128 * 128;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * TILE);
    const int G = p.K / p.a_kblock, C = p.flag_chunks, R = p.flag_rows, me = p.first_block;
    const int xs_n = p.a_kblock / 128;
    const int T = (R / 128) * xs_n;                 // tiles per chunk (>= copy_ctas, checked on the host)
    const int64_t total = (int64_t)C * T;
    const int cidx = blockIdx.x, cc = p.copy_ctas;
    const int n = cidx < total ? (int)((total - cidx + cc - 1) / cc) : 0;
    uint32_t* counters = p.copy_flags + G * C;     // this rank's per-chunk arrival counters
    const uint32_t full0 = smem_u32(bars), stage0 = smem_u32(smem);
    const int tid = threadIdx.x, nthr = blockDim.x;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) mbar_init(full0 + 8 * s, 1);
        fence_mbarrier_init();
    }
    __syncthreads();

    auto coords = [&](int i, int& c, int& x, int& row) {
        const int64_t q = cidx + (int64_t)i * cc;
        c = (int)(q / T);
        const int w = (int)(q - (int64_t)c * T);
        x = (w % xs_n) * 128;
        row = c * R + (w / xs_n) * 128;
    };
    auto ends_chunk = [&](int i) {
        const int64_t q = cidx + (int64_t)i * cc;
        return i == n - 1 || (q / T) != ((q + cc) / T);
    };
    auto issue = [&](int i) {   // thread 0
        int c, x, row;
        coords(i, c, x, row);
        const uint32_t bar = full0 + 8 * (i % S);
        mbar_arrive_expect_tx(bar, TILE);
        tma_load_2d(stage0 + (uint32_t)(i % S) * TILE, &tmA, bar, x, me * p.M + row);
    };
    if (tid == 0)
        for (int i = 0; i < min(S, n); ++i) issue(i);
    int issued = min(S, n);
    int i = 0;
    for (; i < n; ++i) {
        const bool got = mbar_wait(full0 + 8 * (i % S), (uint32_t)((i / S) & 1), p.status, nullptr);
        if (__syncthreads_or(!got)) break;
        int c, x, row;
        coords(i, c, x, row);
        const uint4* st = reinterpret_cast<const uint4*>(smem + (size_t)(i % S) * TILE);
        const int64_t grow0 = (int64_t)me * p.M + row;
        for (int v = tid; v < (int)(TILE / 16); v += nthr) {
            const int r = v >> 3, c16 = v & 7;
            const uint4 val = st[r * 8 + (c16 ^ (r & 7))];
            const int64_t off = (grow0 + r) * p.a_kblock + x + c16 * 16;
            for (int h = 0; h < G; ++h)
                if (h != me) *reinterpret_cast<uint4*>(pm.peer_a[h] + off) = val;
        }
        const bool last = ends_chunk(i);
        if (last) __threadfence_system();          // this thread's stores of the chunk are visible
        __syncthreads();                           // the stage is free, every thread's stores are fenced
        if (tid == 0) {
            if (issued < n) issue(issued++);
            if (last) {
                const uint32_t old = atomicAdd(counters + c, 1u);
                if (old == (uint32_t)cc - 1) {
                    atomicExch(counters + c, 0u);
                    __threadfence_system();
                    for (int h = 0; h < G; ++h)
                        if (h != me) st_release_sys_u32(pm.flags[h] + me * C + c, p.ready_token);
                }
            }
        }
    }
    if (i < n && tid == 0) {
        // unwinding: every load in flight lands before the CTA's shared memory goes away
        for (int j = i + 1; j < issued; ++j) mbar_wait(full0 + 8 * (j % S), (uint32_t)((j / S) & 1), nullptr, nullptr);
    }
    __syncthreads();
}

template <int ACT, bool PAIR, bool COPY = false>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const GemmParams p,
                   const __grid_constant__ typename std::conditional<COPY, PeerMaps, NoPeerMaps>::type pm) {
    using namespace gemm;
    using C = Cfg<PAIR>;
    // The kernel has no static shared memory, so the dynamic region starts at
    // the base of the CTA's shared window, which is 1024-byte aligned (the
    // 128B-swizzle atoms need it).  Checked; a misaligned base records an error.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (smem_u32(smem_raw) & 1023u) {
        if (threadIdx.x == 0) record_status(p.status, KZ_ERR_INVALID_ARGUMENT);
        return;
    }
    uint8_t* smem = smem_raw;
    if constexpr (COPY) {
        if ((int)blockIdx.x < p.copy_ctas) {
            griddep_launch_dependents();
            griddep_wait();
            if (p.partials && threadIdx.x == 0) {
                // copy CTAs own partials slots too (no output rows: zero)
                p.partials[1 + blockIdx.x] = 0u;
                if (blockIdx.x == 0) p.partials[0] = gridDim.x;
            }
            gemm_copy_role(tmA, pm, p, smem);
            return;
        }
    }
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_STAGE;
    uint8_t* sEpi = sB + C::STAGES * C::B_STAGE;
    float* sColv = reinterpret_cast<float*>(sEpi + EPI_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + EPI_BYTES + COLV_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* red = tmem_slot + 2;   // EPI_WARPS words: epilogue absmax per warp

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int cbase = COPY ? p.copy_ctas : 0;                               // copy CTAs come first
    const int unit = PAIR ? (int)((blockIdx.x - cbase) >> 1) : (int)(blockIdx.x - cbase);   // pair or CTA
    const int units = PAIR ? (int)((gridDim.x - cbase) >> 1) : (int)(gridDim.x - cbase);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + C::STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * C::STAGES), tempty0 = smem_u32(bars + 2 * C::STAGES + NUM_ACC);
    const uint32_t drain = smem_u32(bars + 2 * C::STAGES + 2 * NUM_ACC);
    const uint32_t sA0 = smem_u32(sA), sB0 = smem_u32(sB);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, PAIR ? 2 * EPI_WARPS : EPI_WARPS);   // one arrive per epilogue warp
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
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // the prologue above overlaps the previous kernel (programmatic dependent
    // launch); from here on A, the scales and the output may be touched
    griddep_launch_dependents();
    griddep_wait();
    // the leader's barriers (TMA completion, accumulator release) and the
    // peer's (the leader's commits), as cluster addresses
    const uint32_t full_lead0 = PAIR ? mapa_shared(full0, 0) : full0;
    const uint32_t tempty_lead0 = PAIR ? mapa_shared(tempty0, 0) : tempty0;
    const uint32_t empty_peer0 = PAIR ? mapa_shared(empty0, 1) : empty0;
    const uint32_t tfull_peer0 = PAIR ? mapa_shared(tfull0, 1) : tfull0;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (whole warp, lane 0 issues)
        int stage = 0;
        uint32_t phase = 0;
        uint32_t armed_mask = 0, armed_phase = 0;   // per stage: armed at least once / parity of last arm
        bool ok = true;
        for (int t = unit; ok && t < p.num_tiles; t += units) {
            int tm, tn;
            tile_coords(t, p, tm, tn);
            const int m0 = tm * C::BM_TILE + (int)rank * C::BM_CTA;   // this CTA's A rows
            const int nb0 = tn * BN + (int)rank * C::BN_CTA;          // this CTA's B rows
            // Every tile walks K from the same k-block, so tiles running at the
            // same time read the same k-slices of their A and B panels (they
            // stay in L2); a gated A starts at the block already resident.  The
            // int32 accumulation is exact, so the k order does not change the
            // result.
            const int rot = p.a_ready ? p.first_block * (p.a_kblock / BK) : 0;
            const int chunk = p.a_ready ? min(m0, p.M - 1) / p.flag_rows : 0;   // this CTA's rows lie in one chunk
            int cur_g = -1;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                int kr = kb + rot;
                if (kr >= p.num_kb) kr -= p.num_kb;
                if (p.a_ready) {
                    // first load of this tile from an A block: wait until its rows have landed
                    const int g = (kr * BK) / p.a_kblock;
                    if (g != cur_g) {
                        cur_g = g;
                        if (g != p.first_block &&
                            !flag_wait(p.a_ready + g * p.flag_chunks + chunk, p.ready_token, p.status, abort_flag)) {
                            ok = false;
                            break;
                        }
                    }
                }
                if (!warp_wait<false>(empty0 + 8 * stage, phase ^ 1, p.status, abort_flag)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    if (leader) mbar_arrive_expect_tx(full0 + 8 * stage, (PAIR ? 2 : 1) * C::STAGE_BYTES);
                    const int kbyte = kr * BK;
                    int ax = kbyte, ay = m0;
                    if (p.a_kblock != p.K) {
                        const int g = kbyte / p.a_kblock;
                        ax = kbyte - g * p.a_kblock;
                        ay = g * p.M + m0;
                    }
                    if constexpr (PAIR) {
                        tma_load_2d_pair(sA0 + stage * C::A_STAGE, &tmA, full_lead0 + 8 * stage, ax, ay);
                        tma_load_2d_pair(sB0 + stage * C::B_STAGE, &tmB, full_lead0 + 8 * stage, kbyte, nb0);
                    } else {
                        tma_load_2d(sA0 + stage * C::A_STAGE, &tmA, full0 + 8 * stage, ax, ay);
                        tma_load_2d(sB0 + stage * C::B_STAGE, &tmB, full0 + 8 * stage, kbyte, nb0);
                    }
                }
                __syncwarp();
                armed_mask |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (!ok && leader) {
            // unwinding: let every armed copy land before the pair exits
            for (int s = 0; s < C::STAGES; ++s)
                if (armed_mask >> s & 1u) mbar_wait(full0 + 8 * s, armed_phase >> s & 1u, nullptr, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader; whole warp, lane 0 issues)
        if (leader) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued = false;
            for (int t = unit; ok && t < p.num_tiles; t += units) {
                if (!warp_wait<PAIR>(tempty0 + 8 * acc, acc_phase ^ 1, p.status, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!warp_wait<false>(full0 + 8 * stage, phase, p.status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    // TMA (async proxy) -> MMA (async proxy) through the mbarrier:
                    // no tcgen05 fence here; one after the accumulator wait per tile
                    if (lane == 0) {
                        const uint32_t a_addr = sA0 + stage * C::A_STAGE, b_addr = sB0 + stage * C::B_STAGE;
#pragma unroll
                        for (int kk = 0; kk < BK / 32; ++kk) {
                            const uint64_t da = smem_desc_k_sw128(a_addr + kk * 32);
                            const uint64_t db = smem_desc_k_sw128(b_addr + kk * 32);
                            if constexpr (PAIR)
                                tc_mma_i8_pair(d, da, db, C::IDESC, (kb | kk) != 0);
                            else
                                tc_mma_i8(d, da, db, C::IDESC, (kb | kk) != 0);
                        }
                        if constexpr (PAIR) {
                            tc_commit_pair(empty0 + 8 * stage);
                            tc_commit_pair(empty_peer0 + 8 * stage);
                        } else {
                            tc_commit(empty0 + 8 * stage);
                        }
                    }
                    __syncwarp();
                    issued = true;
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if (lane == 0) {
                    if constexpr (PAIR) {
                        tc_commit_pair(tfull0 + 8 * acc);
                        tc_commit_pair(tfull_peer0 + 8 * acc);
                    } else {
                        tc_commit(tfull0 + 8 * acc);
                    }
                }
                __syncwarp();
                if (++acc == NUM_ACC) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            if (!ok && issued) {
                // unwinding: wait for every MMA issued so far before TMEM is freed
                if (lane == 0) {
                    if constexpr (PAIR) tc_commit_pair(drain); else tc_commit(drain);
                    mbar_wait(drain, 0, nullptr, nullptr);
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 2 .. 2 + EPI_WARPS)
        // warp w reads TMEM sub-partition (w & 3), i.e. tile rows 32 (w & 3) .. +31
        // of this CTA, and column half (w - 2) / 4 of the 256-column tile.
        const int ew = warp - 2;
        const int sub = warp & 3;
        const int half = ew >> 2;
        const int row_in_tile = (int)rank * C::BM_CTA + sub * 32 + lane;
        const uint32_t epi0 = smem_u32(sEpi) + (uint32_t)(ew * EPI_BUF);
        float* tcs = sColv;          // [BN] column scales of the current tile
        float* tb = sColv + BN;      // [BN] bias
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t amax = 0;
        uint32_t qchunk = 0;                       // chunks this warp has staged so far
        const bool vec_ok_f32 = p.out_f32 && (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out_f32) & 15u) == 0);
        const bool vec_ok_i32 = p.out_i32 && (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out_i32) & 15u) == 0);
        constexpr int CH_PER_WARP = BN / 32 / 2;   // 4 chunks of 32 columns per column half
        // After a timed-out wait a warp stays "not alive" but keeps walking the
        // tile loop, so every epilogue warp executes the same named barriers.
        bool alive = true;
        for (int t = unit; t < p.num_tiles; t += units) {
            int tm, tn;
            tile_coords(t, p, tm, tn);
            const int m0 = tm * C::BM_TILE, n0 = tn * BN;
            const int m = m0 + row_in_tile;
            const bool row_ok = m < p.M;
            float rs = 0.0f;
            const int nchunks = min(BN / 32, (p.N - n0 + 31) / 32);
            const int c_begin = half * CH_PER_WARP;
            const int c_end = min(c_begin + CH_PER_WARP, nchunks);
            // stage the tile's column scales and bias once for all epilogue warps
            if (p.out_f32) {
                rs = __ldg(p.row_scale + (int64_t)min(m, p.M - 1) * p.rs_stride);
                asm volatile("bar.sync 2, %0;" ::"n"(32 * EPI_WARPS) : "memory");   // previous tile's readers done
                const int nl = min(n0 + ew * 32 + lane, p.N - 1);
                tcs[ew * 32 + lane] = __ldg(p.col_scale + (int64_t)nl * p.cs_stride);
                tb[ew * 32 + lane] = p.bias ? __ldg(p.bias + nl) : 0.0f;
                asm volatile("bar.sync 2, %0;" ::"n"(32 * EPI_WARPS) : "memory");
            }
            if (alive) alive = warp_wait<PAIR>(tfull0 + 8 * acc, acc_phase, p.status, abort_flag);
            if (!alive) continue;
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN);
            uint32_t ra[32], rb[32];
            if (c_begin < c_end) {
                tmem_ld_32x32b_x32(tbase + (uint32_t)(c_begin * 32), ra);
                tc_wait_ld();
            }
            for (int c = c_begin; c < c_end; ++c) {
                // the next chunk's TMEM load runs while this chunk is processed
                const bool more = c + 1 < c_end;
                uint32_t r[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) r[j] = ra[j];
                if (more) tmem_ld_32x32b_x32(tbase + (uint32_t)((c + 1) * 32), rb);
                const int nb = n0 + c * 32;
                uint32_t v[32];
                if (p.out_f32) {
                    const float4* cs4 = reinterpret_cast<const float4*>(tcs + c * 32);
                    const float4* b4 = reinterpret_cast<const float4*>(tb + c * 32);
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
                if (p.tma_out && KZ_EPI_DIRECT) {
                    // each lane writes its row's 32 values as four 32-byte stores (whole sectors)
                    if (row_ok) {
                        uint32_t* dst = (p.out_f32 ? reinterpret_cast<uint32_t*>(p.out_f32)
                                                   : reinterpret_cast<uint32_t*>(p.out_i32)) +
                                        (int64_t)m * p.ldo + nb;
                        if (nb + 32 <= p.N && p.ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(dst) & 31u) == 0) {
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + 8 * j),
                                             "r"(v[8 * j]), "r"(v[8 * j + 1]), "r"(v[8 * j + 2]), "r"(v[8 * j + 3]),
                                             "r"(v[8 * j + 4]), "r"(v[8 * j + 5]), "r"(v[8 * j + 6]), "r"(v[8 * j + 7])
                                             : "memory");
                        } else {
                            for (int j = 0; j < 32 && nb + j < p.N; ++j) dst[j] = v[j];
                        }
                    }
                } else if (p.tma_out) {
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
                        tma_store_2d(&tmOut, buf, nb, m0 + (int)rank * C::BM_CTA + sub * 32);
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
                if (more) {
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) ra[j] = rb[j];
                }
            }
            // every read of this accumulator by this warp is complete: hand it back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(tempty_lead0 + 8 * acc);
                else mbar_arrive(tempty0 + 8 * acc);
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
            if (lane == 0) red[ew] = amax;
            asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory");   // epilogue warps only
            if (ew == 0 && lane == 0) {
                uint32_t mx = 0;
                for (int w = 0; w < EPI_WARPS; ++w) mx = max(mx, red[w]);
                p.partials[1 + blockIdx.x] = mx;
                if (blockIdx.x == 0) p.partials[0] = gridDim.x;
            }
        }
    }

    tc_fence_before();
    if constexpr (PAIR) cluster_sync(); else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS); else tmem_dealloc(tmem_base, TMEM_COLS);
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

template <int ACT, bool PAIR, bool COPY = false>
static int set_smem_attr() {
    KZ_CHECK_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<ACT, PAIR, COPY>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm::Cfg<PAIR>::SMEM_BYTES));
    return KZ_OK;
}

// Per-device first-call state below is atomic: host threads of a threaded
// mesh may make their first calls at the same time (repeating the set-up is
// harmless).
static int ensure_gemm_attrs(int dev) {
    static std::atomic<int> done[64];
    if (dev >= 0 && dev < 64 && done[dev]) return KZ_OK;
    int st = set_smem_attr<KZ_ACT_NONE, false>();
    if (!st) st = set_smem_attr<KZ_ACT_RELU, false>();
    if (!st) st = set_smem_attr<KZ_ACT_GELU, false>();
    if (!st) st = set_smem_attr<KZ_ACT_NONE, true>();
    if (!st) st = set_smem_attr<KZ_ACT_RELU, true>();
    if (!st) st = set_smem_attr<KZ_ACT_GELU, true>();
    if (!st) st = set_smem_attr<KZ_ACT_NONE, true, true>();
    if (st) return st;
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
    int pair;
    int dev;
    bool operator==(const TmapKey& o) const {
        return a == o.a && b == o.b && out == o.out && M == o.M && N == o.N && K == o.K && a_kblock == o.a_kblock &&
               ldo == o.ldo && out_kind == o.out_kind && pair == o.pair && dev == o.dev;
    }
};
struct TmapEntry {
    TmapKey key;
    CUtensorMap a, b, out;
    bool valid;
};
constexpr int kTmapCache = 64;   // a chunked, multi-layer forward cycles through dozens of (A, out) pairs
thread_local TmapEntry t_tmap_cache[kTmapCache];
thread_local int t_tmap_next = 0;

template <int ACT, bool PAIR, bool COPY = false>
static int launch_gemm(int grid, cudaStream_t s, const TmapEntry* ent, const GemmParams& p,
                       const PeerMaps* peers = nullptr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(gemm::THREADS);
    cfg.dynamicSmemBytes = gemm::Cfg<PAIR>::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[2] = {};
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (PAIR) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    if constexpr (COPY) {
        KZ_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_i8_kernel<ACT, PAIR, true>, ent->a, ent->b, ent->out, p, *peers));
    } else {
        KZ_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_i8_kernel<ACT, PAIR, false>, ent->a, ent->b, ent->out, p,
                                         NoPeerMaps{0}));
    }
    return KZ_OK;
}

// SM budget of the GEMMs per device (0: every SM), kz_set_sm_count_target.
static std::atomic<int> g_sm_target[64];

// How many CTA pairs of the pair kernel can be resident at once (cached per device).
static int max_active_pairs(int dev) {
    static std::atomic<int> cached[64];
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)(sm_count() / 2));
    cfg.blockDim = dim3(gemm::THREADS);
    cfg.dynamicSmemBytes = gemm::Cfg<true>::SMEM_BYTES;
    cudaLaunchAttribute attr[1] = {};
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_i8_kernel<KZ_ACT_NONE, true>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sm_count() / 2;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

}  // namespace kz

using namespace kz;

static int gemm_i8_impl(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
                        const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
                        const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
                        uint32_t* absmax_partials, const uint32_t* a_ready, uint32_t ready_token, int first_block,
                        int64_t flag_rows, int8_t* const* peers, uint32_t* const* peer_flags, int copy_ctas,
                        kz_stream_t stream) {
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
    p.a_ready = a_ready;
    p.ready_token = ready_token;
    p.first_block = first_block;
    p.flag_rows = (int)std::min<int64_t>(std::max<int64_t>(flag_rows, 1), std::max<int64_t>(M, 1));
    p.flag_chunks = (int)((M + p.flag_rows - 1) / p.flag_rows);
    p.copy_ctas = peers ? copy_ctas : 0;
    p.copy_flags = const_cast<uint32_t*>(a_ready);
    // Gated A arrives in row chunks: group as many tile-rows as one chunk
    // holds, so the first tiles need the first chunk only.
    p.group_m = a_ready ? std::max(1, std::min(gemm::GROUP_M, p.flag_rows / 256)) : gemm::GROUP_M;

    if (K == 0) {
        int grid = (int)std::min<int64_t>((M * N + 255) / 256, (int64_t)sm_count() * 4);
        if (grid > KZ_PARTIALS_WORDS - 3) grid = KZ_PARTIALS_WORDS - 3;
        gemm_i8_k0_kernel<<<grid, 256, 0, s>>>(p);
        return launch_status("gemm_i8_k0_kernel");
    }
    KZ_REQUIRE(A && B, "kz_gemm_i8: A or B is NULL");
    KZ_REQUIRE(K % 16 == 0, "kz_gemm_i8: K must be a multiple of 16 (TMA row pitch)");
    KZ_REQUIRE(K % p.a_kblock == 0, "kz_gemm_i8: a_kblock must divide K");
    KZ_REQUIRE(p.a_kblock == K || p.a_kblock % 128 == 0, "kz_gemm_i8: a_kblock must be K or a multiple of 128");
    if (a_ready) {
        KZ_REQUIRE(p.a_kblock % 128 == 0 && K / p.a_kblock <= 32,
                   "kz_gemm_i8_gated: a_kblock must be a multiple of 128 with at most 32 blocks");
        KZ_REQUIRE(first_block >= 0 && first_block < K / p.a_kblock, "kz_gemm_i8_gated: first_block out of range");
        KZ_REQUIRE(flag_rows >= M || (flag_rows > 0 && flag_rows % 128 == 0),
                   "kz_gemm_i8_gated: flag_rows must be >= M or a positive multiple of 128");
    }
    KZ_REQUIRE((reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0,
               "kz_gemm_i8: A and B must be 16-byte aligned");
    // CTA pairs (256-row tiles) unless the whole problem fits one 128-row tile
    const bool pair = M > 128 && sm_count() >= 2;
    const int bm_tile = pair ? gemm::Cfg<true>::BM_TILE : gemm::Cfg<false>::BM_TILE;
    const int bn_cta = pair ? gemm::Cfg<true>::BN_CTA : gemm::Cfg<false>::BN_CTA;
    p.num_kb = (int)((K + gemm::BK - 1) / gemm::BK);
    p.tiles_m = (int)((M + bm_tile - 1) / bm_tile);
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
    const TmapKey key{A, B, out_ptr, M, N, K, p.a_kblock, ldo, p.tma_out ? (out_f32 ? 1 : 2) : 0, pair ? 1 : 0, dev};
    TmapEntry* ent = nullptr;
    for (int i = 0; i < kTmapCache; ++i)
        if (t_tmap_cache[i].valid && t_tmap_cache[i].key == key) ent = &t_tmap_cache[i];
    if (!ent) {
        TmapEntry fresh;
        memset(&fresh, 0, sizeof(fresh));
        fresh.key = key;
        const uint64_t a_rows = (uint64_t)M * (uint64_t)(K / p.a_kblock);
        st = make_tmap_i8(&fresh.a, A, (uint64_t)p.a_kblock, a_rows, gemm::BK, 128);
        if (st) return st;
        st = make_tmap_i8(&fresh.b, B, (uint64_t)K, (uint64_t)N, gemm::BK, (uint32_t)bn_cta);
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

    const int target = dev >= 0 && dev < 64 ? g_sm_target[dev].load() : 0;
    int grid;
    if (pair) {
        int cap = max_active_pairs(dev);
        if (target > 0) cap = std::max(1, std::min(cap, target / 2));
        const int pairs = std::max(1, std::min(p.num_tiles, cap - p.copy_ctas / 2));
        grid = 2 * pairs;
    } else {
        grid = std::min(p.num_tiles, target > 0 ? std::min(target, sm_count()) : sm_count());
    }
    if (grid > KZ_PARTIALS_WORDS - 3 - p.copy_ctas) grid = (KZ_PARTIALS_WORDS - 3 - p.copy_ctas) & ~1;
    if (peers) {
        // fused all-gather: the peers' buffer and flag pointers, copy CTAs in
        // front of the computing pairs
        KZ_REQUIRE(pair && act == KZ_ACT_NONE, "kz_gemm_i8_allgather: needs M > 128 and act none");
        PeerMaps pm;
        memset(&pm, 0, sizeof(pm));
        const int G = (int)(K / p.a_kblock);
        for (int h = 0; h < G; ++h) {
            if (h == first_block) continue;
            KZ_REQUIRE(peers[h] && (reinterpret_cast<uintptr_t>(peers[h]) & 15u) == 0 && peer_flags[h],
                       "kz_gemm_i8_allgather: peer buffers must be non-NULL and 16-byte aligned, peer flags non-NULL");
            pm.peer_a[h] = peers[h];
            pm.flags[h] = peer_flags[h];
        }
        return launch_gemm<KZ_ACT_NONE, true, true>(grid + p.copy_ctas, s, ent, p, &pm);
    }
    if (pair) {
        if (act == KZ_ACT_RELU) return launch_gemm<KZ_ACT_RELU, true>(grid, s, ent, p);
        if (act == KZ_ACT_GELU) return launch_gemm<KZ_ACT_GELU, true>(grid, s, ent, p);
        return launch_gemm<KZ_ACT_NONE, true>(grid, s, ent, p);
    }
    if (act == KZ_ACT_RELU) return launch_gemm<KZ_ACT_RELU, false>(grid, s, ent, p);
    if (act == KZ_ACT_GELU) return launch_gemm<KZ_ACT_GELU, false>(grid, s, ent, p);
    return launch_gemm<KZ_ACT_NONE, false>(grid, s, ent, p);
}

extern "C" int kz_set_sm_count_target(int sms) {
    KZ_REQUIRE(sms >= 0, "kz_set_sm_count_target: sms must be >= 0");
    int dev = 0;
    KZ_CHECK_CUDA(cudaGetDevice(&dev));
    KZ_REQUIRE(dev >= 0 && dev < 64, "kz_set_sm_count_target: device ordinal out of range");
    g_sm_target[dev] = sms;
    return KZ_OK;
}

extern "C" int kz_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
                          const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
                          const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
                          uint32_t* absmax_partials, kz_stream_t stream) {
    return gemm_i8_impl(A, B, M, N, K, a_kblock, row_scale, rs_stride, col_scale, cs_stride, bias, act, out_f32,
                        out_i32, ldo, absmax_partials, nullptr, 0, 0, 0, nullptr, nullptr, 0, stream);
}

extern "C" int kz_gemm_i8_gated(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int64_t a_kblock,
                                const float* row_scale, int64_t rs_stride, const float* col_scale, int64_t cs_stride,
                                const float* bias, int act, float* out_f32, int32_t* out_i32, int64_t ldo,
                                uint32_t* absmax_partials, const uint32_t* a_ready, uint32_t ready_token,
                                int first_block, int64_t flag_rows, kz_stream_t stream) {
    KZ_REQUIRE(a_ready != nullptr, "kz_gemm_i8_gated: a_ready is NULL");
    return gemm_i8_impl(A, B, M, N, K, a_kblock, row_scale, rs_stride, col_scale, cs_stride, bias, act, out_f32,
                        out_i32, ldo, absmax_partials, a_ready, ready_token, first_block, flag_rows, nullptr, nullptr,
                        0, stream);
}

extern "C" int kz_gemm_i8_allgather(const int8_t* A, int8_t* const* peer_A, uint32_t* const* peer_flags, int world,
                                    int rank, const int8_t* B, int64_t M, int64_t N, int64_t K, const float* row_scale,
                                    int64_t rs_stride, const float* col_scale, int64_t cs_stride, float* out_f32,
                                    int64_t ldo, uint32_t* absmax_partials, uint32_t* flags, uint32_t token,
                                    int64_t flag_rows, int copy_ctas, kz_stream_t stream) {
    KZ_REQUIRE(peer_A && peer_flags && flags, "kz_gemm_i8_allgather: peer_A, peer_flags and flags must be non-NULL");
    KZ_REQUIRE(world >= 2 && world <= kMaxPeers && K % world == 0, "kz_gemm_i8_allgather: need 2 <= world <= 8 and world | K");
    KZ_REQUIRE(rank >= 0 && rank < world, "kz_gemm_i8_allgather: rank out of range");
    KZ_REQUIRE(copy_ctas >= 2 && copy_ctas % 2 == 0 && copy_ctas <= 32, "kz_gemm_i8_allgather: copy_ctas must be even, 2..32");
    KZ_REQUIRE(flag_rows > 0 && flag_rows % 128 == 0 && M % flag_rows == 0,
               "kz_gemm_i8_allgather: flag_rows must be a multiple of 128 dividing M");
    KZ_REQUIRE((K / world) % 128 == 0, "kz_gemm_i8_allgather: K / world must be a multiple of 128");
    // every unit (row chunk of one rank's block) has at least one tile per copy CTA
    const int64_t tiles_per_unit = (flag_rows / 128) * ((K / world) / 128);
    if (copy_ctas > tiles_per_unit) copy_ctas = (int)std::max<int64_t>(2, tiles_per_unit & ~1ll);
    KZ_REQUIRE(copy_ctas <= tiles_per_unit, "kz_gemm_i8_allgather: row chunks too small for two copy CTAs");
    return gemm_i8_impl(A, B, M, N, K, K / world, row_scale, rs_stride, col_scale, cs_stride, nullptr, KZ_ACT_NONE,
                        out_f32, nullptr, ldo, absmax_partials, flags, token, rank, flag_rows, peer_A, peer_flags,
                        copy_ctas, stream);
}
