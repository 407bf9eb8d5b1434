// The ridge GEMM family for B200 (sm_100a):  C[M,N] = A[M,K] * B[N,K]^T
//
//   A  FP16, row-major M x K (K contiguous, leading dimension lda)
//   B  FP16, column-major K x N, i.e. stored N x K with K contiguous (ldb)
//   C  FP16, row-major M x N (ldc); accumulation is FP32 in Tensor Memory.
//
// This is the Blackwell re-design of the tile-config-templated tensor-core GEMM
// that ridge models and autotunes (reference: bench/kernels/gemm-mma.cuh:116-343,
// an sm_80 cp.async + ldmatrix + mma.sync kernel). The tile knobs keep their
// meaning -- BM x BN output tile, BK reduction depth per pipeline stage, number
// of stages, grouped-M launch order (gemm-mma.cuh:158-178) -- but the machinery
// under them is new:
//
//   * one producer thread issues TMA bulk-tensor loads of the A and B tiles into
//     a `stages`-deep shared-memory ring guarded by full/empty mbarriers
//     (replaces the cp.async prologue/mainloop, gemm-mma.cuh:212-291);
//   * one MMA thread issues tcgen05.mma (kind::f16) that read both operands
//     straight from the 64B/128B-swizzled shared-memory tiles and accumulate
//     FP32 into TMEM (replaces ldmatrix + mma.sync and register accumulators);
//   * `warps` epilogue warps drain finished accumulators TMEM -> registers ->
//     FP16 -> swizzled shared-memory staging -> TMA bulk store, while the MMA
//     thread already fills the second TMEM accumulator with the next tile
//     (replaces the smem-staged FP32 epilogue, gemm-mma.cuh:293-342);
//   * the kernel is persistent: grid = min(tiles, SMs x CTAs/SM) tile units,
//     each walking tiles u, u + units, ... in grouped-M order.
//
// CG = 2 is the 2-CTA variant for 256-row tiles: a cluster of two CTAs on a
// TPC computes one 256 x BN tile with cta_group::2 MMAs (M = 256). Each CTA
// TMA-loads its own 128 rows of A and its own half of the BN rows of B, and
// holds the 128 x BN FP32 accumulator of its rows in its own TMEM; only the
// leader CTA (rank 0) issues MMAs, and its commits arrive on both CTAs'
// barriers. No load is multicast: every byte is fetched by the CTA that holds it.
//
// M, N and K need not be multiples of the tile: TMA zero-fills out-of-range
// operand elements and clips out-of-range stores.
//
// Warp roles (threads = (2 + warps) * 32):
//   warp 0        lane 0: TMA producer
//   warp 1        TMEM allocator; lane 0: MMA issuer (leader CTA only)
//   warps 2..     epilogue. A warp may only touch TMEM lanes 32*(warp%4) ..
//                 +31, so 4 epilogue warps cover the 128 accumulator rows and
//                 8 warps split the columns between two such groups.

#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "ptx_sm100.cuh"

namespace ridge_b200 {

constexpr int kMaxStages = 8;

template <int BM_, int BN_, int BK_, int WARPS_, int CG_>
struct GemmTraits {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, kEpiWarps = WARPS_, CG = CG_;
    static_assert(BM == 64 || BM == 128 || BM == 256, "BM must be 64, 128 or 256");
    static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
    static_assert(BK == 32 || BK == 64 || BK == 128,
                  "BK must be 32 or 64 (one 64B / 128B swizzle row) or 128 (two 128B atoms)");
    static_assert(WARPS_ == 4 || WARPS_ == 8, "epilogue warps must be 4 or 8");
    static_assert(CG == 1 || (CG == 2 && BM == 256), "the 2-CTA variant computes 256-row tiles");

    static constexpr int kRowsA = BM / CG;                 // A rows held by one CTA
    static constexpr int kRowsB = BN / CG;                 // B rows (N) held by one CTA
    static constexpr int kUmmaM = CG == 2 ? 256 : (BM == 64 ? 64 : 128);
    static constexpr int kMHalves = (CG == 1 && BM == 256) ? 2 : 1;  // MMAs per K-step along M
    static constexpr int kUmmaK = 16;                      // K per tcgen05.mma (FP16)
    static constexpr int kSwizzle = BK >= 64 ? 128 : BK * 2;  // bytes per swizzle row
    // K atoms per stage: a 128B-swizzled row holds 64 FP16 of K, so a BK=128
    // stage is two atoms, each (rows x 128 B), loaded by one 3-D TMA box.
    static constexpr int kAtoms = BK >= 64 ? BK / 64 : 1;
    static constexpr int kAtomK = BK / kAtoms;               // K per atom
    static constexpr int kTileABytes = kRowsA * BK * 2;
    static constexpr int kTileBBytes = kRowsB * BK * 2;
    static constexpr int kStageBytes = kTileABytes + kTileBBytes;
    static constexpr int kAccCols = BN * kMHalves;         // FP32 TMEM columns per accumulator
    static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
    static constexpr int kTmemColsRaw = kAccCols * kAccBufs;
    static constexpr int kTmemCols = kTmemColsRaw <= 32    ? 32
                                     : kTmemColsRaw <= 64  ? 64
                                     : kTmemColsRaw <= 128 ? 128
                                     : kTmemColsRaw <= 256 ? 256
                                                           : 512;
    static constexpr int kThreads = (2 + kEpiWarps) * 32;
    // Epilogue: each warp drains kEpiPerWarp chunks of 32 rows x 32 columns,
    // kEpiLd at a time. With pairs, a pair of column-adjacent chunks goes out
    // as one 32 x 64 TMA store from a 4 KB staging buffer (rows of 128 B,
    // 128B-swizzled); otherwise each chunk is a 32 x 32 store from one of two
    // 2 KB buffers (rows of 64 B, 64B-swizzled). 4 KB of staging per warp
    // either way.
    static constexpr int kEpiRowsPerWarp = BM == 64 ? 16 : 32;
    static constexpr int kEpiGroups = kEpiWarps / 4;  // warps sharing a TMEM lane quarter
    static constexpr int kEpiPerHalf = (BN / 32) / kEpiGroups;
    static constexpr int kEpiPerWarp = kMHalves * kEpiPerHalf;
    static constexpr int kEpiLd = kEpiPerHalf % 2 == 0 ? 2 : 1;
    static constexpr int kEpiBoxCols = 32 * kEpiLd;
    static constexpr int kEpiChunkBytes = 32 * 64;
    static constexpr int kEpiBytes = kEpiWarps * 2 * kEpiChunkBytes;
    // FP32 floats of one CTA's split-K partial tile: 128 lanes x BN per M-half
    // (an M=64 tile keeps the 32-lane chunk layout, half of it unused).
    static constexpr int kPartialFloats = kMHalves * 128 * BN;
    static constexpr int kBarrierBytes = 256;
    static constexpr int kAlignSlack = 1024;
    static constexpr uint32_t kIdesc = make_idesc_f16_f32(kUmmaM, BN);

    static constexpr int smem_bytes(int stages) {
        return kAlignSlack + stages * kStageBytes + kEpiBytes + kBarrierBytes;
    }
};

// Extra destinations of every C tile: the same tile coordinates stored through
// each of these maps too (another GPU's copy of C, over NVLink). Used by the
// fused N-slab GEMM + all-gather; empty for an ordinary launch.
constexpr int kMaxPeers = 7;
struct PeerMaps {
    CUtensorMap map[kMaxPeers];
};

struct GemmParams {
    __half* C;
    int M, N, K;
    long long ldc;
    int groupM;
    int stages;
    int tma_store;  // 1: epilogue stores through the C tensor map; 0: direct st.global
    int epi_stride; // staging bytes per epilogue warp: 4096, or 8192 for two pair buffers
    int tma_issuers; // producer threads issuing TMA loads: 1, 2 or 4
    int num_peers;  // destinations in PeerMaps besides tmap_c (TMA-store epilogue only)
    int* err;
    // Split-K tail ("data-parallel + stream-K"): tiles [0, dp_tiles) run whole,
    // one per unit per round; the remaining sk_tiles tiles are each split into
    // sk_splits contiguous K ranges, one range per unit, which that unit
    // computes before (sk_first) or after its whole tiles. Each epilogue warp of a split takes a ticket from
    // counters[2 * ((sk * CG + rank) * warps + warp)] when its accumulator is
    // ready; all but the last publish their FP32 partial into their split's
    // slot of `workspace` and count it in the next int; the last waits for
    // those (they are already running), folds them into its registers in
    // split order and stores C, then resets both ints to 0, so they start at
    // 0 every launch.
    int dp_tiles;
    int sk_tiles;
    int sk_splits;
    int sk_first;  // 1: a unit's split range precedes its whole tiles; 0: it follows them
    float* workspace;
    int* counters;
};

// One unit of work: a tile and the K-block range [kb0, kb1) to accumulate.
// split < 0 marks a whole (data-parallel) tile.
struct WorkItem {
    int tile, kb0, kb1, split, sk;
};

__device__ __forceinline__ bool get_item(const GemmParams& p, int unit, int num_units, int num_kb,
                                         int i, WorkItem& w) {
    const bool has_split = unit < p.sk_tiles * p.sk_splits;
    // The split tiles are the first sk_tiles tiles of the grouped order when
    // they run first (so they share L2 panels with the first whole tiles, run
    // at the same time) and the last ones otherwise.
    const int whole0 = p.sk_first ? p.sk_tiles : 0;
    auto split_item = [&]() {
        w.sk = unit / p.sk_splits;
        w.split = unit - w.sk * p.sk_splits;
        w.tile = p.sk_first ? w.sk : p.dp_tiles + w.sk;
        w.kb0 = int((long long)num_kb * w.split / p.sk_splits);
        w.kb1 = int((long long)num_kb * (w.split + 1) / p.sk_splits);
        return true;
    };
    // With sk_first a unit's split-K range comes before its whole tiles, so
    // its partial exchange overlaps the next tile's MMAs on the other TMEM
    // accumulator instead of trailing the last one; otherwise it comes last.
    if (has_split && p.sk_first) {
        if (i == 0) return split_item();
        --i;
    }
    const int dp_count = p.dp_tiles > unit ? (p.dp_tiles - unit + num_units - 1) / num_units : 0;
    if (i < dp_count) {
        w.tile = whole0 + unit + i * num_units;
        w.kb0 = 0;
        w.kb1 = num_kb;
        w.split = -1;
        w.sk = -1;
        return true;
    }
    if (has_split && !p.sk_first && i == dp_count) return split_item();
    return false;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* ptr) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

// Grouped-M tile order, the same mapping as the reference launch order
// (gemm-mma.cuh:158-178): tiles are taken groupM row-tiles at a time, column by
// column inside the group, so units running at the same moment share A row
// panels and B column panels in L2.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int groupM, int& tm,
                                            int& tn) {
    const int per_group = groupM * num_n;
    const int group = tile / per_group;
    const int first_m = group * groupM;
    const int rows = min(num_m - first_m, groupM);
    const int in_group = tile - group * per_group;
    tm = first_m + in_group % rows;
    tn = in_group / rows;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

#ifdef RIDGE_TRACE
// Timeline probe (built only with -DRIDGE_TRACE, never in the library): per
// CTA, [0] entry, [1 + i] MMA issue of item i done, [32 + i] epilogue of item i
// done (warp 2), [63] exit, in %globaltimer nanoseconds.
// (relocatable device code: defined once, in gemm_host.cu)
extern __device__ unsigned long long g_ridge_trace[512][64];
#define RIDGE_TRACE_AT(slot)                                                   \
    do {                                                                       \
        if (blockIdx.x < 512) g_ridge_trace[blockIdx.x][(slot)] = global_timer_ns(); \
    } while (0)
#else
#define RIDGE_TRACE_AT(slot) \
    do {                     \
    } while (0)
#endif

template <int BM, int BN, int BK, int WARPS, int CG>
__global__ void __launch_bounds__((2 + WARPS) * 32, 1)
    ridge_gemm_sm100(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_c,
                     const __grid_constant__ PeerMaps peers, const GemmParams p) {
    using T = GemmTraits<BM, BN, BK, WARPS, CG>;
    extern __shared__ uint8_t smem_raw[];

    // 1024-byte alignment: the swizzle patterns are functions of absolute
    // shared-memory address bits, so TMA writes and UMMA descriptor reads agree
    // only when every tile starts on a 1024-byte boundary.
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw_addr);

    const int stages = p.stages;
    const uint32_t epi_base = base + stages * T::kStageBytes;
    const uint32_t bars = epi_base + uint32_t(T::kEpiWarps * p.epi_stride);
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (kMaxStages + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * kMaxStages + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * kMaxStages + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * kMaxStages + 4);
    uint8_t* bar_ptr = base_ptr + (bars - base);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 8 * (2 * kMaxStages + 5));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_cta_rank() : 0u;
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        RIDGE_TRACE_AT(0);
        for (int s = 0; s < stages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < T::kAccBufs; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), CG * T::kEpiWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        if (p.tma_store) tma_prefetch_desc(&tmap_c);
        for (int d = 0; d < p.num_peers; ++d) tma_prefetch_desc(&peers.map[d]);
    }
    if (warp == 1) {
        tmem_alloc<CG>(smem_u32(tmem_slot), T::kTmemCols);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    __syncwarp();  // barrier.cluster is .aligned: every warp arrives converged
    if constexpr (CG == 2) {
        cluster_sync();  // both CTAs' barriers and TMEM exist before any remote use
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m = (p.M + BM - 1) / BM;
    const int num_n = (p.N + BN - 1) / BN;
    const int num_kb = (p.K + BK - 1) / BK;
    const int unit = blockIdx.x / CG;
    const int num_units = gridDim.x / CG;

    if (warp == 0 && lane < p.tma_issuers) {
        // ------------------------------------------------------ TMA producer
        // tma_issuers (1, 2 or 4) issuing threads. With 4, stages alternate
        // between two lane pairs; with 2 or 4, lane 2p of a pair loads A (and
        // arms the stage barrier) while lane 2p+1 loads B; with 1, lane 0
        // loads both. In a 2-CTA pair both CTAs' loads complete on the
        // leader's full barrier, armed with the bytes of both. A load may
        // complete before its phase is armed; the phase cannot finish before
        // the arming lane arrives.
        const int npairs = p.tma_issuers >= 4 ? 2 : 1;
        const bool single = p.tma_issuers == 1;
        const bool loads_a = single || (lane & 1) == 0;
        const int my_pair = single ? 0 : lane >> 1;
        const uint32_t leader_full0 = CG == 2 ? map_to_cta(full_bar(0), 0) : full_bar(0);
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;  // stages issued by all lanes so far (this lane's view)
        bool ok = true;
        WorkItem w;
        for (int it = 0; ok && get_item(p, unit, num_units, num_kb, it, w); ++it) {
            int tm, tn;
            tile_coords(w.tile, num_m, num_n, p.groupM, tm, tn);
            const int a_row = tm * BM + int(rank) * T::kRowsA;
            const int b_row = tn * BN + int(rank) * T::kRowsB;
            for (int kb = w.kb0; kb < w.kb1; ++kb) {
                if (int(issued % npairs) == my_pair) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.err,
                                   kErrTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = base + stage * T::kStageBytes;
                    const uint32_t fb =
                        CG == 1 ? full_bar(stage) : leader_full0 + 8u * uint32_t(stage);
                    if (loads_a && leader)
                        mbar_arrive_expect_tx(full_bar(stage), CG * T::kStageBytes);
                    auto load = [&](bool a_side) {
                        const uint32_t dst = a_side ? sa : sa + T::kTileABytes;
                        const void* map = a_side ? static_cast<const void*>(&tmap_a)
                                                 : static_cast<const void*>(&tmap_b);
                        const int row = a_side ? a_row : b_row;
                        if constexpr (T::kAtoms == 1) {
                            if constexpr (CG == 1)
                                tma_load_2d(dst, map, fb, kb * BK, row);
                            else
                                tma_load_2d_pair(dst, map, fb, kb * BK, row);
                        } else {
                            if constexpr (CG == 1)
                                tma_load_3d(dst, map, fb, 0, row, kb * T::kAtoms);
                            else
                                tma_load_3d_pair(dst, map, fb, 0, row, kb * T::kAtoms);
                        }
                    };
                    load(loads_a);
                    if (single) load(false);
                }
                ++issued;
                if (++stage == stages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        if (!ok && leader && loads_a) {
            // Abort path: let every load already in flight land before the CTA
            // can exit (in a pair the leader's barriers count the follower's
            // bytes too, and neither CTA exits before the final cluster
            // barrier). Stage issue i went to ring slot i % stages with parity
            // (i / stages) & 1; only the newest issue per slot can be pending,
            // and this lane armed the slots with i & 1 == my_pair.
            const long long first = issued > stages ? issued - stages : 0;
            for (long long i = first; i < issued; ++i) {
                if (int(i % npairs) != my_pair) continue;
                mbar_wait(full_bar(int(i % stages)), uint32_t((i / stages) & 1), nullptr, p.err,
                          kErrTimeoutDrain);
            }
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        WorkItem w;
        for (int it = 0; ok && get_item(p, unit, num_units, num_kb, it, w); ++it) {
            if (!mbar_wait<CG == 2>(tempty_bar(acc), acc_phase ^ 1u, abort_flag, p.err,
                                    kErrTimeoutMma)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d_base = tmem_base + uint32_t(acc * T::kAccCols);
            for (int kb = w.kb0; kb < w.kb1; ++kb) {
                if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err, kErrTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = base + stage * T::kStageBytes;
                const uint32_t sb = sa + T::kTileABytes;
#pragma unroll
                for (int kk = 0; kk < BK / T::kUmmaK; ++kk) {
                    // K step kk lives in atom kk / (atom K / 16), at byte
                    // offset 32 * (kk mod that) inside the atom's rows.
                    constexpr int kStepsPerAtom = T::kAtomK / T::kUmmaK;
                    const int atom = kk / kStepsPerAtom;
                    const int in_atom = (kk % kStepsPerAtom) * T::kUmmaK * 2;
                    const uint64_t bdesc = make_smem_desc<T::kSwizzle>(
                        sb + atom * T::kRowsB * T::kSwizzle + in_atom);
#pragma unroll
                    for (int h = 0; h < T::kMHalves; ++h) {
                        const uint64_t adesc = make_smem_desc<T::kSwizzle>(
                            sa + atom * T::kRowsA * T::kSwizzle + h * 128 * T::kSwizzle +
                            in_atom);
                        umma_f16<CG>(d_base + h * BN, adesc, bdesc, T::kIdesc,
                                     (kb > w.kb0 || kk > 0) ? 1u : 0u);
                    }
                }
                // Free the stage (in both CTAs of a pair) when these MMAs finish.
                if constexpr (CG == 1)
                    umma_commit(empty_bar(stage));
                else
                    umma_commit_pair(empty_bar(stage), 0x3);
                if (++stage == stages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (it < 31) RIDGE_TRACE_AT(1 + it);
            // Accumulator ready for the epilogue (of both CTAs of a pair).
            if constexpr (CG == 1)
                umma_commit(tfull_bar(acc));
            else
                umma_commit_pair(tfull_bar(acc), 0x3);
            if (++acc == T::kAccBufs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (!ok) {
            // Abort path: wait for every MMA already issued before TMEM is freed.
            if constexpr (CG == 1)
                umma_commit(drain_bar);
            else
                umma_commit_pair(drain_bar, 0x1);
            mbar_wait(drain_bar, 0, nullptr, p.err, kErrTimeoutDrain);
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue
        const int epi = warp - 2;
        const int quad = warp & 3;        // TMEM lane sub-partition this warp may access
        const int group = epi >> 2;       // column group when 8 warps share 4 sub-partitions
        constexpr int kChunks = BN / 32;  // 32 FP32 columns per tcgen05.ld
        const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
        // Remote (leader) accumulator-empty barrier for the follower of a pair.
        const uint32_t tempty0 = CG == 2 ? map_to_cta(tempty_bar(0), 0) : tempty_bar(0);
        const uint32_t stage_buf0 = epi_base + uint32_t(epi * p.epi_stride);
        const bool two_pair_bufs = p.epi_stride >= 2 * 4096;
        uint32_t pidx = 0;  // pair stores of this warp so far
        int buf = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        WorkItem w;
        for (int it = 0; get_item(p, unit, num_units, num_kb, it, w); ++it) {
            int tm, tn;
            tile_coords(w.tile, num_m, num_n, p.groupM, tm, tn);
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(tfull_bar(acc), acc_phase, abort_flag, p.err, kErrTimeoutEpilogue);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            // Split-K bookkeeping for this item: where the tile's FP32 partial
            // slots live (one per split, in split order) and this warp's two
            // counters: [0] tickets the arrivals, [1] counts published partials.
            constexpr long long kTileFloats = T::kPartialFloats;
            float* ws_tile = nullptr;
            int* counter = nullptr;
            if (w.split >= 0) {
                counter = p.counters + 2 * ((w.sk * CG + int(rank)) * WARPS + epi);
                const long long slot0 = (long long)w.sk * p.sk_splits;
                ws_tile = p.workspace + (slot0 * CG + rank) * kTileFloats;
            }
            // This warp's chunks of the tile are drained kLd at a time:
            // both TMEM loads are issued before one wait (tcgen05.wait::ld
            // waits for all of a thread's loads), and the next group's loads
            // are issued before the current group is stored, so the TMEM load
            // latency (hundreds of cycles while the tensor core is writing the
            // other accumulator) is paid once per kLd chunks and hides behind
            // the stores.
            constexpr int kPerHalf = T::kEpiPerHalf;
            constexpr int kPerWarp = T::kEpiPerWarp;
            constexpr int kLd = T::kEpiLd;
            // chunk ci of this warp: M-half ci / kPerHalf, column chunk
            // group * kPerHalf + ci % kPerHalf (a warp's chunks are adjacent
            // columns, so a pair forms one 64-column store)
            auto chunk_taddr = [&](int ci) {
                const int hh = ci / kPerHalf, jj = group * kPerHalf + ci % kPerHalf;
                return tmem_base + (uint32_t(quad * 32) << 16) +
                       uint32_t(acc * T::kAccCols + hh * BN + jj * 32);
            };
            const int tile_row0 = tm * BM + int(rank) * T::kRowsA;
            // Split-K partial chunks use a lane-contiguous layout: float4 v of
            // lane L of chunk c sits at ((c * 8 + v) * 32 + L), so every
            // warp-wide store or load covers 512 contiguous bytes. Producer
            // and folding warps map warps to chunks identically.
            auto ws_offset = [&](int ci) {
                const int h = ci / kPerHalf, j = group * kPerHalf + ci % kPerHalf;
                const long long chunk_id = (long long)(h * kChunks + j) * 4 + quad;
                return chunk_id * 8 * 32 * 4 + lane * 4;
            };
            auto warp_row0_of = [&](int ci) {
                // M=128 / 256-pair UMMA: row r of this CTA lives in TMEM lane r.
                // M=64 UMMA: rows 16q..16q+15 live in lanes 32q..32q+15.
                return BM == 64 ? quad * 16 : (ci / kPerHalf) * 128 + quad * 32;
            };
            // A warp whose rows all lie at or beyond M has nothing to reduce.
            auto warp_live_of = [&](int ci) {
                return (long long)tile_row0 + warp_row0_of(ci) < p.M;
            };
            auto publish = [&](int ci, const uint32_t (&r)[32]) {
                // Publish this split's FP32 partial chunk into its slot.
                if (!warp_live_of(ci)) return;
                float4* dst = reinterpret_cast<float4*>(
                    ws_tile + (long long)w.split * CG * kTileFloats + ws_offset(ci));
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    __stcg(dst + v * 32, make_float4(__uint_as_float(r[4 * v]),
                                                     __uint_as_float(r[4 * v + 1]),
                                                     __uint_as_float(r[4 * v + 2]),
                                                     __uint_as_float(r[4 * v + 3])));
            };
            auto pack = [&](const uint32_t (&r)[32], uint32_t (&packed)[16]) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    packed[e] = pack_half2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
            };
            // Last arrival of a split tile: r holds this split's own partial
            // (split w.split); fold in every other split's published partial so
            // that r becomes p_0 + p_1 + ... + p_{s-1} added left to right in
            // split order -- the same sum whichever split arrives last, so the
            // result is deterministic. The prefix before w.split is summed
            // apart, then added to r (x + y == y + x exactly), and the later
            // partials are added to r in place.
            auto fold_into = [&](int ci, uint32_t (&r)[32]) {
                if (!warp_live_of(ci)) return;
                auto src = [&](int sp) {
                    return reinterpret_cast<const float4*>(
                        ws_tile + (long long)sp * CG * kTileFloats + ws_offset(ci));
                };
                auto add_into_r = [&](const float4 (&q)[8]) {
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        r[4 * v] = __float_as_uint(__uint_as_float(r[4 * v]) + q[v].x);
                        r[4 * v + 1] = __float_as_uint(__uint_as_float(r[4 * v + 1]) + q[v].y);
                        r[4 * v + 2] = __float_as_uint(__uint_as_float(r[4 * v + 2]) + q[v].z);
                        r[4 * v + 3] = __float_as_uint(__uint_as_float(r[4 * v + 3]) + q[v].w);
                    }
                };
                if (w.split > 0) {
                    float4 pre[8];
#pragma unroll
                    for (int v = 0; v < 8; ++v) pre[v] = __ldcg(src(0) + v * 32);
                    for (int sp = 1; sp < w.split; ++sp) {
                        float4 q[8];
#pragma unroll
                        for (int v = 0; v < 8; ++v) q[v] = __ldcg(src(sp) + v * 32);
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            pre[v].x += q[v].x;
                            pre[v].y += q[v].y;
                            pre[v].z += q[v].z;
                            pre[v].w += q[v].w;
                        }
                    }
                    add_into_r(pre);
                }
                for (int sp = w.split + 1; sp < p.sk_splits; ++sp) {
                    float4 q[8];
#pragma unroll
                    for (int v = 0; v < 8; ++v) q[v] = __ldcg(src(sp) + v * 32);
                    add_into_r(q);
                }
            };
            auto store_chunk = [&](int ci, const uint32_t (&packed)[16]) {
                const int j = group * kPerHalf + ci % kPerHalf;
                const int warp_row0 = warp_row0_of(ci);
                const int col0 = tn * BN + j * 32;
                if (p.tma_store) {
                    // Stage this warp's 32 x 32 chunk (one 64-byte row per
                    // lane, 64B-swizzled: 16-byte unit c of row r sits at
                    // unit c ^ ((r >> 1) & 3), conflict-free) and hand it to
                    // a TMA store, which clips rows/columns outside C.
                    // Buffer b's stores are issued (and waited on) by lane b,
                    // so the warp has two issuing threads.
                    const uint32_t sbuf = stage_buf0 + uint32_t(buf * T::kEpiChunkBytes);
                    if (lane == buf) tma_store_wait_read<0>();  // this buffer's last store has read it
                    __syncwarp();
                    const uint32_t row_addr = sbuf + uint32_t(lane * 64);
                    const uint32_t sw = uint32_t((lane >> 1) & 3);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                         row_addr + ((uint32_t(c) ^ sw) << 4)),
                                     "r"(packed[4 * c]), "r"(packed[4 * c + 1]),
                                     "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3])
                                     : "memory");
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == buf) {
                        tma_store_2d(&tmap_c, sbuf, col0, tile_row0 + warp_row0);
#pragma unroll 1
                        for (int d = 0; d < p.num_peers; ++d)
                            tma_store_2d(&peers.map[d], sbuf, col0, tile_row0 + warp_row0);
                        tma_store_commit();
                    }
                    buf ^= 1;
                    return;
                }
                const bool row_live = (BM != 64 || lane < 16);
                const long long row = (long long)tile_row0 + warp_row0 + lane;
                if (!row_live || row >= p.M) return;
                __half* crow = p.C + row * p.ldc;
                if (vec_ok && col0 + 32 <= p.N) {
                    uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2],
                                            packed[4 * v + 3]);
                } else {
                    // Ragged columns: element stores, fully unrolled so
                    // `packed` stays in registers.
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const uint32_t word = packed[e >> 1];
                        const unsigned short bits = (e & 1) ? (unsigned short)(word >> 16)
                                                            : (unsigned short)(word & 0xffff);
                        if (col0 + e < p.N) crow[col0 + e] = __ushort_as_half(bits);
                    }
                }
            };
            // One 32 x 64 TMA store of chunks ci, ci + 1 (column-adjacent).
            // Row r of the 4 KB buffer is 128 B; its 16-byte unit c sits at
            // c ^ (r & 7) (the 128B swizzle, conflict-free).
            auto store_pair = [&](int ci, const uint32_t (&pa)[16], const uint32_t (&pb)[16]) {
                const int j = group * kPerHalf + ci % kPerHalf;
                const int col0 = tn * BN + j * 32;
                // Destination d (0: this C, d > 0: peer d - 1) is stored by lane
                // d, so the copies to other GPUs leave in parallel. One buffer:
                // the previous pair's stores have read it; two: the stores
                // before those have read this one (each issuing lane waits on
                // its own stores).
                const uint32_t sbuf = stage_buf0 + (two_pair_bufs ? (pidx & 1u) * 4096u : 0u);
                if (lane <= p.num_peers) {
                    if (two_pair_bufs)
                        tma_store_wait_read<1>();
                    else
                        tma_store_wait_read<0>();
                }
                __syncwarp();
                const uint32_t row_addr = sbuf + uint32_t(lane * 128);
                const uint32_t sw = uint32_t(lane & 7);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                     row_addr + ((uint32_t(c) ^ sw) << 4)),
                                 "r"(pa[4 * c]), "r"(pa[4 * c + 1]), "r"(pa[4 * c + 2]),
                                 "r"(pa[4 * c + 3])
                                 : "memory");
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                                     row_addr + ((uint32_t(c + 4) ^ sw) << 4)),
                                 "r"(pb[4 * c]), "r"(pb[4 * c + 1]), "r"(pb[4 * c + 2]),
                                 "r"(pb[4 * c + 3])
                                 : "memory");
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane <= p.num_peers) {
                    tma_store_2d(lane == 0 ? static_cast<const void*>(&tmap_c)
                                           : static_cast<const void*>(&peers.map[lane - 1]),
                                 sbuf, col0, tile_row0 + warp_row0_of(ci));
                    tma_store_commit();
                }
                ++pidx;
            };
            uint32_t ra[32], rb[32];
            auto load_group = [&](int ci) {
                tmem_ld_32x32b_x32(chunk_taddr(ci), ra);
                if constexpr (kLd == 2) tmem_ld_32x32b_x32(chunk_taddr(ci + 1), rb);
            };
            auto wait_group = [&]() {
                tmem_wait_ld(ra);
                if constexpr (kLd == 2) tmem_wait_ld(rb);
            };
            auto store_group = [&](int ci, const uint32_t (&pa)[16], const uint32_t (&pb)[16]) {
                if constexpr (kLd == 2) {
                    if (p.tma_store) {
                        store_pair(ci, pa, pb);
                    } else {
                        store_chunk(ci, pa);
                        store_chunk(ci + 1, pb);
                    }
                } else {
                    store_chunk(ci, pa);
                }
            };
            // Every TMEM read of this accumulator is done: hand it back.
            auto release_acc = [&]() {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 1)
                        mbar_arrive(tempty_bar(acc));
                    else
                        mbar_arrive_cluster(tempty0 + 8u * acc);
                }
            };
            load_group(0);
            wait_group();
            if (w.split >= 0) {
                // Split-K item (warp-uniform branch). The warp takes a ticket
                // as soon as its accumulator is ready. Every split but the
                // last to arrive publishes its FP32 partial and counts it; the
                // last waits for those s - 1 partials and folds them into its
                // own accumulator registers, then stores C. The last only ever
                // waits for splits that have already taken a ticket, i.e. that
                // are running and past their MMAs, so no split needs another
                // to be scheduled; the wait is bounded all the same.
                int ticket = 0;
                if (lane == 0) ticket = atomicAdd(counter, 1);
                ticket = __shfl_sync(0xffffffffu, ticket, 0);
                if (ticket != p.sk_splits - 1) {
#pragma unroll 1
                    for (int ci = 0; ci < kPerWarp; ci += kLd) {
                        publish(ci, ra);
                        if constexpr (kLd == 2) publish(ci + 1, rb);
                        if (ci + kLd < kPerWarp) {
                            __syncwarp();
                            load_group(ci + kLd);
                            wait_group();
                        }
                    }
                    release_acc();
                    __threadfence();  // the partial is visible before it is counted
                    __syncwarp();
                    if (lane == 0) atomicAdd(counter + 1, 1);
                } else {
                    if (lane == 0) {
                        const int want = p.sk_splits - 1;
                        if (ld_acquire_gpu(counter + 1) < want) {
                            const uint64_t t0 = global_timer_ns();
                            while (ld_acquire_gpu(counter + 1) < want) {
                                if (*abort_flag) break;
                                if (global_timer_ns() - t0 > RIDGE_WAIT_LIMIT_NS) {
                                    *abort_flag = 1;
                                    atomicCAS(p.err, 0, int(kErrTimeoutSplitK));
                                    break;
                                }
                            }
                        }
                    }
                    __syncwarp();
                    __threadfence();  // the partials published before the count
#pragma unroll 1
                    for (int ci = 0; ci < kPerWarp; ci += kLd) {
                        const bool more = ci + kLd < kPerWarp;
                        uint32_t pa[16], pb[16];
                        fold_into(ci, ra);
                        pack(ra, pa);
                        if constexpr (kLd == 2) {
                            fold_into(ci + 1, rb);
                            pack(rb, pb);
                        }
                        if (more) {
                            __syncwarp();
                            load_group(ci + kLd);
                        }
                        store_group(ci, pa, pb);
                        if (more) wait_group();
                    }
                    release_acc();
                    if (lane == 0) {  // every split arrived: ready for the next launch
                        counter[0] = 0;
                        counter[1] = 0;
                    }
                }
            } else {
#pragma unroll 1
                for (int ci = 0; ci < kPerWarp; ci += kLd) {
                    const bool more = ci + kLd < kPerWarp;
                    uint32_t pa[16], pb[16];
                    pack(ra, pa);
                    if constexpr (kLd == 2) pack(rb, pb);
                    if (more) {
                        __syncwarp();
                        load_group(ci + kLd);  // lands while this group is stored
                    }
                    store_group(ci, pa, pb);
                    if (more) wait_group();
                }
                release_acc();
            }
            if (warp == 2 && lane == 0 && it < 31) RIDGE_TRACE_AT(32 + it);
            if (++acc == T::kAccBufs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // lanes 0 and 1 issue chunk stores, lanes 0..num_peers pair stores
        if (p.tma_store && (lane < 2 || lane <= p.num_peers)) tma_store_wait_all<0>();
    }

    tc_fence_before();
    __syncwarp();
    if constexpr (CG == 2) {
        cluster_sync();  // neither CTA frees TMEM or exits while its peer may still use it
    } else {
        __syncthreads();
    }
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<CG>(tmem_base, T::kTmemCols);
    }
    if (threadIdx.x == 0) RIDGE_TRACE_AT(63);
}

}  // namespace ridge_b200
