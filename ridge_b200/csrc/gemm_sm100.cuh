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
//   * one MMA thread issues tcgen05.mma (128xBNx16 or 64xBNx16, kind::f16) that
//     read both operands straight from the 64B/128B-swizzled shared-memory
//     tiles and accumulate FP32 into TMEM (replaces ldmatrix + mma.sync and the
//     register accumulators);
//   * `warps` epilogue warps drain finished accumulators TMEM -> registers ->
//     FP16 -> global memory while the MMA thread already fills the second TMEM
//     accumulator with the next tile (replaces the smem-staged FP32 epilogue,
//     gemm-mma.cuh:293-342);
//   * the kernel is persistent: grid = min(tiles, SMs x CTAs/SM) and each CTA
//     walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... in grouped-M order.
//
// M, N and K need not be multiples of the tile: TMA zero-fills out-of-range
// operand elements and the epilogue predicates rows and columns.
//
// Warp roles (threads = (2 + warps) * 32):
//   warp 0        lane 0: TMA producer
//   warp 1        TMEM allocator; lane 0: MMA issuer
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

template <int BM_, int BN_, int BK_, int WARPS_>
struct GemmTraits {
    static constexpr int BM = BM_, BN = BN_, BK = BK_, kEpiWarps = WARPS_;
    static_assert(BM == 64 || BM == 128 || BM == 256, "BM must be 64, 128 or 256");
    static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
    static_assert(BK == 32 || BK == 64, "BK must be 32 or 64 (one 64B or 128B swizzle row)");
    static_assert(WARPS_ == 4 || WARPS_ == 8, "epilogue warps must be 4 or 8");

    static constexpr int kUmmaM = BM == 64 ? 64 : 128;  // rows per tcgen05.mma
    static constexpr int kMHalves = BM == 256 ? 2 : 1;  // MMAs per K-step along M
    static constexpr int kUmmaK = 16;                    // K per tcgen05.mma (FP16)
    static constexpr int kSwizzle = BK * 2;              // bytes per operand row
    static constexpr int kTileABytes = BM * BK * 2;
    static constexpr int kTileBBytes = BN * BK * 2;
    static constexpr int kStageBytes = kTileABytes + kTileBBytes;
    static constexpr int kAccCols = BN * kMHalves;       // FP32 TMEM columns per accumulator
    static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
    static constexpr int kTmemColsRaw = kAccCols * kAccBufs;
    static constexpr int kTmemCols = kTmemColsRaw <= 32    ? 32
                                     : kTmemColsRaw <= 64  ? 64
                                     : kTmemColsRaw <= 128 ? 128
                                     : kTmemColsRaw <= 256 ? 256
                                                           : 512;
    static constexpr int kThreads = (2 + kEpiWarps) * 32;
    static constexpr int kBarrierBytes = 256;
    static constexpr int kAlignSlack = 1024;
    static constexpr uint32_t kIdesc = make_idesc_f16_f32(kUmmaM, BN);

    static constexpr int smem_bytes(int stages) {
        return kAlignSlack + stages * kStageBytes + kBarrierBytes;
    }
};

struct GemmParams {
    __half* C;
    int M, N, K;
    long long ldc;
    int groupM;
    int stages;
    int* err;
};

// Grouped-M tile order, the same mapping as the reference launch order
// (gemm-mma.cuh:158-178): tiles are taken groupM row-tiles at a time, column by
// column inside the group, so CTAs running at the same moment share A row
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

template <int BM, int BN, int BK, int WARPS>
__global__ void __launch_bounds__((2 + WARPS) * 32, 1)
    ridge_gemm_sm100(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, const GemmParams p) {
    using T = GemmTraits<BM, BN, BK, WARPS>;
    extern __shared__ uint8_t smem_raw[];

    // 1024-byte alignment: the 128B swizzle pattern is a function of absolute
    // shared-memory address bits, so TMA writes and UMMA descriptor reads agree
    // only when every tile starts on a 1024-byte boundary.
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw_addr);

    const int stages = p.stages;
    const uint32_t bars = base + stages * T::kStageBytes;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (kMaxStages + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * kMaxStages + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * kMaxStages + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * kMaxStages + 4);
    uint8_t* bar_ptr = base_ptr + stages * T::kStageBytes;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 8 * (2 * kMaxStages + 5));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < T::kAccBufs; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), T::kEpiWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc<1>(smem_u32(tmem_slot), T::kTmemCols);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m = (p.M + BM - 1) / BM;
    const int num_n = (p.N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (p.K + BK - 1) / BK;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            int tm, tn;
            tile_coords(tile, num_m, num_n, p.groupM, tm, tn);
            for (int kb = 0; kb < num_kb; ++kb) {
                if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.err,
                               kErrTimeoutProducer)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = base + stage * T::kStageBytes;
                mbar_arrive_expect_tx(full_bar(stage), T::kStageBytes);
                tma_load_2d(sa, &tmap_a, full_bar(stage), kb * BK, tm * BM);
                tma_load_2d(sa + T::kTileABytes, &tmap_b, full_bar(stage), kb * BK, tn * BN);
                ++issued;
                if (++stage == stages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        if (!ok) {
            // Abort path: let every load already in flight land before the CTA
            // can exit. Issue i went to stage i % stages with parity
            // (i / stages) & 1; only the newest issue per stage can be pending.
            const long long first = issued > stages ? issued - stages : 0;
            for (long long i = first; i < issued; ++i) {
                mbar_wait(full_bar(int(i % stages)), uint32_t((i / stages) & 1), nullptr, p.err,
                          kErrTimeoutDrain);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, p.err, kErrTimeoutMma)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d_base = tmem_base + uint32_t(acc * T::kAccCols);
            for (int kb = 0; kb < num_kb; ++kb) {
                if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err, kErrTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = base + stage * T::kStageBytes;
                const uint32_t sb = sa + T::kTileABytes;
#pragma unroll
                for (int kk = 0; kk < BK / T::kUmmaK; ++kk) {
                    const uint64_t bdesc = make_smem_desc<T::kSwizzle>(sb + kk * T::kUmmaK * 2);
#pragma unroll
                    for (int h = 0; h < T::kMHalves; ++h) {
                        const uint64_t adesc = make_smem_desc<T::kSwizzle>(
                            sa + h * 128 * BK * 2 + kk * T::kUmmaK * 2);
                        umma_f16<1>(d_base + h * BN, adesc, bdesc, T::kIdesc,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(empty_bar(stage));  // frees the stage when these MMAs finish
                if (++stage == stages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            umma_commit(tfull_bar(acc));  // accumulator ready for the epilogue
            if (++acc == T::kAccBufs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (!ok) {
            // Abort path: wait for every MMA already issued before TMEM is freed.
            umma_commit(drain_bar);
            mbar_wait(drain_bar, 0, nullptr, p.err, kErrTimeoutDrain);
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue
        const int epi = warp - 2;
        const int quad = warp & 3;        // TMEM lane sub-partition this warp may access
        const int group = epi >> 2;       // column group when 8 warps share 4 sub-partitions
        constexpr int kGroups = WARPS / 4;
        constexpr int kChunks = BN / 32;  // 32 FP32 columns per tcgen05.ld
        const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int tm, tn;
            tile_coords(tile, num_m, num_n, p.groupM, tm, tn);
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait(tfull_bar(acc), acc_phase, abort_flag, p.err, kErrTimeoutEpilogue);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < T::kMHalves; ++h) {
                // M=128 UMMA: row r lives in TMEM lane r. M=64 UMMA: rows
                // 16q..16q+15 live in lanes 32q..32q+15 of sub-partition q.
                const int row_in_tile =
                    BM == 64 ? quad * 16 + lane : h * 128 + quad * 32 + lane;
                const bool row_live = (BM != 64 || lane < 16);
                const long long row = (long long)tm * BM + row_in_tile;
                const bool row_ok = row_live && row < p.M;
                __half* crow = p.C + row * p.ldc;
#pragma unroll
                for (int j = group; j < kChunks; j += kGroups) {
                    uint32_t r[32];
                    const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) +
                                           uint32_t(acc * T::kAccCols + h * BN + j * 32);
                    tmem_ld_32x32b_x32(taddr, r);
                    tmem_wait_ld();
                    const int col0 = tn * BN + j * 32;
                    if (row_ok) {
                        uint32_t packed[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            __half2 h2 = __floats2half2_rn(__uint_as_float(r[2 * e]),
                                                           __uint_as_float(r[2 * e + 1]));
                            packed[e] = *reinterpret_cast<uint32_t*>(&h2);
                        }
                        if (vec_ok && col0 + 32 <= p.N) {
                            uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
                            for (int v = 0; v < 4; ++v)
                                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1],
                                                    packed[4 * v + 2], packed[4 * v + 3]);
                        } else {
                            const __half* hv = reinterpret_cast<const __half*>(packed);
                            for (int e = 0; e < 32 && col0 + e < p.N; ++e) crow[col0 + e] = hv[e];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
            if (++acc == T::kAccBufs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, T::kTmemCols);
    }
}

}  // namespace ridge_b200
