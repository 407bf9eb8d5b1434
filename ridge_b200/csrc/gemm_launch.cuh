// Launch glue shared by the instantiation files: turns a GemmTraits instance
// into a KernelEntry with a type-erased launcher.
#pragma once

#include <cstdio>

#include "gemm_registry.h"
#include "gemm_sm100.cuh"

namespace ridge_b200 {

template <int BM, int BN, int BK, int W>
cudaError_t launch_1cta(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                        const GemmParams* params, int grid_ctas, int smem_bytes,
                        cudaStream_t stream) {
    using T = GemmTraits<BM, BN, BK, W>;
    ridge_gemm_sm100<BM, BN, BK, W>
        <<<grid_ctas, T::kThreads, smem_bytes, stream>>>(*tmap_a, *tmap_b, *params);
    return cudaGetLastError();
}

template <int BM, int BN, int BK, int W>
KernelEntry make_entry_1cta() {
    using T = GemmTraits<BM, BN, BK, W>;
    KernelEntry e;
    e.BM = BM;
    e.BN = BN;
    e.BK = BK;
    e.warps = W;
    e.cta_group = 1;
    e.tile_a_rows = BM;
    e.tile_b_rows = BN;
    e.stage_bytes = T::kStageBytes;
    e.fixed_smem = T::kAlignSlack + T::kBarrierBytes;
    e.tmem_cols = T::kTmemCols;
    e.acc_bufs = T::kAccBufs;
    e.threads = T::kThreads;
    e.func = reinterpret_cast<const void*>(&ridge_gemm_sm100<BM, BN, BK, W>);
    e.launch = &launch_1cta<BM, BN, BK, W>;
    static char name[96];
    std::snprintf(name, sizeof(name), "ridge_gemm_sm100<%d, %d, %d, %d>", BM, BN, BK, W);
    e.name = name;
    return e;
}

}  // namespace ridge_b200
