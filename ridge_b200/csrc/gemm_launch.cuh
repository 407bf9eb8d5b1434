// Launch glue shared by the instantiation files: turns a GemmTraits instance
// into a KernelEntry with a type-erased launcher.
#pragma once

#include <cstdio>

#include "gemm_registry.h"
#include "gemm_sm100.cuh"

namespace ridge_b200 {

template <int BM, int BN, int BK, int W, int CG>
cudaError_t launch_gemm(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                        const CUtensorMap* tmap_c, const PeerMaps* peers,
                        const GemmParams* params, int grid_ctas, int smem_bytes,
                        cudaStream_t stream) {
    using T = GemmTraits<BM, BN, BK, W, CG>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid_ctas), 1, 1);
    cfg.blockDim = dim3(T::kThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(smem_bytes);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if constexpr (CG > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = CG;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, ridge_gemm_sm100<BM, BN, BK, W, CG>, *tmap_a, *tmap_b,
                              *tmap_c, *peers, *params);
}

template <int BM, int BN, int BK, int W, int CG>
KernelEntry make_entry() {
    using T = GemmTraits<BM, BN, BK, W, CG>;
    KernelEntry e;
    e.BM = BM;
    e.BN = BN;
    e.BK = BK;
    e.warps = W;
    e.cta_group = CG;
    e.tile_a_rows = T::kRowsA;
    e.tile_b_rows = T::kRowsB;
    e.epi_rows = T::kEpiRowsPerWarp;
    e.epi_cols = T::kEpiBoxCols;
    e.partial_floats = T::kPartialFloats;
    e.stage_bytes = T::kStageBytes;
    e.fixed_smem = T::kAlignSlack + T::kEpiBytes + T::kBarrierBytes;
    e.tmem_cols = T::kTmemCols;
    e.acc_bufs = T::kAccBufs;
    e.threads = T::kThreads;
    e.func = reinterpret_cast<const void*>(&ridge_gemm_sm100<BM, BN, BK, W, CG>);
    e.launch = &launch_gemm<BM, BN, BK, W, CG>;
    static char name[96];
    std::snprintf(name, sizeof(name), "ridge_gemm_sm100<%d, %d, %d, %d, %d>", BM, BN, BK, W, CG);
    e.name = name;
    return e;
}

}  // namespace ridge_b200
