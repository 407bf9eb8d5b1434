// Host-side registry of compiled GEMM kernels. Each instantiation file
// (gemm_inst_bm*.cu) contributes one KernelEntry per (BM, BN, BK, warps,
// cta_group) template instance; `stages` and `groupM` are runtime parameters of
// every kernel, so they do not multiply the number of instantiations.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <vector>

namespace ridge_b200 {

struct GemmParams;
struct PeerMaps;

using LaunchFn = cudaError_t (*)(const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                 const CUtensorMap* tmap_c, const PeerMaps* peers,
                                 const GemmParams* params, int grid_ctas, int smem_bytes,
                                 cudaStream_t stream);

struct KernelEntry {
    int BM, BN, BK, warps, cta_group;
    int tile_a_rows;      // rows of A one CTA loads per stage (BM, or BM/2 for a 2-CTA pair)
    int tile_b_rows;      // rows of B (N x K storage) one CTA loads per stage
    int epi_rows;         // rows of one epilogue TMA store box
    int epi_cols;         // columns of one epilogue TMA store box (32: 64B swizzle, 64: 128B)
    int partial_floats;   // FP32 floats of one CTA's split-K partial tile
    int stage_bytes;      // shared memory per pipeline stage, per CTA
    int fixed_smem;       // alignment slack + epilogue staging + barriers
    int tmem_cols;        // TMEM columns allocated per CTA
    int acc_bufs;         // TMEM accumulators
    int threads;
    const void* func;     // the __global__ function, for attribute queries
    LaunchFn launch;
    const char* name;
};

void register_bm64(std::vector<KernelEntry>& out);
void register_bm128(std::vector<KernelEntry>& out);
void register_bm256(std::vector<KernelEntry>& out);
void register_bm256_pair(std::vector<KernelEntry>& out);

}  // namespace ridge_b200
