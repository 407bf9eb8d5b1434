// N-slab sharding helpers for a GEMM split across ranks by column slabs of B
// with A replicated (each rank computes C[:, n0:n0+n_slab] = A * B_slab).
//
// The reference is single-GPU (README.md:154 there); this is the B200 build's
// multi-GPU mode. The data path needs no collective: a slab is an ordinary
// GEMM on rows [n0, n0 + n_slab) of B's N x K storage. When the caller wants
// the full C on every rank, the slabs are all-gathered (NCCL over NVLink, from
// the host side) into a slab-major buffer, and ridge_slabs_to_rowmajor
// re-lays them out into row-major C.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/ridge_b200.h"

namespace {

// C[i, r*slab_cols + j] = slabs[r][i][j], one thread per 8 halves (16 bytes)
// when every row start is 16-byte aligned, else per half.
__global__ void slabs_to_rowmajor_vec(const uint4* __restrict__ slabs, uint4* __restrict__ C,
                                      int64_t M, int64_t N, int32_t nranks, int64_t slab_cols,
                                      int64_t ldc) {
    const int64_t vec_per_row = slab_cols / 8;
    const int64_t total = int64_t(nranks) * M * vec_per_row;
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
         v += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = v / (M * vec_per_row);
        const int64_t rem = v - r * M * vec_per_row;
        const int64_t i = rem / vec_per_row;
        const int64_t j8 = rem - i * vec_per_row;
        const int64_t col = r * slab_cols + j8 * 8;
        if (col >= N) continue;
        if (col + 8 <= N) {
            C[(i * ldc + col) / 8] = slabs[v];
        } else {
            const __half* src = reinterpret_cast<const __half*>(slabs + v);
            __half* dst = reinterpret_cast<__half*>(C) + i * ldc + col;
            for (int e = 0; e < 8 && col + e < N; ++e) dst[e] = src[e];
        }
    }
}

__global__ void slabs_to_rowmajor_scalar(const uint16_t* __restrict__ slabs,
                                         uint16_t* __restrict__ C, int64_t M, int64_t N,
                                         int32_t nranks, int64_t slab_cols, int64_t ldc) {
    const int64_t total = int64_t(nranks) * M * slab_cols;
    for (int64_t x = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; x < total;
         x += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = x / (M * slab_cols);
        const int64_t rem = x - r * M * slab_cols;
        const int64_t i = rem / slab_cols;
        const int64_t j = rem - i * slab_cols;
        const int64_t col = r * slab_cols + j;
        if (col < N) C[i * ldc + col] = slabs[x];
    }
}

// ncclAllGather from the process's libnccl.so.2: the one the caller's
// communicator came from (a framework usually has it loaded already), so the
// library does not link NCCL itself.
using AllGatherFn = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                                     cudaStream_t);
using AllReduceFn = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                     ncclComm_t, cudaStream_t);
void* nccl_symbol(const char* name) {
    static std::once_flag once;
    static void* lib = nullptr;
    std::call_once(once, [] {
        lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    });
    return lib ? dlsym(lib, name) : nullptr;
}
AllGatherFn nccl_allgather() { return reinterpret_cast<AllGatherFn>(nccl_symbol("ncclAllGather")); }
AllReduceFn nccl_allreduce() { return reinterpret_cast<AllReduceFn>(nccl_symbol("ncclAllReduce")); }

// One int per device for the completion barrier's all-reduce.
int* barrier_word() {
    static std::mutex mu;
    static int* words[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev] && cudaMalloc(&words[dev], sizeof(int)) != cudaSuccess) words[dev] = nullptr;
    return words[dev];
}

}  // namespace

extern "C" {

int ridge_slab_bounds(int64_t N, int32_t nranks, int32_t rank, int64_t align, int64_t* n0,
                      int64_t* n_slab) {
    if (N < 0 || nranks <= 0 || rank < 0 || rank >= nranks || align <= 0 || !n0 || !n_slab)
        return RIDGE_EINVAL;
    const int64_t per = ((N + nranks - 1) / nranks + align - 1) / align * align;
    const int64_t start = std::min<int64_t>(N, int64_t(rank) * per);
    *n0 = start;
    *n_slab = std::min<int64_t>(per, N - start);
    return RIDGE_OK;
}

int ridge_slabs_to_rowmajor(const void* slabs, void* C, int64_t M, int64_t N, int32_t nranks,
                            int64_t slab_cols, int64_t ldc, void* stream) {
    if (M < 0 || N < 0 || nranks <= 0 || slab_cols < 0 || ldc < N) return RIDGE_EINVAL;
    if (int64_t(nranks) * slab_cols < N) return RIDGE_EINVAL;
    if (M == 0 || N == 0) return RIDGE_OK;
    if (!slabs || !C) return RIDGE_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = slab_cols % 8 == 0 && ldc % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(slabs) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(C) & 15) == 0;
    const int block = 256;
    const int grid = 148 * 8;
    if (vec)
        slabs_to_rowmajor_vec<<<grid, block, 0, s>>>(static_cast<const uint4*>(slabs),
                                                     static_cast<uint4*>(C), M, N, nranks,
                                                     slab_cols, ldc);
    else
        slabs_to_rowmajor_scalar<<<grid, block, 0, s>>>(static_cast<const uint16_t*>(slabs),
                                                        static_cast<uint16_t*>(C), M, N, nranks,
                                                        slab_cols, ldc);
    return int(cudaGetLastError());
}

int ridge_gemm_sharded(const ridge_tile_config* cfg, const void* A, const void* B_slab,
                       void* C_slab, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                       int32_t nranks, int32_t rank, int32_t gather_full_c, void* nccl_comm,
                       void* slabs, void* C_full, int64_t ldc_full, void* stream) {
    constexpr int64_t kAlign = 256;
    if (!cfg || M < 0 || N < 0 || K < 0) return RIDGE_EINVAL;
    int64_t n0 = 0, ns = 0, per = 0, unused = 0;
    int st = ridge_slab_bounds(N, nranks, rank, kAlign, &n0, &ns);
    if (st != RIDGE_OK) return st;
    st = ridge_slab_bounds(N, nranks, 0, kAlign, &unused, &per);
    if (st != RIDGE_OK) return st;
    if (gather_full_c && (!C_full || ldc_full < N || (nranks > 1 && (!nccl_comm || !slabs))))
        return RIDGE_EINVAL;
    if (M > 0 && ns > 0) {
        st = ridge_gemm_launch(cfg, A, B_slab, C_slab, M, ns, K, lda, ldb, per, stream);
        if (st != RIDGE_OK) return st;
    }
    if (!gather_full_c || M == 0 || N == 0) return RIDGE_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (nranks == 1) {
        // nothing to exchange: the one slab is C
        cudaError_t e = cudaMemcpy2DAsync(C_full, size_t(ldc_full) * 2, C_slab, size_t(per) * 2,
                                          size_t(N) * 2, size_t(M), cudaMemcpyDeviceToDevice, s);
        return int(e);
    }
    AllGatherFn ag = nccl_allgather();
    if (!ag) return RIDGE_ECOMM;
    if (ag(C_slab, slabs, size_t(M * per), ncclHalf, static_cast<ncclComm_t>(nccl_comm), s) !=
        ncclSuccess)
        return RIDGE_ECOMM;
    return ridge_slabs_to_rowmajor(slabs, C_full, M, N, nranks, per, ldc_full, stream);
}

int ridge_gemm_sharded_p2p(const ridge_tile_config* cfg, const void* A, const void* B_slab,
                           int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                           int32_t nranks, int32_t rank, void* const* c_full, int64_t ldc,
                           void* nccl_comm, void* stream) {
    constexpr int64_t kAlign = 256;
    if (!cfg || !c_full || M < 0 || N < 0 || K < 0 || nranks < 1 || nranks > 8 || ldc < N)
        return RIDGE_EINVAL;
    int64_t n0 = 0, ns = 0;
    int st = ridge_slab_bounds(N, nranks, rank, kAlign, &n0, &ns);
    if (st != RIDGE_OK) return st;
    const bool fenced = nccl_comm && nranks > 1;
    AllReduceFn ar = nullptr;
    int* word = nullptr;
    if (fenced) {
        // Entry barrier: this rank's tiles go into every peer's C, so no rank
        // may start before all ranks are done with what their streams held
        // before this call (reading the previous result, typically).
        ar = nccl_allreduce();
        word = barrier_word();
        if (!ar || !word) return RIDGE_ECOMM;
        if (ar(word, word, 1, ncclInt32, ncclSum, static_cast<ncclComm_t>(nccl_comm),
               static_cast<cudaStream_t>(stream)) != ncclSuccess)
            return RIDGE_ECOMM;
    }
    if (M > 0 && ns > 0) {
        // this rank's slab of every rank's C: the same tile coordinates,
        // offset by n0 columns in each buffer
        void* peers[8];
        int np = 0;
        for (int r = 0; r < nranks; ++r) {
            if (!c_full[r]) return RIDGE_EINVAL;
            if (r != rank) peers[np++] = static_cast<__half*>(c_full[r]) + n0;
        }
        st = ridge_gemm_launch_multi(cfg, A, B_slab, static_cast<__half*>(c_full[rank]) + n0, M,
                                     ns, K, lda, ldb, ldc, peers, np, stream);
        if (st != RIDGE_OK) return st;
    }
    if (!fenced) return RIDGE_OK;
    // Completion barrier: every rank's tiles have landed in this rank's C.
    if (ar(word, word, 1, ncclInt32, ncclSum, static_cast<ncclComm_t>(nccl_comm),
           static_cast<cudaStream_t>(stream)) != ncclSuccess)
        return RIDGE_ECOMM;
    return RIDGE_OK;
}

int64_t ridge_ipc_handle_bytes(void) { return int64_t(sizeof(cudaIpcMemHandle_t)); }

int ridge_device_alloc(int64_t bytes, void** ptr) {
    if (bytes <= 0 || !ptr) return RIDGE_EINVAL;
    return int(cudaMalloc(ptr, size_t(bytes)));
}

int ridge_device_free(void* ptr) { return int(cudaFree(ptr)); }

int ridge_ipc_export(const void* base, void* handle) {
    if (!base || !handle) return RIDGE_EINVAL;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
    if (e != cudaSuccess) return int(e);
    std::memcpy(handle, &h, sizeof(h));
    return RIDGE_OK;
}

int ridge_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return RIDGE_EINVAL;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return int(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int ridge_ipc_close(void* ptr) { return int(cudaIpcCloseMemHandle(ptr)); }

}  // extern "C"
