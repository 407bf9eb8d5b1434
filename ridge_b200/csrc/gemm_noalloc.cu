// A GEMM entry point that allocates no device memory.
//
// Some callers cannot allocate device memory on their own: code that runs
// inside a memory-pool arena handed to it by a host framework, a plugin whose
// host has banned cudaMalloc on the hot path (allocation synchronises the
// device and fragments a pre-planned pool), or a process that has already
// given every free byte to someone else. ridge_gemm_launch allocates its
// split-K workspace on first use, and ridge_gemm_launch_ws needs the caller to
// provide one. ridge_gemm_launch_noalloc instead uses one fixed scratch array
// that lives in this library's own device image: every GPU that loads the
// library holds it (kNoAllocScratchBytes) until the process exits, and no
// call ever allocates or frees memory.
//
// The caller still passes A, B and C. The array's host-side name is not a
// device address, so the host code below looks its device address up with
// cudaGetSymbolAddress, once per device, and hands that pointer to the kernel.

#include <cuda_runtime.h>

#include <mutex>

#include "../../include/ridge_b200.h"

namespace {

constexpr int64_t kNoAllocScratchBytes = 16ll << 20;  // 16 MiB per device
constexpr int64_t kCounterAreaBytes = 64 * 1024;      // head of any ridge workspace
constexpr int kMaxDevices = 64;

// The scratch: split-K counters (first 64 KB, must be zero between calls) and
// FP32 partial tiles. Static device storage starts zeroed at module load.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
    std::once_flag once;
    cudaError_t err = cudaSuccess;
    void* ptr = nullptr;
};
ScratchSlot g_slot[kMaxDevices];

// Set-up, once per device, with that device current: resolve the device
// address of the scratch array and clear its counter area.
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return int(e);
    if (dev < 0 || dev >= kMaxDevices) return RIDGE_ENOTSUP;
    ScratchSlot& s = g_slot[dev];
    std::call_once(s.once, [&] {
        void* p = nullptr;
        s.err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (s.err != cudaSuccess) return;
        s.err = cudaMemset(p, 0, size_t(kCounterAreaBytes));
        if (s.err != cudaSuccess) return;
        s.ptr = p;
    });
    if (s.err != cudaSuccess) return int(s.err);
    *out = s.ptr;
    return RIDGE_OK;
}

}  // namespace

namespace ridge_b200 {

// Sets every byte of the scratch's split-K counter area on the current device
// to `byte`, if that device's scratch was set up. ridge_device_error(clear)
// calls it with 0 after a kernel gave up mid-launch (its counters may be left
// non-zero, and the next split launch would then never find its last
// arrival); the self-test plants non-zero counters with it.
int noalloc_fill_counters(int byte) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return int(e);
    if (dev < 0 || dev >= kMaxDevices || !g_slot[dev].ptr) return RIDGE_OK;
    return int(cudaMemset(g_slot[dev].ptr, byte, size_t(kCounterAreaBytes)));
}

}  // namespace ridge_b200

extern "C" {

int64_t ridge_gemm_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int ridge_gemm_launch_noalloc(const ridge_tile_config* cfg, const void* A, const void* B,
                              void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                              int64_t ldc, void* stream) {
    int st = ridge_config_valid_for_shape(cfg, M, N, K, lda, ldb, ldc);
    if (st != RIDGE_OK) return st;
    int64_t need = 0;
    st = ridge_gemm_workspace_size(cfg, M, N, K, &need);
    if (st != RIDGE_OK) return st;
    if (need > kNoAllocScratchBytes) return RIDGE_ENOSCRATCH;
    void* scratch = nullptr;
    st = scratch_for_current_device(&scratch);
    if (st != RIDGE_OK) return st;
    return ridge_gemm_launch_ws(cfg, A, B, C, M, N, K, lda, ldb, ldc, scratch,
                                kNoAllocScratchBytes, stream);
}

}  // extern "C"
