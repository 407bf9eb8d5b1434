// End-to-end GEMM on host buffers, with the PCIe copies pipelined against the
// kernel.
//
// A caller holding A, B and C in host memory would otherwise copy A and B in,
// launch, and copy C out, one after the other: at 4096^3 the copies take ~18x
// the kernel. ridge_gemm_host splits the M dimension into panels and runs
// three streams: host->device copies (B, then A panel by panel), the kernel
// (the caller's stream, one launch per panel as soon as its A panel has
// landed) and device->host copies of each finished C panel, which overlap the
// next panels' inbound copies (PCIe is full duplex). The step then costs about
// the inbound bytes over the link plus one panel's kernel and outbound copy.
//
// Device staging buffers, the two copy streams and the events are kept per
// device and grown on demand (growing frees the old buffers, which waits for
// the device). Calls on one device are ordered on the GPU: a call's first copy
// waits for the previous call's last one, so the shared buffers are never
// overwritten while in use. Page-locked host buffers give the overlap; with
// pageable ones the driver stages the copies and they serialise.

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/ridge_b200.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxPanels = 64;

struct HostPipe {
    std::mutex mu;
    bool init = false;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_start = nullptr, ev_b = nullptr, ev_done = nullptr;
    cudaEvent_t ev_a[kMaxPanels] = {}, ev_c[kMaxPanels] = {};
    bool have_done = false;
    void* a = nullptr;
    void* b = nullptr;
    void* c = nullptr;
    size_t a_bytes = 0, b_bytes = 0, c_bytes = 0;
};
HostPipe g_pipe[kMaxDevices];

int init_pipe(HostPipe& p) {
    if (p.init) return RIDGE_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&p.s_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p.s_out, cudaStreamNonBlocking);
    const unsigned fl = cudaEventDisableTiming;
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_start, fl);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_b, fl);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_done, fl);
    for (int i = 0; i < kMaxPanels && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&p.ev_a[i], fl);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.ev_c[i], fl);
    }
    if (e != cudaSuccess) return int(e);
    p.init = true;
    return RIDGE_OK;
}

int grow(void*& ptr, size_t& have, size_t need) {
    if (need <= have) return RIDGE_OK;
    if (ptr) {
        cudaError_t e = cudaFree(ptr);  // implies a device-wide wait
        ptr = nullptr;
        have = 0;
        if (e != cudaSuccess) return int(e);
    }
    cudaError_t e = cudaMalloc(&ptr, need);
    if (e != cudaSuccess) {
        ptr = nullptr;
        return int(e);
    }
    have = need;
    return RIDGE_OK;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

}  // namespace

extern "C" {

int ridge_gemm_host(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                    int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                    int32_t panels, void* stream) {
    if (!cfg || M < 0 || N < 0 || K < 0 || panels < 0 || panels > kMaxPanels)
        return RIDGE_EINVAL;
    if (M == 0 || N == 0) return RIDGE_OK;
    if (!C || (K > 0 && (!A || !B)) || lda < K || ldb < K || ldc < N) return RIDGE_EINVAL;
    ridge_variant_info info;
    int st = ridge_config_check(cfg, &info);
    if (st != RIDGE_OK) return st;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return int(e);
    if (dev < 0 || dev >= kMaxDevices) return RIDGE_ENOTSUP;
    HostPipe& p = g_pipe[dev];
    std::lock_guard<std::mutex> lock(p.mu);
    if ((st = init_pipe(p)) != RIDGE_OK) return st;

    // Device copies keep 16-byte row pitches (TMA): K and N rounded up to 8.
    const int64_t dlda = std::max<int64_t>(8, round_up(K, 8));
    const int64_t dldc = round_up(N, 8);
    const size_t es = 2;  // FP16
    if ((st = grow(p.a, p.a_bytes, size_t(M * dlda) * es)) != RIDGE_OK) return st;
    if ((st = grow(p.b, p.b_bytes, size_t(N * dlda) * es)) != RIDGE_OK) return st;
    if ((st = grow(p.c, p.c_bytes, size_t(M * dldc) * es)) != RIDGE_OK) return st;

    // Panels: whole multiples of the tile height; by default about 4 of them.
    // Measured at 4096^3 (pinned buffers): 1 panel 1.92 ms, 2: 1.65, 4: 1.56,
    // 8: 1.64, 16: 1.70; the copies out slow the copies in by ~30% while they
    // overlap, so more, smaller panels stop paying beyond 4. The floor is the
    // 64 MiB inbound at ~53 GB/s, 1.22 ms.
    const int64_t want = panels > 0 ? panels : 4;
    const int64_t rows = std::max<int64_t>(cfg->BM, round_up((M + want - 1) / want, cfg->BM));
    const int64_t np = (M + rows - 1) / rows;
    if (np > kMaxPanels) return RIDGE_EINVAL;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Inputs are ready in the caller's stream order; the staging buffers are
    // free once the previous call on this device has copied its C out.
    e = cudaEventRecord(p.ev_start, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.s_in, p.ev_start, 0);
    if (e == cudaSuccess && p.have_done) e = cudaStreamWaitEvent(p.s_in, p.ev_done, 0);
    if (e != cudaSuccess) return int(e);

    if (K > 0) {
        e = cudaMemcpy2DAsync(p.b, size_t(dlda) * es, B, size_t(ldb) * es, size_t(K) * es,
                              size_t(N), cudaMemcpyHostToDevice, p.s_in);
        if (e == cudaSuccess) e = cudaEventRecord(p.ev_b, p.s_in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, p.ev_b, 0);
        if (e != cudaSuccess) return int(e);
    }
    for (int64_t i = 0; i < np; ++i) {
        const int64_t m0 = i * rows, mp = std::min(rows, M - m0);
        unsigned char* ad = static_cast<unsigned char*>(p.a) + size_t(m0 * dlda) * es;
        unsigned char* cd = static_cast<unsigned char*>(p.c) + size_t(m0 * dldc) * es;
        if (K > 0) {
            e = cudaMemcpy2DAsync(ad, size_t(dlda) * es,
                                  static_cast<const unsigned char*>(A) + size_t(m0 * lda) * es,
                                  size_t(lda) * es, size_t(K) * es, size_t(mp),
                                  cudaMemcpyHostToDevice, p.s_in);
            if (e == cudaSuccess) e = cudaEventRecord(p.ev_a[i], p.s_in);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(s, p.ev_a[i], 0);
            if (e != cudaSuccess) return int(e);
        }
        st = ridge_gemm_launch(cfg, ad, p.b, cd, mp, N, K, dlda, dlda, dldc, s);
        if (st != RIDGE_OK) return st;
        e = cudaEventRecord(p.ev_c[i], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p.s_out, p.ev_c[i], 0);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(static_cast<unsigned char*>(C) + size_t(m0 * ldc) * es,
                                  size_t(ldc) * es, cd, size_t(dldc) * es, size_t(N) * es,
                                  size_t(mp), cudaMemcpyDeviceToHost, p.s_out);
        if (e != cudaSuccess) return int(e);
    }
    e = cudaEventRecord(p.ev_done, p.s_out);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, p.ev_done, 0);
    if (e != cudaSuccess) return int(e);
    p.have_done = true;
    return RIDGE_OK;
}

}  // extern "C"
