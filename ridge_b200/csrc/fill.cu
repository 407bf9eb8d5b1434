// Deterministic synthetic GEMM inputs generated on the device.
//
// The reference fills its operands on the host with a 32-bit LCG,
// s <- s * 1664525 + 1013904223, value = ((s >> 16) & 0x7fff) / 32767 - 0.5,
// rounded to FP16 (bench/check-gemm.cu:139-145). This kernel produces the same
// sequence bit for bit, in parallel: element i needs the state after i + 1
// steps, which is an affine map s -> a_n * s + c_n that the host composes by
// repeated squaring, so each thread jumps straight to the start of its chunk.
// range 0 keeps the reference's U(-0.5, 0.5); range 1 maps the same draw to
// U(-1, 1) (value = 2 * draw - 1), the benchmark inputs.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/ridge_b200.h"

namespace ridge_b200 {
namespace {

constexpr uint32_t kLcgA = 1664525u;
constexpr uint32_t kLcgC = 1013904223u;
constexpr int kChunk = 16;  // consecutive elements per thread

struct Affine {
    uint32_t a, c;  // s -> a * s + c (mod 2^32)
};

__host__ __device__ inline Affine compose(Affine first, Affine then) {
    return Affine{then.a * first.a, then.a * first.c + then.c};
}

__host__ __device__ inline Affine power(uint64_t n) {
    Affine result{1u, 0u};
    Affine step{kLcgA, kLcgC};
    while (n) {
        if (n & 1) result = compose(result, step);
        step = compose(step, step);
        n >>= 1;
    }
    return result;
}

__global__ void lcg_fill_kernel(__half* out, int64_t n, uint32_t seed, int unit) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t first = t * kChunk;
    if (first >= n) return;
    const Affine jump = power(uint64_t(first));
    uint32_t s = jump.a * seed + jump.c;
#pragma unroll
    for (int e = 0; e < kChunk; ++e) {
        if (first + e >= n) break;
        s = s * kLcgA + kLcgC;
        float v = float((s >> 16) & 0x7fffu) / 32767.0f;
        v = unit ? 2.0f * v - 1.0f : v - 0.5f;
        out[first + e] = __float2half_rn(v);
    }
}

}  // namespace
}  // namespace ridge_b200

extern "C" int ridge_fill_lcg(void* out, int64_t n, uint32_t* state, int32_t range, void* stream) {
    using namespace ridge_b200;
    if (!state || n < 0 || (range != 0 && range != 1) || (n > 0 && !out)) return RIDGE_EINVAL;
    if (n == 0) return RIDGE_OK;
    const int64_t threads = (n + kChunk - 1) / kChunk;
    const int block = 256;
    const int64_t grid = (threads + block - 1) / block;
    if (grid > 0x7fffffff) return RIDGE_EINVAL;
    lcg_fill_kernel<<<unsigned(grid), block, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half*>(out), n, *state, range);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return int(e);
    const Affine adv = power(uint64_t(n));
    *state = adv.a * *state + adv.c;
    return RIDGE_OK;
}
