// ref_shim.cu -- exposes the reference's own code as a C ABI for parity checks.
//
// TEST INFRASTRUCTURE ONLY (the checker, never the product). Compiled by
// oracle/Makefile straight from the reference sources where they lie, into
// oracle/_ref/libridge_ref.so; nothing of the reference is copied into this
// repository. The reference's check-gemm.cu is included with its main()
// renamed so that its file-local helpers become callable:
//   referenceGemm      bench/check-gemm.cu:98-108   FP64 host GEMM (the CPU baseline)
//   errorStats         bench/check-gemm.cu:121-135
//   fillDeterministic  bench/check-gemm.cu:139-145
// and the reference's sm_80 GPU kernel table (bench/kernels/gemm-mma.cu), which
// compiles unchanged for sm_100a and serves as a legacy-kernel parity point.
// The A100 cost model (src/model.cpp, src/hardware.cpp, src/mma.cpp) is linked
// in as well, behind ref_predict_a100.
#define main ridge_reference_check_gemm_main
#include "check-gemm.cu"
#undef main

#include "ridge/hardware.h"
#include "ridge/model.h"

#include <cstring>
#include <thread>

extern "C" {

void ref_fill(uint16_t* out, size_t n, unsigned seed) {
    std::vector<half> v(n);
    fillDeterministic(v, seed);
    std::memcpy(out, v.data(), n * sizeof(half));
}

// C (M x N, FP64) = A (M x K, row-major) * B (K x N, row-major), the reference's
// own loop, split by rows over `threads` host threads (each thread calls
// referenceGemm on its row block; the per-element arithmetic is unchanged).
void ref_gemm_f64(const uint16_t* A, const uint16_t* B, double* C, int M, int N, int K,
                  int threads) {
    std::vector<half> hb(size_t(K) * N);
    std::memcpy(hb.data(), B, hb.size() * sizeof(half));
    if (threads < 1) threads = 1;
    if (threads > M) threads = M > 0 ? M : 1;
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        const int r0 = int((long long)M * t / threads), r1 = int((long long)M * (t + 1) / threads);
        pool.emplace_back([&, r0, r1] {
            const int rows = r1 - r0;
            if (rows <= 0) return;
            std::vector<half> ha(size_t(rows) * K);
            std::memcpy(ha.data(), A + size_t(r0) * K, ha.size() * sizeof(half));
            std::vector<double> hc(size_t(rows) * N);
            referenceGemm(ha, hb, hc, rows, N, K);
            std::memcpy(C + size_t(r0) * N, hc.data(), hc.size() * sizeof(double));
        });
    }
    for (auto& th : pool) th.join();
}

void ref_error_stats(const float* got, const double* ref, size_t n, double* frob, double* max_rel) {
    std::vector<float> g(got, got + n);
    std::vector<double> r(ref, ref + n);
    const ErrStats e = errorStats(g, r);
    *frob = e.frob;
    *max_rel = e.maxRel;
}

int ref_num_variants() { return ridgebench::numVariants(); }

// out: BM, BN, BK, WM, WN, stages, groupM, smemBytes, threads, regsPerThread
void ref_variant_info(int i, int* out) {
    const ridgebench::KernelVariant& v = ridgebench::variant(i);
    const int vals[10] = {v.BM, v.BN, v.BK, v.WM, v.WN, v.stages, v.groupM, v.smemBytes, v.threads,
                          v.regsPerThread};
    std::memcpy(out, vals, sizeof(vals));
}

// The reference kernel: A (M x K) row-major, B (K x N) row-major, C FP32.
int ref_launch_variant(int i, const void* A, const void* B, float* C, int M, int N, int K,
                       void* stream) {
    return int(ridgebench::variant(i).launch(static_cast<const half*>(A),
                                             static_cast<const half*>(B), C, M, N, K,
                                             static_cast<cudaStream_t>(stream)));
}

// The reference A100 model on the built-in placeholders (calibrated=0) or a
// JSON file. cfg: M, N, K, BM, BN, BK, warpM, warpN, stages, regsPerThread.
// out: predictedTFLOPS, bottleneck, computeTFLOPS, hbmTFLOPS, peakTensorTFLOPS,
// smEfficiency, occFactor, arithmeticIntensity, baseIntensity, l2ReuseFactor,
// waveEfficiency, totalCtas, ctaSlots, wavesExact, envelopeEfficiency,
// tPrologueCycles, tEpilogueCycles, tBodyCycles, kSteps, numWarps, ctasPerSM,
// tComputeCycles, tSmemCycles, tStepCycles  (24 doubles)
int ref_predict_a100(const long long* cfg, const char* hw_json, double* out) {
    ridge::HardwareModel hw = ridge::HardwareModel::a100();
    if (hw_json && hw_json[0]) {
        std::string err;
        if (!ridge::HardwareModel::loadFromJson(hw_json, hw, err)) return -1;
    }
    ridge::GemmConfig c;
    c.M = cfg[0]; c.N = cfg[1]; c.K = cfg[2];
    c.BM = int(cfg[3]); c.BN = int(cfg[4]); c.BK = int(cfg[5]);
    c.warpM = int(cfg[6]); c.warpN = int(cfg[7]); c.stages = int(cfg[8]);
    c.regsPerThread = int(cfg[9]);
    const ridge::Prediction p = ridge::predict(c, hw);
    const double v[24] = {p.predictedTFLOPS, double(int(p.bottleneck)), p.computeTFLOPS,
                          p.hbmTFLOPS, p.peakTensorTFLOPS, p.smEfficiency, p.occFactor,
                          p.arithmeticIntensity, p.baseIntensity, p.l2ReuseFactor,
                          p.waveEfficiency, p.totalCtas, p.ctaSlots, p.wavesExact,
                          p.envelopeEfficiency, p.tPrologueCycles, p.tEpilogueCycles,
                          p.tBodyCycles, p.kSteps, double(p.numWarps), double(p.ctasPerSM),
                          p.tComputeCycles, p.tSmemCycles, p.tStepCycles};
    std::memcpy(out, v, sizeof(v));
    return 0;
}

}  // extern "C"
