// Instantiates the 2-CTA (cta_group::2) BM=256 members of the GEMM family (every BN, BK and
// epilogue-warp count); stages and groupM are runtime parameters.
#include "gemm_launch.cuh"

namespace ridge_b200 {

#define RIDGE_1CTA(BN, BK, W) out.push_back(make_entry<256, BN, BK, W, 2>())

void register_bm256_pair(std::vector<KernelEntry>& out) {
    RIDGE_1CTA(64, 32, 4);
    RIDGE_1CTA(64, 32, 8);
    RIDGE_1CTA(64, 64, 4);
    RIDGE_1CTA(64, 64, 8);
    RIDGE_1CTA(128, 32, 4);
    RIDGE_1CTA(128, 32, 8);
    RIDGE_1CTA(128, 64, 4);
    RIDGE_1CTA(128, 64, 8);
    RIDGE_1CTA(256, 32, 4);
    RIDGE_1CTA(256, 32, 8);
    RIDGE_1CTA(256, 64, 4);
    RIDGE_1CTA(256, 64, 8);
    RIDGE_1CTA(64, 128, 4);
    RIDGE_1CTA(64, 128, 8);
    RIDGE_1CTA(128, 128, 4);
    RIDGE_1CTA(128, 128, 8);
    RIDGE_1CTA(256, 128, 4);
    RIDGE_1CTA(256, 128, 8);
}

#undef RIDGE_1CTA

}  // namespace ridge_b200
