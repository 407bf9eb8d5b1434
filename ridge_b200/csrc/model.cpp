// The ridge cost model re-derived for the B200 GEMM family (ridge_predict).
//
// Reference: src/model.cpp:22-146 (A100, mma.sync kernel). That model times
// one K-step of one CTA as tensor issue PLUS ldmatrix time (in series, because
// mma.sync consumes registers ldmatrix just wrote), derates by occupancy, wave
// quantisation and a fill/drain envelope, and caps by an HBM roofline with an
// sqrt(ctaSlots) L2 reuse factor.
//
// On sm_100a the kernel is different in kind, so the terms are re-derived:
//   * tcgen05.mma reads both operands straight from shared memory; whether the
//     operand reads add to or overlap the MMA is a calibrated constant
//     (hw.smem_mma_overlap: 1 = max, 0 = sum), measured by the calibration
//     microbenchmark rather than assumed;
//   * latency is hidden by pipeline depth (stages), not by resident warps: the
//     per-K-block period is max(t_kblock, (L + t_kblock) / stages) for TMA
//     latency L -- the B200 analogue of the reference's occupancy factor;
//   * the TMA fill from L2 is its own ceiling (all 148 SMs load at once);
//   * the persistent kernel walks ceil(tiles / slots) tiles per CTA, with the
//     epilogue of tile i overlapping the mainloop of tile i+1 when two TMEM
//     accumulators fit, and exposed when only one does;
//   * the HBM ceiling uses DRAM traffic from a round-by-round walk of the
//     grouped-M tile order (groupM now matters to the prediction, which the
//     reference model could not express -- README.md:162 there), with panels
//     of the previous round kept in L2 when they fit;
//   * wave quantisation is counted over 148 SMs (74 pairs for 2-CTA tiles).

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "../../include/ridge_b200.h"

namespace {

struct Geometry {
    int cg;              // CTAs per tile
    int halves;          // MMAs per K-step along M in one CTA
    int rows_per_cta;    // A rows one CTA holds
    double mma_m_ratio;  // cycle multiplier of the UMMA shape
};

Geometry geometry(const ridge_tile_config& t, const ridge_hw& hw) {
    Geometry g;
    g.cg = t.cta_group == 2 ? 2 : 1;
    g.halves = (g.cg == 1 && t.BM == 256) ? 2 : 1;
    g.rows_per_cta = t.BM / g.cg;
    g.mma_m_ratio = (g.cg == 1 && t.BM == 64) ? hw.umma_m64_ratio : 1.0;
    return g;
}

// DRAM bytes for the grouped-M persistent walk: round r runs tiles
// [r*slots, (r+1)*slots). Within a round, concurrently running CTAs share
// every A row-panel and B column-panel through L2 (they sweep K together), so
// each panel is read from DRAM at most once per round; a panel also used in
// the previous round is still in L2 if that round's panels fit in the
// effective L2 capacity. C is written once.
double dram_bytes(int64_t M, int64_t N, int64_t K, int BM, int BN, int groupM, int64_t slots,
                  double l2_bytes) {
    const int64_t num_m = (M + BM - 1) / BM;
    const int64_t num_n = (N + BN - 1) / BN;
    const int64_t tiles = num_m * num_n;
    const double a_panel = double(std::min<int64_t>(BM, M)) * K * 2.0;
    const double b_panel = double(std::min<int64_t>(BN, N)) * K * 2.0;
    const double c_bytes = double(M) * N * 2.0;
    const double l2_eff = 0.75 * l2_bytes;
    // Whole problem fits: every operand byte is read once.
    if (double(M) * K * 2.0 + double(N) * K * 2.0 <= l2_eff)
        return double(M) * K * 2.0 + double(N) * K * 2.0 + c_bytes;
    std::vector<int64_t> last_a(num_m, -2), last_b(num_n, -2);
    double total = c_bytes;
    double prev_footprint = 0.0;
    const int64_t per_group = int64_t(groupM) * num_n;
    for (int64_t r = 0, t0 = 0; t0 < tiles; ++r, t0 += slots) {
        const int64_t t1 = std::min(tiles, t0 + slots);
        const bool prev_fits = prev_footprint <= l2_eff;
        double footprint = 0.0;
        for (int64_t t = t0; t < t1; ++t) {
            const int64_t group = t / per_group;
            const int64_t first_m = group * groupM;
            const int64_t rows = std::min<int64_t>(num_m - first_m, groupM);
            const int64_t in_group = t - group * per_group;
            const int64_t tm = first_m + in_group % rows;
            const int64_t tn = in_group / rows;
            if (last_a[tm] != r) {
                if (!(last_a[tm] == r - 1 && prev_fits)) total += a_panel;
                last_a[tm] = r;
                footprint += a_panel;
            }
            if (last_b[tn] != r) {
                if (!(last_b[tn] == r - 1 && prev_fits)) total += b_panel;
                last_b[tn] = r;
                footprint += b_panel;
            }
        }
        prev_footprint = footprint;
    }
    return total;
}

// Smooth maximum (p-norm) of two times that overlap: equals the larger when
// one dominates, and exceeds it when both are close -- two limits that each
// nearly bind do not overlap perfectly. It also keeps the losing limit in the
// prediction, so configs held to the same bound are still ordered.
double soft_max(double a, double b, double p = 4.0) {
    const double m = std::max(a, b);
    if (m <= 0.0) return 0.0;
    return m * std::pow(std::pow(a / m, p) + std::pow(b / m, p), 1.0 / p);
}

// The compute side and the DRAM side of a launch overlap more closely than two
// limits inside the SM pipeline do: their smooth maximum is taken sharper.
constexpr double kHbmOverlapP = 8.0;

}  // namespace

extern "C" {

const char* ridge_bottleneck_string(int32_t b) {
    switch (b) {
        case RIDGE_BOTTLENECK_TENSOR_CORE: return "TENSOR_CORE";
        case RIDGE_BOTTLENECK_SMEM: return "SMEM";
        case RIDGE_BOTTLENECK_HBM: return "HBM";
        case RIDGE_BOTTLENECK_OCCUPANCY: return "OCC";
        case RIDGE_BOTTLENECK_WAVES: return "WAVES";
        case RIDGE_BOTTLENECK_ENVELOPE: return "ENVELOPE";
        case RIDGE_BOTTLENECK_DOES_NOT_FIT: return "DOES_NOT_FIT";
        case RIDGE_BOTTLENECK_EPILOGUE: return "EPILOGUE";
        case RIDGE_BOTTLENECK_L2: return "L2";
    }
    return "UNKNOWN";
}

int ridge_predict(const ridge_gemm_config* cfg, const ridge_hw* hw, ridge_prediction* out) {
    if (!cfg || !hw || !out) return RIDGE_EINVAL;
    ridge_prediction p;
    std::memset(&p, 0, sizeof(p));
    const ridge_tile_config& t = cfg->tile;
    const int64_t M = cfg->M, N = cfg->N, K = cfg->K;
    if (M <= 0 || N <= 0 || K <= 0 || hw->num_sms <= 0 || hw->clock_hz <= 0) return RIDGE_EINVAL;

    ridge_variant_info info;
    if (ridge_config_check(&t, &info) != RIDGE_OK) {
        p.bottleneck = RIDGE_BOTTLENECK_DOES_NOT_FIT;
        *out = p;
        return RIDGE_OK;
    }
    ridge_tile_config tc = t;
    tc.cta_group = info.cfg.cta_group;
    const Geometry g = geometry(tc, *hw);

    // Residency: shared memory (plus the 1 KB the driver reserves per CTA),
    // TMEM columns and threads bound the CTAs per SM.
    const int by_smem = hw->smem_bytes_per_sm / (info.smem_bytes + 1024);
    const int by_tmem = hw->tmem_cols_per_sm / info.tmem_cols;
    const int by_threads = 2048 / info.threads;
    const int cps = std::min(std::min(by_smem, by_tmem), std::min(by_threads, hw->max_ctas_per_sm));
    if (cps < 1) {
        p.bottleneck = RIDGE_BOTTLENECK_DOES_NOT_FIT;
        *out = p;
        return RIDGE_OK;
    }
    p.ctas_per_sm = cps;
    p.acc_buffers = info.acc_buffers;

    // ---- one pipeline stage (BK of K) of one CTA, in SM cycles at the
    // clock the part holds under sustained tensor load.
    const double kb = std::ceil(double(K) / t.BK);
    const double mma_per_stage = double(g.halves) * (t.BK / 16);
    // One tcgen05.mma on this SM: N/256 of a 128x256x16 MMA, unless reading
    // its operands from shared memory takes longer (A: the 128 -- or 64 --
    // rows this SM multiplies; B: the BN columns it holds, half of them in a
    // 2-CTA pair, whose peer reads the other half).
    const double a_rows = t.BM == 64 ? 64.0 : 128.0;
    const double b_cols = double(t.BN) / g.cg;
    const double t_issue = hw->umma_cycles_128x256 * (double(t.BN) / 256.0) * g.mma_m_ratio;
    const double t_read = (a_rows + b_cols) * 16.0 * 2.0 / hw->smem_bytes_per_cycle;
    const double ov = std::min(1.0, std::max(0.0, hw->smem_mma_overlap));
    const double t_one = ov * std::max(t_issue, t_read) + (1.0 - ov) * (t_issue + t_read);
    const double t_mma = mma_per_stage * t_one;
    // TMA fill: a stage is one box of A and one of B, both issued by the one
    // producer thread, so a CTA fills a stage in two box times (tma_box_cycles
    // per box of BK=64, scaled for BK=32 and the two-atom BK=128 box; fitted on
    // GEMM timings); the stage's bytes also cannot arrive faster than this
    // SM's share of the aggregate L2 -> shared memory rate.
    const double box_ratio =
        t.BK == 128 ? hw->tma_box2_ratio : (t.BK == 32 ? hw->tma_box32_ratio : 1.0);
    const double stage_bytes = (double(g.rows_per_cta) + double(t.BN) / g.cg) * t.BK * 2.0;
    const double l2_bytes_per_cycle_sm = hw->l2_bytes_per_sec / hw->num_sms / hw->clock_hz;
    const double t_fill =
        soft_max(2.0 * hw->tma_box_cycles * box_ratio, stage_bytes / l2_bytes_per_cycle_sm);
    const double t_smem = mma_per_stage * t_read;

    // ---- residency and the persistent walk (with the launcher's split-K tail)
    const int64_t num_m = (M + t.BM - 1) / t.BM;
    const int64_t num_n = (N + t.BN - 1) / t.BN;
    const int64_t tiles = num_m * num_n;
    const int64_t units = std::max<int64_t>(1, int64_t(hw->num_sms / g.cg) * cps);
    const int64_t rem = tiles >= units ? tiles % units : tiles;
    int64_t splits = 1;
    if (t.split_k != 1 && rem > 0)
        splits = std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(units / rem, 8),
                                                        int64_t(kb) / 4));
    const int64_t dp_tiles = splits >= 2 ? tiles - rem : tiles;
    const int64_t grid_units = std::max(std::min(tiles, units), splits >= 2 ? rem * splits : 0);
    // CTAs actually sharing one SM (a small grid leaves SMs with fewer).
    const double resident =
        std::min(double(cps), std::max(1.0, double(grid_units) * g.cg / hw->num_sms));

    // Operand bytes from DRAM (grouped-M walk, L2 reuse) against all operand
    // bytes the TMA moves into shared memory: loads of panels no earlier round
    // left in L2 wait for DRAM, not for L2.
    const double a_b_reads =
        dram_bytes(M, N, K, t.BM, t.BN, t.groupM, std::min(tiles, units), hw->l2_bytes) -
        double(M) * N * 2.0;
    const double fill_total = double(tiles) * kb * double(t.BM + t.BN) * t.BK * 2.0;
    const double f_dram = std::min(1.0, std::max(0.0, a_b_reads / std::max(fill_total, 1.0)));
    const double t_lat = hw->tma_latency_cycles +
                         f_dram * std::max(0.0, hw->tma_latency_hbm_cycles - hw->tma_latency_cycles);

    // Shared on-SM resources (tensor core, shared memory) serve the resident
    // CTAs in turn; each CTA's fill and its load latency are its own.
    // The SM keeps about four boxes in flight in all (one CTA with four
    // issuing threads already reaches it), so resident CTAs share that
    // budget exactly like they share the tensor core.
    const double t_stage = soft_max(t_mma, t_fill) * resident / hw->pipeline_efficiency;
    // A ring slot refills only after its MMAs finish: the load then waits
    // behind the pair's current box (t_fill) and travels for the unloaded
    // latency, so `stages` slots must cover (latency + t_fill + t_stage).
    const double t_period = std::max(t_stage, (t_lat + t_fill + t_stage) / double(t.stages));
    const double t_main_whole = kb * t_period;

    const double c_bytes_tile = double(g.rows_per_cta) * t.BN * 2.0;
    const double epi_bpc = t.warps == 8 ? hw->epi_bytes_per_cycle_w8 : hw->epi_bytes_per_cycle_w4;
    const double t_epi = c_bytes_tile / epi_bpc;
    // Turning a tile over costs a fixed hand-off on top of the drain (the
    // accumulator's full/empty barrier round trip; across the two SMs of a
    // pair); measured on short-K calibration GEMMs.
    const double t_turn =
        (g.cg == 2 ? hw->pair_tile_overhead_cycles : hw->tile_overhead_cycles) * resident;
    auto tile_period = [&](double t_main) {
        return (info.acc_buffers >= 2 ? soft_max(t_main, t_epi) : t_main + t_epi) + t_turn;
    };
    const double dp_rounds = std::ceil(double(dp_tiles) / double(std::min(units, std::max<int64_t>(dp_tiles, 1))));
    const double dp_per_unit = dp_tiles > 0 ? std::ceil(double(dp_tiles) / double(std::min(tiles, units))) : 0.0;
    (void)dp_rounds;
    double t_unit = dp_per_unit * tile_period(t_main_whole);
    double t_sk = 0.0;
    // The launcher runs a unit's split range before its whole tiles when those
    // fill at most six rounds (the partial exchange then overlaps the next
    // tile), after them otherwise.
    const bool sk_first = splits >= 2 && double(dp_tiles) / double(units) <= 6.0;
    if (splits >= 2) {
        // One K range of 1/splits. All but the last split to arrive write their
        // FP32 partial (twice the bytes of an FP16 tile, at the drain rate); the
        // last reads those splits - 1 partials and drains the tile.
        const double partial_bytes = double(g.rows_per_cta) * t.BN * 4.0;
        const double fixup = partial_bytes / epi_bpc +
                             double(splits - 1) * partial_bytes / (2.0 * epi_bpc) + t_epi;
        t_sk = std::ceil(kb / double(splits)) * t_period;
        if (sk_first && dp_per_unit > 0)
            t_sk += std::max(0.0, fixup - tile_period(t_main_whole));  // hidden behind a tile
        else
            t_sk += fixup;
        t_unit += t_sk;
    }
    if ((splits < 2 || sk_first) && info.acc_buffers >= 2 && dp_per_unit > 0)
        t_unit += std::min(t_main_whole, t_epi);  // the last tile's epilogue drains alone
    const double t_prologue = t_lat;
    t_unit += t_prologue;
    const double compute_sec = t_unit / hw->clock_hz;

    // ---- HBM: operand reads (grouped-M walk, L2 reuse), C writes, split-K partials
    const double c_write = double(M) * N * 2.0;
    const double partial_traffic =
        splits >= 2 ? 2.0 * double(rem) * splits * g.cg * double(g.rows_per_cta) * t.BN * 4.0
                    : 0.0;
    const double hbm_sec = a_b_reads / hw->hbm_bytes_per_sec + c_write / hw->c_write_bytes_per_sec +
                           partial_traffic / hw->c_write_bytes_per_sec;

    const double flops = 2.0 * double(M) * double(N) * double(K);
    const double peak_flops_per_cycle_sm = 2.0 * 128.0 * 256.0 * 16.0 / hw->umma_cycles_128x256;
    p.peak_tensor_tflops = peak_flops_per_cycle_sm * hw->clock_hz * hw->num_sms / 1e12;
    // The launch overhead is paid once, outside the overlap of the two limits.
    p.compute_tflops = flops / (compute_sec + hw->launch_overhead_sec) / 1e12;
    p.hbm_tflops = flops / (hbm_sec + hw->launch_overhead_sec) / 1e12;
    p.predicted_seconds = soft_max(compute_sec, hbm_sec, kHbmOverlapP) + hw->launch_overhead_sec;
    p.predicted_tflops = flops / p.predicted_seconds / 1e12;
    p.dram_bytes = a_b_reads + c_write;
    p.arithmetic_intensity = flops / p.dram_bytes;

    p.k_blocks = kb;
    p.t_mma_cycles = t_mma;
    p.t_smem_cycles = t_smem;
    p.t_l2_cycles = t_fill;
    p.t_step_cycles = t_stage;
    p.t_period_cycles = t_period;
    p.t_epilogue_cycles = t_epi;
    p.t_tile_cycles = tile_period(t_main_whole);
    p.t_prologue_cycles = t_prologue;
    p.total_tiles = double(tiles);
    p.tile_slots = double(units);
    p.waves_exact = double(tiles) / double(units);

    // Efficiency factors (1 = not limiting); the worst one names the label.
    const double ideal_unit = double(tiles) * kb * (mma_per_stage * t_issue) / double(units);
    p.smem_efficiency = t_issue / t_one;
    p.l2_efficiency = std::min(1.0, t_mma * resident / t_stage);
    p.occ_factor = t_stage / t_period;
    p.wave_efficiency = double(tiles) * kb * t_period / (double(units) * (t_unit - t_prologue));
    p.wave_efficiency = std::min(1.0, p.wave_efficiency);
    p.epilogue_efficiency = t_main_whole / tile_period(t_main_whole);
    p.envelope_efficiency =
        std::min(1.0, (t_unit - t_prologue) / (t_unit + hw->launch_overhead_sec * hw->clock_hz));
    (void)ideal_unit;

    if (hbm_sec > compute_sec) {
        p.bottleneck = RIDGE_BOTTLENECK_HBM;
    } else {
        struct F {
            double v;
            int label;
        } f[] = {{p.wave_efficiency, RIDGE_BOTTLENECK_WAVES},
                 {p.envelope_efficiency, RIDGE_BOTTLENECK_ENVELOPE},
                 {p.epilogue_efficiency, RIDGE_BOTTLENECK_EPILOGUE},
                 {p.smem_efficiency, RIDGE_BOTTLENECK_SMEM},
                 {p.l2_efficiency, RIDGE_BOTTLENECK_L2},
                 {p.occ_factor, RIDGE_BOTTLENECK_OCCUPANCY}};
        double worst = 2.0;
        int label = RIDGE_BOTTLENECK_TENSOR_CORE;
        for (const F& x : f)
            if (x.v < worst) {
                worst = x.v;
                label = x.label;
            }
        p.bottleneck = worst >= 0.95 ? RIDGE_BOTTLENECK_TENSOR_CORE : label;
    }
    *out = p;
    return RIDGE_OK;
}

}  // extern "C"
