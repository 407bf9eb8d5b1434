// ridge-predict: the B200 cost model from the command line.
//
// Same interface as the reference CLI (tools/ridge-predict.cpp:15-168): single
// prediction from flags, or --batch in.csv --out out.csv, which copies every
// row (and `#` comment line) and appends the prediction columns, matching input
// columns by name so a measured sweep can be fed straight in. Python tools get
// their predictions here or through ridge_predict in the library -- one copy of
// the math.
//
// Kept from the reference: --gpu / --hw / --m --n --k / --bm --bn --bk /
// --stages / --batch / --out and the eight pred_* columns. The sm_80 warp-tile
// flags (--warpm --warpn --regs) are accepted and ignored (tcgen05 has no warp
// tile). New: --warps --groupm --cta-group --split-k, and the input columns
// warps, groupM, cta_group, split_k (defaults when absent, so reference CSVs
// still parse).

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/ridge_b200.h"

namespace {

void usage() {
    std::printf(
        "ridge-predict: predict B200 FP16 tcgen05 GEMM throughput and bottleneck.\n"
        "Usage:\n"
        "  ridge-predict [--gpu b200 | --hw model.json]\n"
        "                [--m M --n N --k K]\n"
        "                [--bm BM --bn BN --bk BK --stages S --warps W --groupm G]\n"
        "                [--cta-group 0|1|2 --split-k 0|1]\n"
        "                [--batch in.csv --out out.csv]\n"
        "Defaults: built-in B200 placeholders, 4096^3, 128x256x64 tile, 4 stages,\n"
        "4 epilogue warps, groupM 8.\n");
}

std::vector<std::string> split_csv(const std::string& line) {
    std::vector<std::string> cells;
    std::string cell;
    std::istringstream ss(line);
    while (std::getline(ss, cell, ',')) cells.push_back(cell);
    return cells;
}

int run_batch(const std::string& in_path, const std::string& out_path, const ridge_hw& hw,
              const ridge_gemm_config& defaults) {
    std::ifstream in(in_path);
    if (!in) {
        std::fprintf(stderr, "cannot open %s\n", in_path.c_str());
        return 1;
    }
    std::ofstream out(out_path);
    if (!out) {
        std::fprintf(stderr, "cannot write %s\n", out_path.c_str());
        return 1;
    }
    std::string line;
    std::vector<std::string> header;
    bool have_header = false;
    int rows = 0;
    while (std::getline(in, line)) {
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (line.empty()) continue;
        if (line[0] == '#') {
            out << line << "\n";
            continue;
        }
        const std::vector<std::string> cells = split_csv(line);
        if (!have_header) {
            header = cells;
            have_header = true;
            out << line
                << ",pred_tflops,pred_bottleneck,pred_compute_ceiling,pred_hbm_ceiling,"
                   "pred_smem_eff,pred_occ_factor,pred_arith_intensity,pred_ctas_per_sm\n";
            continue;
        }
        auto col = [&](const char* name, long long def) -> long long {
            for (size_t i = 0; i < header.size() && i < cells.size(); ++i)
                if (header[i] == name) return std::atoll(cells[i].c_str());
            return def;
        };
        ridge_gemm_config g = defaults;
        g.M = col("M", g.M);
        g.N = col("N", g.N);
        g.K = col("K", g.K);
        g.tile.BM = int(col("BM", g.tile.BM));
        g.tile.BN = int(col("BN", g.tile.BN));
        g.tile.BK = int(col("BK", g.tile.BK));
        g.tile.stages = int(col("stages", g.tile.stages));
        g.tile.warps = int(col("warps", g.tile.warps));
        g.tile.groupM = int(col("groupM", g.tile.groupM));
        g.tile.cta_group = int(col("cta_group", g.tile.cta_group));
        g.tile.split_k = int(col("split_k", g.tile.split_k));
        ridge_prediction p;
        if (ridge_predict(&g, &hw, &p) != RIDGE_OK) {
            std::fprintf(stderr, "%s: row %d: invalid shape\n", in_path.c_str(), rows + 1);
            return 1;
        }
        out << line << ',' << p.predicted_tflops << ',' << ridge_bottleneck_string(p.bottleneck)
            << ',' << p.compute_tflops << ',' << p.hbm_tflops << ',' << p.smem_efficiency << ','
            << p.occ_factor << ',' << p.arithmetic_intensity << ',' << p.ctas_per_sm << '\n';
        ++rows;
    }
    std::fprintf(stderr, "predicted %d rows -> %s (%s constants)\n", rows, out_path.c_str(),
                 hw.calibrated ? "calibrated" : "placeholder");
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    ridge_gemm_config cfg;
    cfg.M = cfg.N = cfg.K = 4096;
    cfg.tile = ridge_tile_config{128, 256, 64, 4, 4, 8, 0, 0};
    std::string gpu = "b200", hw_path, batch_in, batch_out;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto next = [&](long long def) -> long long {
            return (i + 1 < argc) ? std::atoll(argv[++i]) : def;
        };
        auto next_s = [&](const std::string& def) -> std::string {
            return (i + 1 < argc) ? std::string(argv[++i]) : def;
        };
        if (a == "--gpu") gpu = next_s(gpu);
        else if (a == "--hw") hw_path = next_s(hw_path);
        else if (a == "--batch") batch_in = next_s(batch_in);
        else if (a == "--out") batch_out = next_s(batch_out);
        else if (a == "--m") cfg.M = next(cfg.M);
        else if (a == "--n") cfg.N = next(cfg.N);
        else if (a == "--k") cfg.K = next(cfg.K);
        else if (a == "--bm") cfg.tile.BM = int(next(cfg.tile.BM));
        else if (a == "--bn") cfg.tile.BN = int(next(cfg.tile.BN));
        else if (a == "--bk") cfg.tile.BK = int(next(cfg.tile.BK));
        else if (a == "--stages") cfg.tile.stages = int(next(cfg.tile.stages));
        else if (a == "--warps") cfg.tile.warps = int(next(cfg.tile.warps));
        else if (a == "--groupm") cfg.tile.groupM = int(next(cfg.tile.groupM));
        else if (a == "--cta-group") cfg.tile.cta_group = int(next(cfg.tile.cta_group));
        else if (a == "--split-k") cfg.tile.split_k = int(next(cfg.tile.split_k));
        else if (a == "--warpm" || a == "--warpn" || a == "--regs") next(0);  // sm_80 only
        else if (a == "-h" || a == "--help") {
            usage();
            return 0;
        } else {
            std::fprintf(stderr, "unknown arg: %s\n", a.c_str());
            usage();
            return 1;
        }
    }
    ridge_hw hw;
    if (!hw_path.empty()) {
        char err[512];
        if (ridge_hw_load_json(hw_path.c_str(), &hw, err, sizeof(err)) != RIDGE_OK) {
            std::fprintf(stderr, "%s\n", err);
            return 1;
        }
    } else if (gpu == "b200") {
        ridge_hw_b200(&hw);
    } else {
        std::fprintf(stderr, "unknown gpu: %s\n", gpu.c_str());
        return 1;
    }
    if (!batch_in.empty())
        return run_batch(batch_in, batch_out.empty() ? "predictions.csv" : batch_out, hw, cfg);

    ridge_prediction p;
    if (ridge_predict(&cfg, &hw, &p) != RIDGE_OK) {
        std::fprintf(stderr, "invalid shape\n");
        return 1;
    }
    std::printf("GPU: %s\n", hw.name);
    std::printf("  constants: %s\n", hw.calibrated ? "calibrated on a B200"
                                                    : "datasheet placeholders, indicative only");
    std::printf("GEMM %lldx%lldx%lld  tile %dx%dx%d  stages %d  warps %d  groupM %d  cta_group %d\n",
                (long long)cfg.M, (long long)cfg.N, (long long)cfg.K, cfg.tile.BM, cfg.tile.BN,
                cfg.tile.BK, cfg.tile.stages, cfg.tile.warps, cfg.tile.groupM, cfg.tile.cta_group);
    if (p.bottleneck == RIDGE_BOTTLENECK_DOES_NOT_FIT) {
        std::printf("  does not fit: shared memory or Tensor Memory exceed the SM\n");
        return 0;
    }
    std::printf("  predicted:    %8.1f TFLOP/s   bottleneck: %s\n", p.predicted_tflops,
                ridge_bottleneck_string(p.bottleneck));
    std::printf("  peak tensor:  %8.1f   compute ceiling: %8.1f   HBM ceiling: %8.1f\n",
                p.peak_tensor_tflops, p.compute_tflops, p.hbm_tflops);
    std::printf("  per stage: mma %.0f  smem-read %.0f  TMA fill %.0f  -> %.0f cycles (period %.0f)\n",
                p.t_mma_cycles, p.t_smem_cycles, p.t_l2_cycles, p.t_step_cycles,
                p.t_period_cycles);
    std::printf("  per tile: epilogue %.0f  tile %.0f cycles   %d accumulator(s)   CTAs/SM %d\n",
                p.t_epilogue_cycles, p.t_tile_cycles, p.acc_buffers, p.ctas_per_sm);
    std::printf("  grid: %.0f tiles in %.0f slots  waves %.2f  wave eff %.3f\n", p.total_tiles,
                p.tile_slots, p.waves_exact, p.wave_efficiency);
    std::printf("  effs: smem %.2f  fill %.2f  latency %.2f  epilogue %.2f  envelope %.3f\n",
                p.smem_efficiency, p.l2_efficiency, p.occ_factor, p.epilogue_efficiency,
                p.envelope_efficiency);
    std::printf("  DRAM %.1f MB  arithmetic intensity %.1f FLOP/byte\n", p.dram_bytes / 1e6,
                p.arithmetic_intensity);
    return 0;
}
