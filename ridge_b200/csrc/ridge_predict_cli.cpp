// ridge-predict: command-line front end of the B200 cost model (ridge_predict
// in libridge_b200).
//
// Drop-in contract with the reference tool (tools/ridge-predict.cpp there):
//   * the flags --gpu, --hw, --m/--n/--k, --bm/--bn/--bk, --stages, --batch,
//     --out; the sm_80 warp-tile flags --warpm/--warpn/--regs are accepted and
//     have no effect (tcgen05 tiles have no warp tile);
//   * --batch IN --out OUT joins by column name: every input line is copied
//     (comment lines starting with '#' too) and each data row gets the eight
//     pred_* columns, so a measured sweep can be fed in as it is.
// This build adds --warps, --groupm, --cta-group, --split-k (and the CSV
// columns warps, groupM, cta_group, split_k, defaulted when absent so older
// CSVs still load) and --json for a machine-readable single prediction.
//
// Structure: a table of option descriptors drives the parser (each names the
// field it sets), a ColumnMap resolves CSV header names to indices once, and
// the single-prediction report is rendered from a list of labelled values.

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ridge_b200.h"

namespace {

struct Options {
    ridge_gemm_config cfg{};
    std::string gpu = "b200";
    std::string hw_json;
    std::string batch_in;
    std::string batch_out = "predictions.csv";
    bool json = false;
    bool help = false;
};

enum class Kind { I64, I32, Text, Flag, Ignored };

struct OptionSpec {
    const char* flag;
    Kind kind;
    void* target;  // int64_t*, int32_t*, std::string* or bool*; unused for Ignored
};

std::vector<OptionSpec> option_table(Options& o) {
    return {
        {"--gpu", Kind::Text, &o.gpu},          {"--hw", Kind::Text, &o.hw_json},
        {"--batch", Kind::Text, &o.batch_in},   {"--out", Kind::Text, &o.batch_out},
        {"--m", Kind::I64, &o.cfg.M},           {"--n", Kind::I64, &o.cfg.N},
        {"--k", Kind::I64, &o.cfg.K},           {"--bm", Kind::I32, &o.cfg.tile.BM},
        {"--bn", Kind::I32, &o.cfg.tile.BN},    {"--bk", Kind::I32, &o.cfg.tile.BK},
        {"--stages", Kind::I32, &o.cfg.tile.stages},
        {"--warps", Kind::I32, &o.cfg.tile.warps},
        {"--groupm", Kind::I32, &o.cfg.tile.groupM},
        {"--cta-group", Kind::I32, &o.cfg.tile.cta_group},
        {"--split-k", Kind::I32, &o.cfg.tile.split_k},
        {"--json", Kind::Flag, &o.json},        {"--help", Kind::Flag, &o.help},
        {"-h", Kind::Flag, &o.help},            {"--warpm", Kind::Ignored, nullptr},
        {"--warpn", Kind::Ignored, nullptr},    {"--regs", Kind::Ignored, nullptr},
    };
}

const char* kHelp =
    "ridge-predict -- B200 (sm_100a) tcgen05 FP16 GEMM cost model\n"
    "\n"
    "  one prediction:  ridge-predict [--m M --n N --k K] [tile flags] [--json]\n"
    "  CSV join:        ridge-predict --batch sweep.csv [--out predictions.csv]\n"
    "\n"
    "  hardware   --gpu b200 (built-in constants) | --hw constants.json\n"
    "  tile       --bm --bn --bk --stages --warps --groupm --cta-group 0|1|2 --split-k 0|1\n"
    "             (--warpm/--warpn/--regs are accepted for old scripts and ignored)\n"
    "  defaults   M = N = K = 4096, 128x256x64 tile, 4 stages, 4 epilogue warps, groupM 8\n";

bool parse_int(const char* text, int64_t* out) {
    if (!text || !*text) return false;
    errno = 0;
    char* end = nullptr;
    const long long v = std::strtoll(text, &end, 10);
    if (errno != 0 || *end != '\0') return false;
    *out = v;
    return true;
}

// Accepts "--flag value" and "--flag=value". Returns false (message printed)
// on an unknown flag, a missing value or a value that is not an integer.
bool parse_args(int argc, char** argv, Options& o) {
    const std::vector<OptionSpec> table = option_table(o);
    for (int i = 1; i < argc; ++i) {
        std::string arg = argv[i];
        std::string inline_value;
        bool has_inline = false;
        const size_t eq = arg.find('=');
        if (arg.rfind("--", 0) == 0 && eq != std::string::npos) {
            inline_value = arg.substr(eq + 1);
            arg.resize(eq);
            has_inline = true;
        }
        const OptionSpec* spec = nullptr;
        for (const OptionSpec& s : table)
            if (arg == s.flag) spec = &s;
        if (!spec) {
            std::fprintf(stderr, "ridge-predict: no such option '%s' (try --help)\n", argv[i]);
            return false;
        }
        if (spec->kind == Kind::Flag) {
            *static_cast<bool*>(spec->target) = true;
            continue;
        }
        const char* value = nullptr;
        if (has_inline) {
            value = inline_value.c_str();
        } else if (i + 1 < argc) {
            value = argv[++i];
        } else {
            std::fprintf(stderr, "ridge-predict: option '%s' needs a value\n", spec->flag);
            return false;
        }
        int64_t n = 0;
        switch (spec->kind) {
            case Kind::Text: *static_cast<std::string*>(spec->target) = value; break;
            case Kind::Ignored: break;
            case Kind::I64:
            case Kind::I32:
                if (!parse_int(value, &n)) {
                    std::fprintf(stderr, "ridge-predict: '%s' wants an integer, got '%s'\n",
                                 spec->flag, value);
                    return false;
                }
                if (spec->kind == Kind::I64)
                    *static_cast<int64_t*>(spec->target) = n;
                else
                    *static_cast<int32_t*>(spec->target) = int32_t(n);
                break;
            case Kind::Flag: break;
        }
    }
    return true;
}

bool load_hardware(const Options& o, ridge_hw* hw) {
    if (!o.hw_json.empty()) {
        char err[512] = {0};
        if (ridge_hw_load_json(o.hw_json.c_str(), hw, err, int(sizeof(err))) != RIDGE_OK) {
            std::fprintf(stderr, "ridge-predict: hardware constants not loaded: %s\n", err);
            return false;
        }
        return true;
    }
    if (o.gpu == "b200" || o.gpu == "B200") return ridge_hw_b200(hw) == RIDGE_OK;
    std::fprintf(stderr, "ridge-predict: no built-in constants for '%s' (only b200; use --hw)\n",
                 o.gpu.c_str());
    return false;
}

// ---------------------------------------------------------------- CSV join

std::vector<std::string> split_fields(const std::string& line) {
    std::vector<std::string> f;
    size_t start = 0;
    for (;;) {
        const size_t comma = line.find(',', start);
        f.push_back(line.substr(start, comma == std::string::npos ? std::string::npos
                                                                  : comma - start));
        if (comma == std::string::npos) return f;
        start = comma + 1;
    }
}

// Header name -> column index, resolved once per file.
class ColumnMap {
  public:
    explicit ColumnMap(const std::vector<std::string>& header) {
        for (size_t i = 0; i < header.size(); ++i) index_.emplace(header[i], i);
    }
    // Stores the integer in column `name` of `row` into *field; a file without
    // that column leaves *field at its default. A malformed cell is an error.
    template <typename T>
    bool get(const std::vector<std::string>& row, const char* name, T* field) const {
        const auto it = index_.find(name);
        if (it == index_.end() || it->second >= row.size()) return true;  // keep the default
        int64_t v = 0;
        if (!parse_int(row[it->second].c_str(), &v)) return false;
        *field = T(v);
        return true;
    }

  private:
    std::unordered_map<std::string, size_t> index_;
};

constexpr const char* kPredColumns =
    "pred_tflops,pred_bottleneck,pred_compute_ceiling,pred_hbm_ceiling,pred_smem_eff,"
    "pred_occ_factor,pred_arith_intensity,pred_ctas_per_sm";

int join_csv(const Options& o, const ridge_hw& hw) {
    std::ifstream in(o.batch_in);
    if (!in) {
        std::fprintf(stderr, "ridge-predict: cannot read '%s'\n", o.batch_in.c_str());
        return 1;
    }
    std::FILE* out = std::fopen(o.batch_out.c_str(), "w");
    if (!out) {
        std::fprintf(stderr, "ridge-predict: cannot create '%s'\n", o.batch_out.c_str());
        return 1;
    }
    std::unique_ptr<ColumnMap> columns;
    std::string line;
    long line_no = 0, predicted = 0;
    int status = 0;
    while (status == 0 && std::getline(in, line)) {
        ++line_no;
        if (!line.empty() && line.back() == '\r') line.pop_back();
        if (line.empty()) continue;
        if (line[0] == '#') {  // comments travel with the data
            std::fprintf(out, "%s\n", line.c_str());
            continue;
        }
        const std::vector<std::string> fields = split_fields(line);
        if (!columns) {
            columns.reset(new ColumnMap(fields));
            std::fprintf(out, "%s,%s\n", line.c_str(), kPredColumns);
            continue;
        }
        ridge_gemm_config g = o.cfg;
        ridge_tile_config& t = g.tile;
        const bool ok = columns->get(fields, "M", &g.M) && columns->get(fields, "N", &g.N) &&
                        columns->get(fields, "K", &g.K) && columns->get(fields, "BM", &t.BM) &&
                        columns->get(fields, "BN", &t.BN) && columns->get(fields, "BK", &t.BK) &&
                        columns->get(fields, "stages", &t.stages) &&
                        columns->get(fields, "warps", &t.warps) &&
                        columns->get(fields, "groupM", &t.groupM) &&
                        columns->get(fields, "cta_group", &t.cta_group) &&
                        columns->get(fields, "split_k", &t.split_k);
        ridge_prediction p;
        if (!ok || ridge_predict(&g, &hw, &p) != RIDGE_OK) {
            std::fprintf(stderr, "ridge-predict: %s line %ld: %s\n", o.batch_in.c_str(), line_no,
                         ok ? "shape or tile the model refuses" : "non-integer value");
            status = 1;
            break;
        }
        std::fprintf(out, "%s,%.9g,%s,%.9g,%.9g,%.9g,%.9g,%.9g,%d\n", line.c_str(),
                     p.predicted_tflops, ridge_bottleneck_string(p.bottleneck), p.compute_tflops,
                     p.hbm_tflops, p.smem_efficiency, p.occ_factor, p.arithmetic_intensity,
                     p.ctas_per_sm);
        ++predicted;
    }
    std::fclose(out);
    if (status == 0)
        std::fprintf(stderr, "ridge-predict: %ld row(s) joined into %s [%s hardware constants]\n",
                     predicted, o.batch_out.c_str(), hw.calibrated ? "measured" : "built-in");
    return status;
}

// ---------------------------------------------------------------- one prediction

struct Item {
    const char* key;
    double value;
    const char* unit;
};

int report_one(const Options& o, const ridge_hw& hw) {
    const ridge_gemm_config& g = o.cfg;
    ridge_prediction p;
    if (ridge_predict(&g, &hw, &p) != RIDGE_OK) {
        std::fprintf(stderr, "ridge-predict: the model refuses this shape or tile\n");
        return 1;
    }
    const bool fits = p.bottleneck != RIDGE_BOTTLENECK_DOES_NOT_FIT;
    const char* limiter = ridge_bottleneck_string(p.bottleneck);
    const std::vector<Item> items = {
        {"tflops", p.predicted_tflops, "TFLOP/s"},
        {"compute_ceiling", p.compute_tflops, "TFLOP/s"},
        {"hbm_ceiling", p.hbm_tflops, "TFLOP/s"},
        {"tensor_peak", p.peak_tensor_tflops, "TFLOP/s"},
        {"seconds", p.predicted_seconds, "s"},
        {"mma_cycles_per_stage", p.t_mma_cycles, "cycles"},
        {"smem_cycles_per_stage", p.t_smem_cycles, "cycles"},
        {"fill_cycles_per_stage", p.t_l2_cycles, "cycles"},
        {"stage_cycles", p.t_step_cycles, "cycles"},
        {"ring_period_cycles", p.t_period_cycles, "cycles"},
        {"epilogue_cycles_per_tile", p.t_epilogue_cycles, "cycles"},
        {"tile_cycles", p.t_tile_cycles, "cycles"},
        {"tiles", p.total_tiles, ""},
        {"tile_slots", p.tile_slots, ""},
        {"waves", p.waves_exact, ""},
        {"wave_efficiency", p.wave_efficiency, ""},
        {"smem_efficiency", p.smem_efficiency, ""},
        {"fill_efficiency", p.l2_efficiency, ""},
        {"latency_factor", p.occ_factor, ""},
        {"epilogue_efficiency", p.epilogue_efficiency, ""},
        {"envelope_efficiency", p.envelope_efficiency, ""},
        {"dram_mbytes", p.dram_bytes / 1e6, "MB"},
        {"flop_per_byte", p.arithmetic_intensity, ""},
        {"ctas_per_sm", double(p.ctas_per_sm), ""},
        {"accumulators", double(p.acc_buffers), ""},
    };
    if (o.json) {
        std::printf("{\"gpu\": \"%s\", \"calibrated\": %s, \"M\": %lld, \"N\": %lld, \"K\": %lld, "
                    "\"tile\": [%d, %d, %d, %d, %d, %d, %d, %d], \"fits\": %s, "
                    "\"bottleneck\": \"%s\"",
                    hw.name, hw.calibrated ? "true" : "false", (long long)g.M, (long long)g.N,
                    (long long)g.K, g.tile.BM, g.tile.BN, g.tile.BK, g.tile.stages, g.tile.warps,
                    g.tile.groupM, g.tile.cta_group, g.tile.split_k, fits ? "true" : "false",
                    limiter);
        for (const Item& it : items) std::printf(", \"%s\": %.9g", it.key, it.value);
        std::printf("}\n");
        return 0;
    }
    std::printf("%lld x %lld x %lld on %s (%s constants)\n", (long long)g.M, (long long)g.N,
                (long long)g.K, hw.name, hw.calibrated ? "measured" : "built-in, unmeasured");
    std::printf("tile BM=%d BN=%d BK=%d stages=%d warps=%d groupM=%d cta_group=%d split_k=%d\n",
                g.tile.BM, g.tile.BN, g.tile.BK, g.tile.stages, g.tile.warps, g.tile.groupM,
                g.tile.cta_group, g.tile.split_k);
    if (!fits) {
        std::printf("=> this tile does not fit on one SM (shared memory or Tensor Memory)\n");
        return 0;
    }
    std::printf("=> %.1f TFLOP/s, limited by %s\n", p.predicted_tflops, limiter);
    for (size_t i = 1; i < items.size(); ++i)
        std::printf("   %-26s %14.4f %s\n", items[i].key, items[i].value, items[i].unit);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    Options o;
    o.cfg.M = o.cfg.N = o.cfg.K = 4096;
    o.cfg.tile = ridge_tile_config{128, 256, 64, 4, 4, 8, 0, 0};
    if (!parse_args(argc, argv, o)) return 2;
    if (o.help) {
        std::fputs(kHelp, stdout);
        return 0;
    }
    ridge_hw hw;
    if (!load_hardware(o, &hw)) return 1;
    return o.batch_in.empty() ? report_one(o, hw) : join_csv(o, hw);
}
