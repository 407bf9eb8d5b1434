// Hardware constants for the B200 cost model: the built-in datasheet
// placeholders and an all-or-nothing loader for the flat calibration JSON.
//
// Reference: src/hardware.cpp:19-34 (HardwareModel::a100) and :149-200
// (loadFromJson). Same contract -- a file either supplies every required
// constant and passes the sanity checks, or nothing is changed and the caller
// gets the reason -- with the B200 constant set.

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>

#include "../../include/ridge_b200.h"

namespace {

void set_err(char* buf, int32_t len, const std::string& msg) {
    if (buf && len > 0) std::snprintf(buf, size_t(len), "%s", msg.c_str());
}

// Reads one flat JSON object of string / number / boolean / null members into
// key -> raw text. Nested objects and arrays are rejected: the calibration
// format is flat by design.
bool parse_flat_json(const std::string& s, std::map<std::string, std::string>& kv,
                     std::string& err) {
    size_t i = 0;
    auto ws = [&] {
        while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
    };
    auto str = [&](std::string& out) -> bool {
        if (i >= s.size() || s[i] != '"') {
            err = "expected a string at offset " + std::to_string(i);
            return false;
        }
        ++i;
        out.clear();
        while (i < s.size() && s[i] != '"') {
            if (s[i] == '\\') {
                if (++i >= s.size()) break;
                const char e = s[i];
                out.push_back(e == 'n' ? '\n' : e == 't' ? '\t' : e);
                ++i;
                continue;
            }
            out.push_back(s[i++]);
        }
        if (i >= s.size()) {
            err = "unterminated string";
            return false;
        }
        ++i;
        return true;
    };
    ws();
    if (i >= s.size() || s[i] != '{') {
        err = "expected '{'";
        return false;
    }
    ++i;
    ws();
    if (i < s.size() && s[i] == '}') return true;
    for (;;) {
        ws();
        std::string key, val;
        if (!str(key)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') {
            err = "expected ':' after \"" + key + "\"";
            return false;
        }
        ++i;
        ws();
        if (i < s.size() && s[i] == '"') {
            if (!str(val)) return false;
        } else if (i < s.size() && (s[i] == '{' || s[i] == '[')) {
            err = "nested value for \"" + key + "\" (the format is flat)";
            return false;
        } else {
            const size_t b = i;
            while (i < s.size() && s[i] != ',' && s[i] != '}' &&
                   !std::isspace(static_cast<unsigned char>(s[i])))
                ++i;
            if (i == b) {
                err = "empty value for \"" + key + "\"";
                return false;
            }
            val = s.substr(b, i - b);
        }
        kv[key] = val;
        ws();
        if (i < s.size() && s[i] == ',') {
            ++i;
            continue;
        }
        if (i < s.size() && s[i] == '}') return true;
        err = "value of \"" + key + "\" is followed by neither a comma nor the closing brace "
              "(byte " + std::to_string(i) + ")";
        return false;
    }
}

bool number(const std::map<std::string, std::string>& kv, const char* key, double& out,
            std::string& err) {
    auto it = kv.find(key);
    if (it == kv.end()) {
        err = std::string("constant \"") + key + "\" is absent (every constant is required)";
        return false;
    }
    char* end = nullptr;
    const double v = std::strtod(it->second.c_str(), &end);
    if (end == it->second.c_str() || *end != '\0' || !std::isfinite(v)) {
        err = std::string("key \"") + key + "\" is not a finite number: " + it->second;
        return false;
    }
    out = v;
    return true;
}

}  // namespace

extern "C" {

// Datasheet-derived placeholders (replaced by a calibration file):
//   148 SMs; 8192 dense FP16 FLOP/cycle/SM, so one 128x256x16 MMA
//   (1,048,576 FLOP) takes 128 cycles; 2.25 PFLOP/s needs ~1.86 GHz, but a
//   1 kW part holds about 1.4 GHz under sustained tensor load; shared memory
//   feeds 128 B/cycle/SM; HBM3e 8 TB/s nominal; L2 126 MB; the GEMM's one
//   producer thread needs about 320 cycles per TMA box.
int ridge_hw_b200(ridge_hw* h) {
    if (!h) return RIDGE_EINVAL;
    std::memset(h, 0, sizeof(*h));
    std::snprintf(h->name, sizeof(h->name), "B200 (datasheet placeholders)");
    h->num_sms = 148;
    h->clock_hz = 1.4e9;
    h->umma_cycles_128x256 = 128.0;
    h->umma_m64_ratio = 1.0;
    h->smem_bytes_per_cycle = 128.0;
    h->smem_mma_overlap = 1.0;
    h->l2_bytes_per_sec = 20e12;
    h->hbm_bytes_per_sec = 6.5e12;
    h->tma_box_cycles = 320.0;
    h->tma_box2_ratio = 1.0;
    h->tma_box32_ratio = 1.0;
    h->pipeline_efficiency = 0.9;
    h->tile_overhead_cycles = 0.0;
    h->pair_tile_overhead_cycles = 0.0;
    h->c_write_bytes_per_sec = 6.5e12;
    h->epi_bytes_per_cycle_w4 = 32.0;
    h->epi_bytes_per_cycle_w8 = 48.0;
    h->tma_latency_cycles = 1000.0;
    h->tma_latency_hbm_cycles = 1000.0;
    h->launch_overhead_sec = 4e-6;
    h->l2_bytes = 126.0 * 1024 * 1024;
    h->smem_bytes_per_sm = 233472;
    h->tmem_cols_per_sm = 512;
    h->max_ctas_per_sm = 32;
    h->calibrated = 0;
    return RIDGE_OK;
}

int ridge_hw_load_json(const char* path, ridge_hw* out, char* errbuf, int32_t errlen) {
    if (!path || !out) {
        set_err(errbuf, errlen, "null argument");
        return RIDGE_EINVAL;
    }
    std::ifstream in(path);
    if (!in) {
        set_err(errbuf, errlen, std::string("cannot open ") + path);
        return RIDGE_EIO;
    }
    std::stringstream ss;
    ss << in.rdbuf();
    std::map<std::string, std::string> kv;
    std::string err;
    if (!parse_flat_json(ss.str(), kv, err)) {
        set_err(errbuf, errlen, std::string(path) + ": " + err);
        return RIDGE_EIO;
    }
    // Build into a temporary: a file that fails part way leaves *out untouched.
    ridge_hw h;
    ridge_hw_b200(&h);
    auto name = kv.find("name");
    std::snprintf(h.name, sizeof(h.name), "%s", name != kv.end() ? name->second.c_str() : path);
    struct Req {
        const char* key;
        double* dst;
    } dbl[] = {{"clockHz", &h.clock_hz},
               {"ummaCycles128x256", &h.umma_cycles_128x256},
               {"ummaM64Ratio", &h.umma_m64_ratio},
               {"smemBytesPerCycle", &h.smem_bytes_per_cycle},
               {"smemMmaOverlap", &h.smem_mma_overlap},
               {"l2BytesPerSec", &h.l2_bytes_per_sec},
               {"hbmBytesPerSec", &h.hbm_bytes_per_sec},
               {"tmaBoxCycles", &h.tma_box_cycles},
               {"tmaBoxCycles128Ratio", &h.tma_box2_ratio},
               {"tmaBoxCycles32Ratio", &h.tma_box32_ratio},
               {"pipelineEfficiency", &h.pipeline_efficiency},
               {"tileOverheadCycles", &h.tile_overhead_cycles},
               {"pairTileOverheadCycles", &h.pair_tile_overhead_cycles},
               {"cWriteBytesPerSec", &h.c_write_bytes_per_sec},
               {"epiBytesPerCycleW4", &h.epi_bytes_per_cycle_w4},
               {"epiBytesPerCycleW8", &h.epi_bytes_per_cycle_w8},
               {"tmaLatencyCycles", &h.tma_latency_cycles},
               {"tmaLatencyHbmCycles", &h.tma_latency_hbm_cycles},
               {"launchOverheadSec", &h.launch_overhead_sec},
               {"l2Bytes", &h.l2_bytes}};
    for (const Req& r : dbl) {
        if (!number(kv, r.key, *r.dst, err)) {
            set_err(errbuf, errlen, std::string(path) + ": " + err);
            return RIDGE_EIO;
        }
    }
    struct ReqI {
        const char* key;
        int32_t* dst;
    } ints[] = {{"numSMs", &h.num_sms},
                {"smemBytesPerSM", &h.smem_bytes_per_sm},
                {"tmemColsPerSM", &h.tmem_cols_per_sm},
                {"maxCtasPerSM", &h.max_ctas_per_sm}};
    for (const ReqI& r : ints) {
        double v = 0;
        if (!number(kv, r.key, v, err)) {
            set_err(errbuf, errlen, std::string(path) + ": " + err);
            return RIDGE_EIO;
        }
        *r.dst = int32_t(v);
    }
    // Values that would make the model divide by zero or silently zero a
    // ceiling are refused rather than loaded.
    if (h.num_sms <= 0 || h.clock_hz <= 0 || h.umma_cycles_128x256 <= 0 ||
        h.umma_m64_ratio <= 0 || h.smem_bytes_per_cycle <= 0 || h.l2_bytes_per_sec <= 0 ||
        h.hbm_bytes_per_sec <= 0 || h.tma_box_cycles <= 0 || h.tma_box2_ratio <= 0 ||
        h.tma_box32_ratio <= 0 || h.pipeline_efficiency <= 0 || h.pipeline_efficiency > 1 ||
        h.tile_overhead_cycles < 0 || h.pair_tile_overhead_cycles < 0 || h.c_write_bytes_per_sec <= 0 ||
        h.epi_bytes_per_cycle_w4 <= 0 ||
        h.epi_bytes_per_cycle_w8 <= 0 || h.tma_latency_cycles < 0 || h.tma_latency_hbm_cycles < 0 || h.launch_overhead_sec < 0 ||
        h.l2_bytes <= 0 || h.smem_bytes_per_sm <= 0 || h.tmem_cols_per_sm <= 0 ||
        h.max_ctas_per_sm <= 0 || h.smem_mma_overlap < 0 || h.smem_mma_overlap > 1) {
        set_err(errbuf, errlen, std::string(path) + ": a required constant is out of range");
        return RIDGE_EINVAL;
    }
    h.calibrated = 1;
    *out = h;
    return RIDGE_OK;
}

}  // extern "C"
