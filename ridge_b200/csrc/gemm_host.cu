// C-ABI front end of the GEMM family: the variant table, config validation,
// TMA tensor-map construction and the launcher (include/ridge_b200.h).
//
// Reference counterparts: the KernelVariant table and launchVariant in
// bench/kernels/gemm-mma.cu:19-141. Differences by design: stages and groupM
// are runtime values (one compiled kernel serves every depth), shapes need not
// divide the tile, and every launch validates its arguments and returns a
// status instead of relying on the caller to skip bad combinations.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "../../include/ridge_b200.h"
#include "gemm_registry.h"
#include "gemm_sm100.cuh"

namespace ridge_b200 {

int noalloc_fill_counters(int byte);  // gemm_noalloc.cu

// Per-device error word written by kernels whose bounded waits expire.
__device__ int g_ridge_device_err = 0;

#ifdef RIDGE_TRACE
__device__ unsigned long long g_ridge_trace[512][64];
#endif

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxDynSmem = 232448;   // 227 KB opt-in limit per CTA on sm_100
constexpr int kSmemPerSm = 233472;    // 228 KB per SM
constexpr int kSmemReservedPerCta = 1024;
constexpr int kTmemColsPerSm = 512;
constexpr int64_t kCounterBytes = 64 * 1024;
constexpr int64_t kMinSplitBlocks = 4;  // K-blocks per split-K range, at least
constexpr int64_t kSplitFirstMaxRounds = 6;  // whole-tile rounds up to which splits run first

// The bounded-wait self-test: one thread waits on an mbarrier that nothing
// will ever complete, through the same mbar_wait the GEMM's pipeline uses,
// with a short limit; when it gives up it raises the abort flag and records
// kErrSelfTest in the error word, exactly as a stalled GEMM stage would.
__global__ void selftest_wait_kernel(int* err, uint64_t limit_ns, unsigned long long* waited,
                                     int* abort_seen) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_timer_ns();
        const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_flag, err, kErrSelfTest, limit_ns);
        *waited = global_timer_ns() - t0;
        *abort_seen = ok ? -1 : abort_flag;
    }
}

const std::vector<KernelEntry>& registry() {
    static const std::vector<KernelEntry> entries = [] {
        std::vector<KernelEntry> v;
        register_bm64(v);
        register_bm128(v);
        register_bm256(v);
        register_bm256_pair(v);
        return v;
    }();
    return entries;
}

struct DeviceState {
    std::once_flag once;
    cudaError_t init_err = cudaSuccess;
    bool is_sm100 = false;
    int num_sms = 0;
    int* err_word = nullptr;
    std::atomic<bool> smem_attr_set[256];
    std::atomic<int> cluster_units[256][kMaxStages + 1];  // 0 = not queried yet
};

DeviceState g_dev[kMaxDevices];

DeviceState* device_state(int* status) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = int(e);
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *status = RIDGE_ENOTSUP;
        return nullptr;
    }
    DeviceState& d = g_dev[dev];
    std::call_once(d.once, [&] {
        cudaDeviceProp prop{};
        d.init_err = cudaGetDeviceProperties(&prop, dev);
        if (d.init_err != cudaSuccess) return;
        d.is_sm100 = prop.major == 10 && prop.minor == 0;
        d.num_sms = prop.multiProcessorCount;
        d.init_err = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err_word), g_ridge_device_err);
        for (auto& f : d.smem_attr_set) f.store(false);
        for (auto& row : d.cluster_units)
            for (auto& u : row) u.store(0);
    });
    if (d.init_err != cudaSuccess) {
        *status = int(d.init_err);
        return nullptr;
    }
    if (!d.is_sm100) {
        *status = RIDGE_ENOTSUP;
        return nullptr;
    }
    *status = RIDGE_OK;
    return &d;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// K-major FP16 operand, `rows` x `cols` (cols = K contiguous), leading
// dimension `ld` elements, box = box_rows x BK with the swizzle equal to one
// BK row (64B for BK=32, 128B for BK=64). Out-of-range elements read as zero.
int make_operand_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                     int box_rows, int bk) {
    auto enc = tensor_map_encoder();
    if (!enc) return RIDGE_ENOTSUP;
    CUresult r;
    if (bk <= 64) {
        cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
        cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
        cuuint32_t box[2] = {cuuint32_t(bk), cuuint32_t(box_rows)};
        cuuint32_t estr[2] = {1, 1};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                bk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        // BK=128: view the operand as (64 columns of an atom) x rows x (K / 64
        // atoms), atom stride 128 B, and load bk/64 atoms per box; the box lands
        // atom-major in shared memory (rows x 128 B per atom), the layout the
        // 128B-swizzled UMMA descriptors read. Needs K to be a multiple of 64.
        cuuint64_t dims[3] = {64, cuuint64_t(rows), cuuint64_t(cols / 64)};
        cuuint64_t strides[2] = {cuuint64_t(ld) * 2, 128};
        cuuint32_t box[3] = {64, cuuint32_t(box_rows), cuuint32_t(bk / 64)};
        cuuint32_t estr[3] = {1, 1, 1};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    return r == CUDA_SUCCESS ? RIDGE_OK : RIDGE_EINVAL;
}

// Producer threads issuing TMA loads: 1 (default), 2 or 4, read once from
// RIDGE_TMA_ISSUERS (a knob for measurement). Measured on the GEMM itself, one
// issuing thread keeps the ring as full as four: the loads are asynchronous,
// and several issuing lanes of one warp spinning on different stage barriers
// only diverge (256x256x128 pair tile, L2-flushed launches: 1385 against 1340
// TFLOP/s at 4096^3, 1547 against 1391-1418 at 8192^3).
int tma_issuers() {
    static const int n = [] {
        const char* v = std::getenv("RIDGE_TMA_ISSUERS");
        const int x = v ? std::atoi(v) : 1;
        return (x == 1 || x == 2 || x == 4) ? x : 1;
    }();
    return n;
}

// BM=256 tiles default to the 2-CTA pair (half the shared-memory operand
// traffic per SM and two TMEM accumulators); cta_group 1 selects the
// single-CTA form explicitly.
int default_cta_group(const ridge_tile_config& c) { return c.BM == 256 ? 2 : 1; }

// Row-major FP16 C (rows x cols, leading dimension ld) for the epilogue's TMA
// stores: box = 32 columns (64 B, 64B swizzle) x box_rows rows. Stores that
// fall outside rows/cols are clipped by the hardware.
int make_output_map(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows, int box_cols) {
    auto enc = tensor_map_encoder();
    if (!enc) return RIDGE_ENOTSUP;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? RIDGE_OK : RIDGE_EINVAL;
}

const KernelEntry* find_entry(const ridge_tile_config& c, int* index = nullptr) {
    const int cg = c.cta_group == 0 ? default_cta_group(c) : c.cta_group;
    const auto& reg = registry();
    for (size_t i = 0; i < reg.size(); ++i) {
        const KernelEntry& e = reg[i];
        if (e.BM == c.BM && e.BN == c.BN && e.BK == c.BK && e.warps == c.warps &&
            e.cta_group == cg) {
            if (index) *index = int(i);
            return &e;
        }
    }
    return nullptr;
}

int smem_for(const KernelEntry& e, int stages) { return e.fixed_smem + stages * e.stage_bytes; }

// Dynamic shared memory a launch requests. When shared memory alone would let
// more CTAs share an SM than Tensor Memory can hold, the request is padded so
// the hardware never co-schedules a CTA whose tcgen05.alloc would have to
// wait for another CTA to exit: such a CTA would only idle on its SM, and the
// grid is sized to the CTAs that can run at once.
int launch_smem(const KernelEntry& e, int stages) {
    int smem = e.fixed_smem + stages * e.stage_bytes;
    const int by_tmem = kTmemColsPerSm / e.tmem_cols;
    const int by_smem = kSmemPerSm / (smem + kSmemReservedPerCta);
    if (by_smem > by_tmem) {
        const int pad_to = kSmemPerSm / (by_tmem + 1) - kSmemReservedPerCta + 1;
        smem = std::max(smem, pad_to);
    }
    return smem;
}

int ctas_per_sm(const KernelEntry& e, int stages) {
    const int by_smem = kSmemPerSm / (smem_for(e, stages) + kSmemReservedPerCta);
    const int by_tmem = kTmemColsPerSm / e.tmem_cols;
    const int by_threads = 2048 / e.threads;
    return std::max(0, std::min(std::min(by_smem, by_tmem), by_threads));
}

// The registered table: the full grid BM, BN in {64,128,256}, BK in {32,64}
// (BASELINE) widened with BK=128 (two K atoms per TMA box, half the boxes per
// unit of MMA work), stages in {2..6}, warps in {4,8}, groupM 8, minus the
// points that overflow shared memory; BM=256 appears twice, as the 2-CTA pair
// and as the single-CTA form.
const std::vector<ridge_tile_config>& variant_table() {
    static const std::vector<ridge_tile_config> table = [] {
        std::vector<ridge_tile_config> t;
        const int bms[] = {64, 128, 256}, bns[] = {64, 128, 256}, bks[] = {32, 64, 128};
        const int stages[] = {2, 3, 4, 5, 6}, warps[] = {4, 8};
        for (int bm : bms)
            for (int bn : bns)
                for (int bk : bks)
                    for (int s : stages)
                        for (int w : warps)
                            for (int cg = 1; cg <= (bm == 256 ? 2 : 1); ++cg) {
                                ridge_tile_config c{bm, bn, bk, s, w, 8, cg, 0};
                                if (ridge_config_check(&c, nullptr) == RIDGE_OK) t.push_back(c);
                            }
        return t;
    }();
    return table;
}

void fill_info(const KernelEntry& e, const ridge_tile_config& c, ridge_variant_info* info) {
    std::memset(info, 0, sizeof(*info));
    info->cfg = c;
    info->cfg.cta_group = e.cta_group;
    info->smem_bytes = smem_for(e, c.stages);
    info->threads = e.threads;
    info->cluster_size = e.cta_group;
    info->tmem_cols = e.tmem_cols;
    info->acc_buffers = e.acc_bufs;
    std::snprintf(info->kernel_name, sizeof(info->kernel_name), "%s", e.name);
    cudaFuncAttributes fa{};
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0 &&
        cudaFuncGetAttributes(&fa, e.func) == cudaSuccess)
        info->regs_per_thread = fa.numRegs;
    else
        cudaGetLastError();
}

// ------------------------------------------------------------------ launch planning

struct LaunchPlan {
    const KernelEntry* e = nullptr;
    int idx = -1;
    int smem = 0;
    int epi_stride = 4096;  // epilogue staging bytes per warp (8192: double-buffered pairs)
    int grid_units = 0;  // CTAs (1-CTA kernels) or CTA pairs
    int dp_tiles = 0, sk_tiles = 0, sk_splits = 1;
    int sk_first = 0;
    size_t ws_partials = 0;  // bytes of FP32 partial tiles
    size_t ws_bytes = 0;     // total workspace (partials + counters)
};

// Co-resident tile units of `e` at depth `stages` on `dev`. 2-CTA pairs must
// sit on one TPC, so those are asked of the runtime (once per kernel, depth
// and device) rather than assumed to be SMs / 2.
int64_t resident_units(const KernelEntry& e, int idx, int stages, int smem, DeviceState* dev) {
    int64_t slots = int64_t(dev->num_sms / e.cta_group) * ctas_per_sm(e, stages);
    if (e.cta_group > 1) {
        std::atomic<int>& cached = dev->cluster_units[idx][stages];
        int units = cached.load(std::memory_order_relaxed);
        if (units == 0) {
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(unsigned(e.cta_group * 2), 1, 1);
            lc.blockDim = dim3(unsigned(e.threads), 1, 1);
            lc.dynamicSmemBytes = size_t(smem);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = unsigned(e.cta_group);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            lc.attrs = attr;
            lc.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, e.func, &lc) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = int(slots);
            }
            units = n;
            cached.store(units, std::memory_order_relaxed);
        }
        slots = std::min<int64_t>(slots, units);
    }
    return std::max<int64_t>(slots, 1);
}

int ensure_smem_attr(const KernelEntry& e, int idx, DeviceState* dev) {
    if (!dev->smem_attr_set[idx].load(std::memory_order_acquire)) {
        cudaError_t ce =
            cudaFuncSetAttribute(e.func, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
        if (ce != cudaSuccess) return int(ce);
        dev->smem_attr_set[idx].store(true, std::memory_order_release);
    }
    return RIDGE_OK;
}

// Grid size and split-K tail for one launch. With U resident units and T
// tiles, whole tiles fill floor(T / U) rounds; the R = T mod U tiles of a
// partial last round (all T when T < U) are split along K into
// s = floor(U / R) ranges (at most 8, at least 4 K-blocks each) so the round
// keeps R * s units busy instead of R. s < 2 means no split.
int make_plan(const ridge_tile_config& cfg, int64_t M, int64_t N, int64_t K, DeviceState* dev,
              LaunchPlan* plan) {
    int idx = -1;
    const KernelEntry* e = find_entry(cfg, &idx);
    if (!e) return RIDGE_EINVAL;
    plan->e = e;
    plan->idx = idx;
    plan->smem = launch_smem(*e, cfg.stages);
    // Kernels that store 32 x 64 pairs get a second 4 KB staging buffer per
    // warp when it fits without costing a co-resident CTA: the next pair is
    // then staged while the previous store is still reading the first.
    plan->epi_stride = 4096;
    if (e->epi_cols == 64) {
        const int want = std::max(plan->smem, smem_for(*e, cfg.stages) + e->warps * 4096);
        auto resident = [&](int s) {
            return std::min(kSmemPerSm / (s + kSmemReservedPerCta), kTmemColsPerSm / e->tmem_cols);
        };
        if (want <= kMaxDynSmem && resident(want) == resident(plan->smem)) {
            plan->smem = want;
            plan->epi_stride = 8192;
        }
    }
    int st = ensure_smem_attr(*e, idx, dev);
    if (st != RIDGE_OK) return st;
    const int64_t tiles = ((M + e->BM - 1) / e->BM) * ((N + e->BN - 1) / e->BN);
    const int64_t units = resident_units(*e, idx, cfg.stages, plan->smem, dev);
    const int64_t num_kb = (K + e->BK - 1) / e->BK;
    if (tiles > int64_t(1) << 30) return RIDGE_EINVAL;
    plan->grid_units = int(std::min(tiles, units));
    plan->dp_tiles = int(tiles);
    plan->sk_tiles = 0;
    plan->sk_splits = 1;
    plan->ws_partials = plan->ws_bytes = 0;
    if (cfg.split_k == 1) return RIDGE_OK;
    const int64_t rem = tiles >= units ? tiles % units : tiles;
    if (rem == 0) return RIDGE_OK;
    // Each K range keeps at least kMinSplitBlocks K-blocks: below that the
    // FP32 partial round-trip costs about what the split saves.
    const int64_t s = std::min<int64_t>(std::min<int64_t>(units / rem, 8), num_kb / kMinSplitBlocks);
    if (s < 2) return RIDGE_OK;
    plan->dp_tiles = int(tiles - rem);
    plan->sk_tiles = int(rem);
    plan->sk_splits = int(s);
    // Split ranges first when the whole tiles fill few rounds: the partial
    // exchange then hides behind the next tile instead of trailing the last
    // one (4096^3, 3 rounds: 1370 -> 1427 TFLOP/s). With many rounds the tail
    // is a small share, and keeping every unit on the same round keeps the
    // tiles in flight together in L2 (16384^3, 55 rounds: 1375 against 1350).
    plan->sk_first = (tiles - rem) / units <= kSplitFirstMaxRounds ? 1 : 0;
    plan->grid_units = int(std::max<int64_t>(std::min(tiles, units), rem * s));
    // Workspace: [counters: kCounterBytes][FP32 partial tiles]. The counter
    // area sits at a fixed offset so that every config sharing a workspace
    // finds it zeroed (the last arrival resets each counter; partials never
    // overlap it).
    if (rem * e->cta_group * e->warps * 8 > kCounterBytes) {  // two ints per warp
        plan->dp_tiles = int(tiles);
        plan->sk_tiles = 0;
        plan->sk_splits = 1;
        plan->grid_units = int(std::min(tiles, units));
        return RIDGE_OK;
    }
    const size_t tile_floats = size_t(e->partial_floats);
    plan->ws_partials = size_t(rem) * s * e->cta_group * tile_floats * 4;  // one slot per split
    plan->ws_bytes = kCounterBytes + plan->ws_partials;
    return RIDGE_OK;
}

// Library-owned split-K workspaces, one per (device, stream), grown on demand
// and zeroed when (re)allocated; kernels leave their counters at zero.
struct WorkspaceCache {
    std::mutex mu;
    std::map<cudaStream_t, std::pair<void*, size_t>> by_stream;
};
WorkspaceCache g_ws[kMaxDevices];

int cached_workspace(int device, cudaStream_t stream, size_t bytes, void** out) {
    WorkspaceCache& c = g_ws[device];
    std::lock_guard<std::mutex> lock(c.mu);
    auto& slot = c.by_stream[stream];
    if (slot.second < bytes) {
        if (slot.first) {
            cudaError_t ce = cudaStreamSynchronize(stream);
            if (ce != cudaSuccess) return int(ce);
            cudaFree(slot.first);
            slot = {nullptr, 0};
        }
        void* p = nullptr;
        const size_t want = std::max<size_t>(bytes, size_t(1) << 20);
        cudaError_t ce = cudaMalloc(&p, want);
        if (ce != cudaSuccess) return int(ce);
        ce = cudaMemsetAsync(p, 0, want, stream);
        if (ce != cudaSuccess) {
            cudaFree(p);
            return int(ce);
        }
        slot = {p, want};
    }
    *out = slot.first;
    return RIDGE_OK;
}

int launch_common(const ridge_tile_config* cfg, const void* A, const void* B, void* C, int64_t M,
                  int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream_v,
                  bool caller_ws, void* workspace, int64_t workspace_bytes,
                  void* const* peer_c = nullptr, int num_peers = 0) {
    int st = ridge_config_valid_for_shape(cfg, M, N, K, lda, ldb, ldc);
    if (st != RIDGE_OK) return st;
    if (M == 0 || N == 0) return RIDGE_OK;
    if (!A || !B || !C) return RIDGE_EINVAL;
    if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
        (reinterpret_cast<uintptr_t>(C) & 1))
        return RIDGE_EINVAL;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    DeviceState* dev = device_state(&st);
    if (!dev) return st;
    if (num_peers < 0 || num_peers > kMaxPeers || (num_peers > 0 && !peer_c)) return RIDGE_EINVAL;
    if (K == 0) {
        cudaError_t e = cudaMemset2DAsync(C, size_t(ldc) * 2, 0, size_t(N) * 2, size_t(M), stream);
        for (int d = 0; d < num_peers && e == cudaSuccess; ++d)
            e = cudaMemset2DAsync(peer_c[d], size_t(ldc) * 2, 0, size_t(N) * 2, size_t(M), stream);
        return int(e);
    }
    LaunchPlan plan;
    st = make_plan(*cfg, M, N, K, dev, &plan);
    if (st != RIDGE_OK) return st;
    const KernelEntry* e = plan.e;

    void* ws = nullptr;
    if (plan.ws_bytes > 0) {
        if (caller_ws) {
            if (!workspace || workspace_bytes < int64_t(plan.ws_bytes) ||
                (reinterpret_cast<uintptr_t>(workspace) & 255))
                return RIDGE_EINVAL;
            ws = workspace;
        } else {
            int device = 0;
            cudaGetDevice(&device);
            st = cached_workspace(device, stream, plan.ws_bytes, &ws);
            if (st != RIDGE_OK) return st;
        }
    }

    CUtensorMap tmap_a, tmap_b, tmap_c;
    st = make_operand_map(&tmap_a, A, M, K, lda, e->tile_a_rows, e->BK);
    if (st != RIDGE_OK) return st;
    st = make_operand_map(&tmap_b, B, N, K, ldb, e->tile_b_rows, e->BK);
    if (st != RIDGE_OK) return st;
    // The TMA-store epilogue needs a 16-byte aligned C with a 16-byte row
    // pitch; otherwise the kernel stores directly from registers.
    const bool tma_store = (reinterpret_cast<uintptr_t>(C) & 15) == 0 && (ldc % 8) == 0;
    std::memset(&tmap_c, 0, sizeof(tmap_c));
    if (tma_store) {
        st = make_output_map(&tmap_c, C, M, N, ldc, e->epi_rows, e->epi_cols);
        if (st != RIDGE_OK) return st;
    }
    // Peer copies of C take the same tile stores through their own maps, so
    // they need the TMA-store epilogue (16-byte aligned, 16-byte pitch).
    PeerMaps peers;
    std::memset(&peers, 0, sizeof(peers));
    if (num_peers > 0 && !tma_store) return RIDGE_EINVAL;
    for (int d = 0; d < num_peers; ++d) {
        if (!peer_c[d] || (reinterpret_cast<uintptr_t>(peer_c[d]) & 15)) return RIDGE_EINVAL;
        st = make_output_map(&peers.map[d], peer_c[d], M, N, ldc, e->epi_rows, e->epi_cols);
        if (st != RIDGE_OK) return st;
    }

    GemmParams p;
    p.C = static_cast<__half*>(C);
    p.M = int(M);
    p.N = int(N);
    p.K = int(K);
    p.ldc = ldc;
    p.groupM = cfg->groupM;
    p.stages = cfg->stages;
    p.tma_store = tma_store ? 1 : 0;
    p.epi_stride = plan.epi_stride;
    p.tma_issuers = tma_issuers();
    p.num_peers = num_peers;
    p.err = dev->err_word;
    p.dp_tiles = plan.dp_tiles;
    p.sk_tiles = plan.sk_tiles;
    p.sk_splits = plan.sk_splits;
    p.sk_first = plan.sk_first;
    p.counters = static_cast<int*>(ws);
    p.workspace = ws ? reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes) : nullptr;
    cudaError_t ce = e->launch(&tmap_a, &tmap_b, &tmap_c, &peers, &p,
                               plan.grid_units * e->cta_group, plan.smem, stream);
    return int(ce);
}

// Sets every byte of the split-K counter areas this library owns on the current
// device (cached workspaces, the no-allocation scratch) to `byte`.
int fill_library_counters(int byte) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return int(e);
    {
        WorkspaceCache& c = g_ws[device];
        std::lock_guard<std::mutex> lock(c.mu);
        for (auto& kv : c.by_stream) {
            if (!kv.second.first) continue;
            e = cudaMemset(kv.second.first, byte, size_t(kCounterBytes));
            if (e != cudaSuccess) return int(e);
        }
    }
    return noalloc_fill_counters(byte);
}

}  // namespace
}  // namespace ridge_b200

using namespace ridge_b200;

extern "C" {

const char* ridge_status_string(int s) {
    switch (s) {
        case RIDGE_OK: return "ok";
        case RIDGE_EINVAL: return "invalid tile config, shape, stride or alignment";
        case RIDGE_EDEVICE: return "a kernel recorded a device-side error (bounded wait expired)";
        case RIDGE_ENOTSUP: return "not supported on this device (needs sm_100)";
        case RIDGE_EIO: return "file missing or unparseable";
        case RIDGE_ERANGE: return "index out of range";
        case RIDGE_ECOMM: return "NCCL missing from the process or an NCCL call failed";
        case RIDGE_ENOSCRATCH:
            return "launch needs more split-K scratch than the fixed no-allocation array holds";
        default: break;
    }
    if (s > 0) return cudaGetErrorString(cudaError_t(s));
    return "unknown ridge status";
}

int ridge_config_check(const ridge_tile_config* cfg, ridge_variant_info* info) {
    if (!cfg) return RIDGE_EINVAL;
    const ridge_tile_config& c = *cfg;
    if (c.stages < 2 || c.stages > kMaxStages || c.groupM < 1) return RIDGE_EINVAL;
    if (c.split_k != 0 && c.split_k != 1) return RIDGE_EINVAL;
    const KernelEntry* e = find_entry(c);
    if (!e) return RIDGE_EINVAL;
    if (smem_for(*e, c.stages) > kMaxDynSmem) return RIDGE_EINVAL;
    if (e->tmem_cols > kTmemColsPerSm) return RIDGE_EINVAL;
    if (ctas_per_sm(*e, c.stages) < 1) return RIDGE_EINVAL;
    if (info) fill_info(*e, c, info);
    return RIDGE_OK;
}

int ridge_num_variants(void) { return int(variant_table().size()); }

int ridge_variant(int index, ridge_variant_info* out) {
    const auto& t = variant_table();
    if (index < 0 || index >= int(t.size()) || !out) return RIDGE_ERANGE;
    return ridge_config_check(&t[index], out);
}

void ridge_print_variant_table(void) {
    std::printf("%3s %4s %4s %3s %6s %5s %5s %3s %7s %5s %5s\n", "idx", "BM", "BN", "BK", "stages",
                "warps", "grpM", "cg", "smemB", "tmem", "accs");
    for (int i = 0; i < ridge_num_variants(); ++i) {
        ridge_variant_info v;
        ridge_variant(i, &v);
        std::printf("%3d %4d %4d %3d %6d %5d %5d %3d %7d %5d %5d\n", i, v.cfg.BM, v.cfg.BN,
                    v.cfg.BK, v.cfg.stages, v.cfg.warps, v.cfg.groupM, v.cfg.cta_group,
                    v.smem_bytes, v.tmem_cols, v.acc_buffers);
    }
}

int ridge_config_valid_for_shape(const ridge_tile_config* cfg, int64_t M, int64_t N, int64_t K,
                                 int64_t lda, int64_t ldb, int64_t ldc) {
    if (ridge_config_check(cfg, nullptr) != RIDGE_OK) return RIDGE_EINVAL;
    if (M < 0 || N < 0 || K < 0) return RIDGE_EINVAL;
    if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
        return RIDGE_EINVAL;
    if (lda < K || ldb < K || ldc < N) return RIDGE_EINVAL;
    if (lda % 8 != 0 || ldb % 8 != 0) return RIDGE_EINVAL;  // TMA: strides multiple of 16 B
    if (lda < 8 || ldb < 8) return RIDGE_EINVAL;
    if (cfg->BK == 128 && K % 64 != 0) return RIDGE_EINVAL;  // whole 64-wide K atoms
    return RIDGE_OK;
}

int ridge_gemm_workspace_size(const ridge_tile_config* cfg, int64_t M, int64_t N, int64_t K,
                              int64_t* bytes) {
    if (!bytes) return RIDGE_EINVAL;
    // The workspace does not depend on the pitches: validate with the
    // smallest legal ones (K rounded up to a multiple of 8).
    const int64_t ld = (std::max<int64_t>(K, 8) + 7) / 8 * 8;
    int st = ridge_config_valid_for_shape(cfg, M, N, K, ld, ld, N);
    if (st != RIDGE_OK) return st;
    *bytes = 0;
    if (M == 0 || N == 0 || K == 0) return RIDGE_OK;
    DeviceState* dev = device_state(&st);
    if (!dev) return st;
    LaunchPlan plan;
    st = make_plan(*cfg, M, N, K, dev, &plan);
    if (st != RIDGE_OK) return st;
    *bytes = int64_t(plan.ws_bytes);
    return RIDGE_OK;
}

int ridge_gemm_launch_ws(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                         int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                         void* workspace, int64_t workspace_bytes, void* stream) {
    return launch_common(cfg, A, B, C, M, N, K, lda, ldb, ldc, stream, true, workspace,
                         workspace_bytes);
}

int ridge_gemm_launch_multi(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                            int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                            int64_t ldc, void* const* peer_c, int32_t num_peers, void* stream) {
    return launch_common(cfg, A, B, C, M, N, K, lda, ldb, ldc, stream, false, nullptr, 0, peer_c,
                         num_peers);
}

int ridge_gemm_launch(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                      int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                      void* stream) {
    return launch_common(cfg, A, B, C, M, N, K, lda, ldb, ldc, stream, false, nullptr, 0);
}

int ridge_gemm_launch_variant(int index, const void* A, const void* B, void* C, int64_t M,
                              int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                              void* stream) {
    const auto& t = variant_table();
    if (index < 0 || index >= int(t.size())) return RIDGE_ERANGE;
    return ridge_gemm_launch(&t[index], A, B, C, M, N, K, lda, ldb, ldc, stream);
}

int ridge_selftest_wait_timeout(int64_t limit_ns, int32_t* code, int64_t* waited_ns) {
    if (limit_ns < 1000000 || limit_ns > 2000000000ll || !code || !waited_ns) return RIDGE_EINVAL;
    int st = RIDGE_OK;
    DeviceState* dev = device_state(&st);
    if (!dev) return st;
    // start from a clean error word so the code read back is this test's
    int32_t before = 0;
    if ((st = ridge_device_error(1, &before)) != RIDGE_OK) return st;
    unsigned long long* d_waited = nullptr;
    int* d_abort = nullptr;
    cudaError_t e = cudaMalloc(&d_waited, sizeof(unsigned long long) + sizeof(int) * 2);
    if (e != cudaSuccess) return int(e);
    d_abort = reinterpret_cast<int*>(d_waited + 1);
    selftest_wait_kernel<<<1, 32>>>(dev->err_word, uint64_t(limit_ns), d_waited, d_abort);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    unsigned long long w = 0;
    int ab = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&w, d_waited, sizeof(w), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&ab, d_abort, sizeof(ab), cudaMemcpyDeviceToHost);
    cudaFree(d_waited);
    if (e != cudaSuccess) return int(e);
    if ((st = ridge_device_error(1, code)) != RIDGE_OK) return st;
    *waited_ns = int64_t(w);
    // the wait must have given up (not completed) and raised the abort flag
    return ab == 1 ? RIDGE_OK : RIDGE_EDEVICE;
}

#ifdef RIDGE_TRACE
// Timeline probe readout (trace builds only): copies and clears the per-CTA
// stamps of the last launch.
int ridge_trace_read(void* host, int64_t bytes) {
    if (bytes < int64_t(sizeof(g_ridge_trace))) return RIDGE_EINVAL;
    cudaError_t e = cudaMemcpyFromSymbol(host, g_ridge_trace, sizeof(g_ridge_trace));
    if (e == cudaSuccess) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_ridge_trace);
        if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(g_ridge_trace));
    }
    return int(e);
}
#endif

int ridge_device_error(int clear, int32_t* code) {
    int st = RIDGE_OK;
    DeviceState* dev = device_state(&st);
    if (!dev) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return int(e);
    int v = 0;
    e = cudaMemcpy(&v, dev->err_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return int(e);
    if (code) *code = v;
    if (clear && v != 0) {
        e = cudaMemset(dev->err_word, 0, sizeof(int));
        if (e != cudaSuccess) return int(e);
        // A kernel that gave up may have left split-K counters non-zero: in
        // the library's cached workspaces and in the no-allocation scratch.
        if ((st = fill_library_counters(0)) != RIDGE_OK) return st;
    }
    return RIDGE_OK;
}

int ridge_selftest_stale_counters(int32_t byte) {
    if (byte < 1 || byte > 255) return RIDGE_EINVAL;
    int st = RIDGE_OK;
    DeviceState* dev = device_state(&st);
    if (!dev) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return int(e);
    if ((st = fill_library_counters(byte)) != RIDGE_OK) return st;
    const int code = kErrSelfTestStale;
    e = cudaMemcpy(dev->err_word, &code, sizeof(int), cudaMemcpyHostToDevice);
    return int(e);
}

}  // extern "C"
