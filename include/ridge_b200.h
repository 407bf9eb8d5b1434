/*
 * ridge_b200.h -- C ABI of the B200-native (sm_100a) ridge GEMM hot path.
 *
 * Plain C: fixed-width integers, plain pointers, no CUDA or torch types. A
 * stream is passed as `void*` (a cudaStream_t; NULL = the legacy default
 * stream). Every entry point returns an int status: 0 = RIDGE_OK, a positive
 * value = the cudaError_t that stopped it, a negative value = one of the
 * RIDGE_E* codes below. Launches are asynchronous on the given stream and never
 * synchronise; the caller owns and frees every buffer.
 *
 * Reference interfaces each declaration replaces are cited beside it; paths are
 * relative to the reference project root (i-nahc/ridge).
 */
#ifndef RIDGE_B200_H
#define RIDGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */

#define RIDGE_OK 0
#define RIDGE_EINVAL (-1)   /* invalid tile config, shape, stride or alignment */
#define RIDGE_EDEVICE (-2)  /* a kernel recorded a device-side error (bounded wait expired) */
#define RIDGE_ENOTSUP (-3)  /* device is not sm_100 / feature not built */
#define RIDGE_EIO (-4)      /* file missing or unparseable */
#define RIDGE_ERANGE (-5)   /* index out of range */
#define RIDGE_ENOSCRATCH (-6) /* launch needs more scratch than ridge_gemm_launch_noalloc has */
#define RIDGE_ECOMM (-7)      /* NCCL missing or an NCCL call failed (ridge_gemm_sharded) */

/* Human-readable text for any status returned by this library. */
const char* ridge_status_string(int status);

/* ---------------------------------------------------------------- tile configs */

/*
 * One tile configuration of the GEMM family. Replaces the kernel-side half of
 * ridge::GemmConfig (include/ridge/config.h:18-39) and the fields of
 * ridgebench::KernelVariant (bench/kernels/gemm-mma.cuh:368-383).
 *   BM, BN   output tile (64, 128 or 256 each)
 *   BK       K depth of one pipeline stage: 32 or 64 FP16 (one 64B / 128B swizzle
 *            row) or 128 (two 128B-swizzled K atoms per TMA box; K a multiple of 64)
 *   stages   shared-memory ring depth: 2..8 accepted by ridge_config_check (where
 *            shared memory allows); the registered table holds 2..6
 *   warps    epilogue warps draining TMEM (4 or 8); the CTA adds one TMA
 *            producer warp and one MMA-issuer warp
 *   groupM   grouped-M launch order width (gemm-mma.cuh:158-178); 1 = row-major
 *   cta_group 1 = one CTA per tile; 2 = BM=256 tile computed by a 2-CTA cluster
 *            with cta_group::2 MMAs (each CTA holds 128 rows). 0 = default
 *            (2 for BM=256, else 1).
 *   split_k  0 = automatic split-K tail: when the tiles leave the last round of
 *            the persistent grid partly idle, that round's tiles are split along
 *            K over the idle units and reduced through an FP32 workspace;
 *            1 = never split (every tile is computed whole by one unit).
 */
typedef struct ridge_tile_config {
    int32_t BM, BN, BK;
    int32_t stages;
    int32_t warps;
    int32_t groupM;
    int32_t cta_group;
    int32_t split_k;
} ridge_tile_config;

/*
 * Compile- and launch-time facts of one registered variant, the analogue of
 * KernelVariant's smemBytes/threads/regsPerThread (gemm-mma.cuh:368-383).
 */
typedef struct ridge_variant_info {
    ridge_tile_config cfg;
    int32_t smem_bytes;      /* dynamic shared memory per CTA */
    int32_t threads;         /* threads per CTA */
    int32_t regs_per_thread; /* from the compiled kernel (cudaFuncGetAttributes); 0 if no GPU */
    int32_t cluster_size;    /* CTAs per cluster (1 or 2) */
    int32_t tmem_cols;       /* Tensor Memory columns allocated per CTA */
    int32_t acc_buffers;     /* TMEM accumulators (2 = epilogue overlaps next tile) */
    char kernel_name[96];    /* name carrying the template args, for ncu -k regex */
} ridge_variant_info;

/* Number of registered variants (replaces ridgebench::numVariants, gemm-mma.cu:121-123). */
int ridge_num_variants(void);

/* Variant i (replaces ridgebench::variant, gemm-mma.cu:125-127). RIDGE_ERANGE if out of range. */
int ridge_variant(int index, ridge_variant_info* out);

/* Prints the variant table to stdout (replaces printVariantTable, gemm-mma.cu:132-141). */
void ridge_print_variant_table(void);

/*
 * Validates a tile config against the hardware limits (227 KB shared memory per
 * CTA, 512 TMEM columns, supported BM/BN/BK/warps/stages). RIDGE_OK or RIDGE_EINVAL.
 * Fills *info when non-NULL.
 */
int ridge_config_check(const ridge_tile_config* cfg, ridge_variant_info* info);

/*
 * Whether `cfg` can run M x N x K with the given leading dimensions. Tiles need
 * not divide the shape (M/N/K tails are handled), but TMA needs lda and ldb to be
 * multiples of 8 elements and ldc must be >= N. RIDGE_OK or RIDGE_EINVAL.
 * (Replaces the caller-side divisibility skip, measure.cu:244-248.)
 */
int ridge_config_valid_for_shape(const ridge_tile_config* cfg, int64_t M, int64_t N, int64_t K,
                                 int64_t lda, int64_t ldb, int64_t ldc);

/* ---------------------------------------------------------------- the GEMM */

/*
 * C[M,N] = A[M,K] * B[K,N], FP16 in, FP32 accumulate, FP16 out.
 *   A  device pointer, row-major M x K, leading dimension lda (>= K)
 *   B  device pointer, column-major K x N (stored N x K), leading dimension ldb (>= K)
 *   C  device pointer, row-major M x N, leading dimension ldc (>= N)
 * A and B must be 16-byte aligned. Asynchronous on `stream`.
 * Replaces KernelVariant::launch, cudaError_t(const half*, const half*, float*,
 * int, int, int, cudaStream_t) (gemm-mma.cuh:382; gemm-mma.cu:19-43).
 */
int ridge_gemm_launch(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                      int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                      void* stream);

/*
 * Device workspace (bytes) a launch of `cfg` on M x N x K needs on the current
 * device for its split-K tail; 0 when the launch does not split. Deterministic
 * for a given config, shape and device.
 */
int ridge_gemm_workspace_size(const ridge_tile_config* cfg, int64_t M, int64_t N, int64_t K,
                              int64_t* bytes);

/*
 * ridge_gemm_launch with a caller-owned workspace of at least
 * ridge_gemm_workspace_size bytes (256-byte aligned). Its first 64 KB are the
 * split-K counter area, which must be zero before the first launch (e.g.
 * cudaMemset once); every launch leaves it zero again, so one workspace can
 * serve any sequence of configs and shapes. Launches that share one workspace
 * must be ordered (one stream); launches with separate workspaces may overlap
 * freely (a split tile is reduced by whichever split arrives last, and no
 * CTA waits on another).
 * ridge_gemm_launch itself keeps such a workspace per device and stream.
 */
int ridge_gemm_launch_ws(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                         int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                         void* workspace, int64_t workspace_bytes, void* stream);

/*
 * ridge_gemm_launch for callers that must not allocate device memory (code
 * running inside a pool or arena owned by its host framework, or on a path
 * where cudaMalloc is forbidden because it synchronises the device). No
 * counterpart in the reference. Instead of allocating a split-K workspace it
 * uses one fixed scratch array inside this library's device image,
 * ridge_gemm_noalloc_scratch_bytes() (16 MiB) on every GPU that loads the
 * library, held until the process exits. A launch whose split-K tail would
 * need more returns RIDGE_ENOSCRATCH (use ridge_gemm_launch or
 * ridge_gemm_launch_ws, or a config with split_k = 1). The first call on a
 * device resolves the array's device address and clears its counter area;
 * make that first call before any stream capture. All calls on a device share
 * the array, so calls that can overlap on the GPU (different streams without
 * ordering) race; order them on one stream. Never allocates or frees memory.
 */
int ridge_gemm_launch_noalloc(const ridge_tile_config* cfg, const void* A, const void* B,
                              void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                              int64_t ldc, void* stream);

/*
 * Self-test of the bounded device waits (no counterpart in the reference):
 * launches one thread that waits, through the GEMM pipeline's own bounded
 * mbarrier wait, on a barrier nothing completes, with a limit of limit_ns
 * (1 ms .. 2 s) instead of the GEMM's 2 s. The wait expires, the kernel raises
 * its abort flag, records code 6 in the device error word and returns; the
 * context stays usable. *code receives the error word read back (6 expected),
 * *waited_ns how long the wait ran. Clears the error word before and after.
 * Synchronises the device. RIDGE_EDEVICE if the wait did not give up.
 */
int ridge_selftest_wait_timeout(int64_t limit_ns, int32_t* code, int64_t* waited_ns);

/*
 * Self-test of the recovery path (no counterpart in the reference): leaves the
 * current device in the state a GEMM that gave up mid-launch can leave behind
 * -- every byte of the split-K counter areas the library owns (its cached
 * workspaces and the no-allocation scratch, where set up) set to `byte`
 * (1..255) and the device error word set to code 7 -- without running a
 * kernel. ridge_device_error(1, ...) must then restore a state in which split
 * launches are correct again. Synchronises the device.
 */
int ridge_selftest_stale_counters(int32_t byte);

/* Size in bytes of ridge_gemm_launch_noalloc's fixed per-device scratch. No counterpart in
 * the reference. */
int64_t ridge_gemm_noalloc_scratch_bytes(void);

/*
 * End-to-end GEMM on HOST buffers: C = A * B^T with A (M x lda), B (N x ldb),
 * C (M x ldc) all FP16 in host memory; pitches need not be multiples of 8.
 * Replaces the host-side sequence of the reference's harness (copy A and B in,
 * KernelVariant::launch, copy C out: bench/measure.cu:121-150 and
 * check-gemm.cu:206-246) with one call that pipelines the copies against the
 * kernel: M is cut into `panels` row panels (0 = about 4), B and then each A
 * panel go over on an internal copy stream, each panel's launch runs on
 * `stream` as soon as its A panel has landed, and each finished C panel comes
 * back on a second internal stream while later panels are still arriving.
 * Returns after enqueueing; `stream` is ordered after the last C copy, so a
 * stream synchronise makes C valid. Page-locked host buffers give the overlap
 * (pageable ones work, serialised by the driver). Device staging buffers are
 * kept per device and grown on demand; growing frees the old ones, which
 * waits for the device. Calls on one device are ordered on the GPU.
 */
int ridge_gemm_host(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                    int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                    int32_t panels, void* stream);

/*
 * ridge_gemm_launch that also stores every C tile into num_peers (<= 7) other
 * M x N buffers with the same pitch ldc, typically copies of C in other GPUs'
 * memory mapped into this process (ridge_ipc_open): the tile goes out once
 * per destination from the same shared-memory staging, as part of the
 * epilogue, so the copies overlap the math. Every destination must be
 * 16-byte aligned with ldc a multiple of 8 (the TMA-store epilogue).
 * No counterpart in the reference (single GPU); the building block of
 * ridge_gemm_sharded_p2p.
 */
int ridge_gemm_launch_multi(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                            int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                            int64_t ldc, void* const* peer_c, int32_t num_peers, void* stream);

/* Same, addressing the variant by its table index. */
int ridge_gemm_launch_variant(int index, const void* A, const void* B, void* C, int64_t M,
                              int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                              void* stream);

/*
 * Reads (and, when clear != 0, resets) the device-side error word of the
 * current device after synchronising it. *code = 0 when no kernel timed out.
 * Clearing a non-zero word also zeroes the split-K counter areas of every
 * workspace the library owns on the device (the cached ones and the
 * no-allocation scratch), which a kernel that gave up may have left non-zero;
 * caller-owned workspaces (ridge_gemm_launch_ws) are the caller's to re-zero.
 * Returns RIDGE_OK, or a CUDA error from the synchronisation.
 */
int ridge_device_error(int clear, int32_t* code);

/* ---------------------------------------------------------------- synthetic inputs */

/*
 * Fills n FP16 values on the device with the reference's deterministic LCG
 * (s = s*1664525 + 1013904223; draw = ((s>>16)&0x7fff)/32767), bit-identical to
 * the host fill fillDeterministic (bench/check-gemm.cu:139-145) it replaces.
 * range 0: value = draw - 0.5 (the reference's U(-0.5,0.5));
 * range 1: value = 2*draw - 1 (U(-1,1), the benchmark inputs).
 * *state is the seed on entry and the LCG state after n draws on return, so
 * consecutive calls continue one stream (A then B from seed 0).
 */
int ridge_fill_lcg(void* out_f16, int64_t n, uint32_t* state, int32_t range, void* stream);

/* ---------------------------------------------------------------- the model */

/*
 * Hardware constants for the cost model (replaces ridge::HardwareModel,
 * include/ridge/hardware.h:9-54). Fields marked [CAL] are measured by the
 * sm_100a calibration microbenchmarks (include/ridge_b200_calibrate.h); the
 * built-in ridge_hw_b200() holds datasheet-derived placeholders.
 */
typedef struct ridge_hw {
    char name[64];
    int32_t num_sms;
    double clock_hz;                 /* [CAL] SM clock under sustained tensor load (power cap) */
    double umma_cycles_128x256;      /* [CAL] SM cycles per 128x256x16 FP16 tcgen05.mma */
    double umma_m64_ratio;           /* [CAL] cycles of a 64xNx16 MMA / cycles of 128xNx16 */
    double smem_bytes_per_cycle;     /* [CAL] operand bytes/cycle/SM the tensor core reads */
    double smem_mma_overlap;         /* [CAL] 1: operand reads overlap the MMA (max); 0: in series (sum) */
    double l2_bytes_per_sec;         /* [CAL] aggregate TMA L2 -> SM fill bandwidth */
    double hbm_bytes_per_sec;        /* [CAL] whole-GPU HBM read bandwidth (TMA streaming) */
    double tma_box_cycles;           /* [CAL] cycles per TMA box per issuing thread, 4 threads issuing */
    double tma_box2_ratio;           /* [CAL] cost of a two-atom (BK=128) box / a one-atom box */
    double tma_box32_ratio;          /* [CAL] cost of a 64-byte-wide (BK=32) box / a one-atom box */
    double pipeline_efficiency;      /* [CAL] steady-state mainloop rate / ideal, from a calibration GEMM */
    double tile_overhead_cycles;     /* [CAL] per-tile turnover beyond the drain, one-CTA tiles */
    double pair_tile_overhead_cycles;/* [CAL] the same for 2-CTA pair tiles */
    double c_write_bytes_per_sec;    /* [CAL] epilogue write rate of a C far larger than L2 */
    double epi_bytes_per_cycle_w4;   /* [CAL] C bytes/cycle/SM drained by 4 epilogue warps */
    double epi_bytes_per_cycle_w8;   /* [CAL] same with 8 epilogue warps */
    double tma_latency_cycles;       /* [CAL] issue -> arrival latency of one stage load */
    double tma_latency_hbm_cycles;   /* [CAL] the same when the operands stream from DRAM */
    double launch_overhead_sec;      /* [CAL] fixed cost of one launch (launch + fill + drain) */
    double l2_bytes;                 /* L2 capacity */
    int32_t smem_bytes_per_sm;
    int32_t tmem_cols_per_sm;
    int32_t max_ctas_per_sm;
    int32_t calibrated;              /* 1 when the [CAL] fields came from a calibration file */
} ridge_hw;

/* One GEMM + tile config for the model (replaces ridge::GemmConfig, config.h:18-39). */
typedef struct ridge_gemm_config {
    int64_t M, N, K;
    ridge_tile_config tile;
} ridge_gemm_config;

/* Bottleneck labels (replaces ridge::Bottleneck, include/ridge/prediction.h:10). */
enum {
    RIDGE_BOTTLENECK_TENSOR_CORE = 0,
    RIDGE_BOTTLENECK_SMEM = 1,
    RIDGE_BOTTLENECK_HBM = 2,
    RIDGE_BOTTLENECK_OCCUPANCY = 3,
    RIDGE_BOTTLENECK_WAVES = 4,
    RIDGE_BOTTLENECK_ENVELOPE = 5,
    RIDGE_BOTTLENECK_DOES_NOT_FIT = 6,
    RIDGE_BOTTLENECK_EPILOGUE = 7,  /* exposed TMEM -> global drain (new on B200) */
    RIDGE_BOTTLENECK_L2 = 8         /* TMA fill from L2 (new on B200) */
};

/* Model output (replaces ridge::Prediction, prediction.h:15-49). Times are
 * SM cycles unless named _sec; efficiencies are in (0, 1]. */
typedef struct ridge_prediction {
    double predicted_tflops;
    int32_t bottleneck;
    double compute_tflops;       /* ceiling from the on-SM pipeline after all deratings */
    double hbm_tflops;           /* HBM roofline ceiling for the modelled DRAM traffic */
    double peak_tensor_tflops;   /* dense tensor peak at this clock */
    double smem_efficiency;      /* t_mma / t_step: operand feed vs tensor issue */
    double l2_efficiency;        /* t_step / max(t_step, t_l2): TMA fill from L2 */
    double occ_factor;           /* t_kblock / pipeline period: latency hidden by `stages` */
    double wave_efficiency;      /* tiles / (rounds * tile slots) */
    double envelope_efficiency;  /* steady-state share: 1 - (prologue + launch) / total */
    double epilogue_efficiency;  /* mainloop share of the per-tile period (epilogue exposure) */
    double arithmetic_intensity; /* FLOP per modelled DRAM byte */
    double dram_bytes;           /* modelled DRAM traffic, grouped-M order and L2 reuse included */
    double total_tiles;
    double tile_slots;           /* concurrently resident CTAs (or CTA pairs) */
    double waves_exact;          /* total_tiles / tile_slots */
    double k_blocks;             /* ceil(K / BK) */
    double t_mma_cycles;         /* per K-block */
    double t_smem_cycles;        /* per K-block */
    double t_l2_cycles;          /* per K-block */
    double t_step_cycles;        /* per K-block, after operand-feed overlap */
    double t_period_cycles;      /* per K-block, after latency hiding */
    double t_epilogue_cycles;    /* per tile */
    double t_tile_cycles;        /* per tile, epilogue overlap included */
    double t_prologue_cycles;    /* first-fill latency per CTA */
    double predicted_seconds;
    int32_t ctas_per_sm;
    int32_t acc_buffers;
} ridge_prediction;

/* Label text, e.g. "TENSOR_CORE" (replaces ridge::toString, model.cpp:9-20). */
const char* ridge_bottleneck_string(int32_t bottleneck);

/* Built-in B200 datasheet placeholders (replaces HardwareModel::a100(), hardware.cpp:19-34). */
int ridge_hw_b200(ridge_hw* out);

/*
 * Loads a calibrated model from flat JSON, all or nothing (replaces
 * HardwareModel::loadFromJson, hardware.cpp:149-200). On failure *out is
 * untouched and errbuf (if non-NULL) receives the reason.
 */
int ridge_hw_load_json(const char* path, ridge_hw* out, char* errbuf, int32_t errlen);

/* Predicts throughput and the binding resource (replaces ridge::predict, model.h:10). */
int ridge_predict(const ridge_gemm_config* cfg, const ridge_hw* hw, ridge_prediction* out);

/* ---------------------------------------------------------------- autotune */

/* One measured candidate. */
typedef struct ridge_tune_entry {
    ridge_tile_config tile;
    double predicted_tflops;
    double measured_tflops;   /* 0 when not benchmarked or failed */
    int32_t device;           /* device that measured it, -1 if none */
    int32_t status;           /* RIDGE_OK or the launch error */
} ridge_tune_entry;

/* Per-shape autotune result. */
typedef struct ridge_tune_result {
    int64_t M, N, K;
    ridge_tile_config best;   /* fastest measured among the benchmarked candidates */
    double best_tflops;
    int32_t benchmarked;      /* candidates timed */
    int32_t candidates;       /* valid candidates ranked by the model */
} ridge_tune_result;

/*
 * Model-pruned empirical autotune (replaces tools/ridge-autotune.py:94-112,
 * which only simulated the benchmark from a CSV): for each shape rank every
 * valid registered variant by ridge_predict, benchmark the top k on the GPUs in
 * `devices` (a host work queue, one worker thread per device, no collective),
 * keep the fastest. k <= 0 benchmarks every candidate (the exhaustive sweep).
 * `entries` (optional, capacity `entries_cap` per shape, row-major
 * [shape][entry]) receives every candidate in model-rank order.
 * Each candidate is timed by ridge_time_gemm_cold (warmup_iters launches, then
 * at least timed_iters L2-flushed launches; a 256 MiB flush buffer per
 * device), the discipline of the headline benchmark.
 * A device that cannot be set up takes no part; a device that hits a CUDA
 * error mid-sweep hands its candidate back to the queue for the other
 * devices and retires. Returns RIDGE_OK when every selected candidate was
 * measured (a candidate whose own launch timed out on the device is measured,
 * with status RIDGE_EDEVICE), RIDGE_EDEVICE when some were left undone.
 */
int ridge_autotune(const int64_t* shapes_mnk, int32_t num_shapes, int32_t k,
                   const int32_t* devices, int32_t num_devices, const ridge_hw* hw,
                   int32_t warmup_iters, int32_t timed_iters, ridge_tune_result* results,
                   ridge_tune_entry* entries, int32_t entries_cap);

/*
 * Times one config on caller-owned device buffers with CUDA events on
 * `stream`: `warmup` launches, a short probe, then three adaptive runs of at
 * least `iters` back-to-back launches (about 20 ms of work each, at most
 * max(400, iters)). *ms_per_launch = mean launch time of the fastest run. Synchronises the stream. Replaces
 * timeTflops (bench/measure.cu:121-150).
 */
int ridge_time_gemm(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                    int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                    int32_t warmup, int32_t iters, void* stream, double* ms_per_launch);

/*
 * Cold timing, the headline benchmark's discipline (no counterpart in the
 * reference, whose measure.cu times warm back-to-back launches): `warmup`
 * launches, then launches each preceded by overwriting `flush_bytes` of the
 * caller's `flush` buffer (make it larger than L2, e.g. 256 MiB, so A and B
 * come from DRAM), with CUDA events around the launch alone: at least `iters`
 * of them, more (up to 200) until about 2 ms of kernel time is sampled.
 * *ms_per_launch = the mean of the middle 60% of those launch times (single
 * event times are quantised to about 1 us). Allocates nothing. Synchronises
 * the stream.
 */
int ridge_time_gemm_cold(const ridge_tile_config* cfg, const void* A, const void* B, void* C,
                         int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                         void* flush, int64_t flush_bytes, int32_t warmup, int32_t iters,
                         void* stream, double* ms_per_launch);

/*
 * Self-test of the autotuner's work queue on the host (no GPU, no counterpart
 * in the reference): num_jobs fake jobs over num_devices fake devices, each
 * job a short sleep (12 ms on slow_device, 2 ms elsewhere). lost_device fails
 * after completing lost_after jobs, handing its current job back (lost_after
 * < 0: it fails its set-up and takes no job). job_device[j] receives the
 * device that completed job j (-1 if none), jobs_per_device[d] the jobs device
 * d completed. Returns what ridge_autotune would: RIDGE_OK when every job was
 * done, RIDGE_EDEVICE otherwise. Pass -1 for no lost / no slow device.
 */
int ridge_farm_selftest(int32_t num_jobs, int32_t num_devices, int32_t lost_device,
                        int32_t lost_after, int32_t slow_device, int32_t* job_device,
                        int32_t* jobs_per_device);

/* ---------------------------------------------------------------- N-slab sharding */

/*
 * Rank `rank` of `nranks` computes its N-column slab of C = A * B for a GEMM
 * split by N-column slabs of B with A replicated: B_slab points at rows
 * [n0, n0 + n_slab) of the N x K storage of B, C_slab is M x n_slab row-major
 * (ldc). The slab bounds come from ridge_slab_bounds. Purely local: no
 * collective; ridge_gemm_sharded below adds the optional all-gather.
 */
int ridge_slab_bounds(int64_t N, int32_t nranks, int32_t rank, int64_t align, int64_t* n0,
                      int64_t* n_slab);
/* (Slab width = ceil(N / nranks) rounded up to `align`; the last slab may be
 * narrower or empty.) */

/*
 * Re-lays out slab-major C (nranks slabs, slab r = M x slab_cols row-major,
 * contiguous, holding C[:, r*slab_cols : (r+1)*slab_cols]) into row-major
 * M x N C (ldc). Columns at or beyond N (padding of the last slab) are
 * dropped. Asynchronous on `stream`.
 */
int ridge_slabs_to_rowmajor(const void* slabs, void* C, int64_t M, int64_t N, int32_t nranks,
                            int64_t slab_cols, int64_t ldc, void* stream);

/*
 * One rank's part of the N-slab GEMM, with the optional gather of the full C
 * (no counterpart in the single-GPU reference; the C-ABI shape named for the
 * sharded configuration). A (M x lda) is replicated; B_slab is this rank's
 * rows [n0, n0 + n_slab) of B's N x K storage (ldb), n0 / n_slab from
 * ridge_slab_bounds(N, nranks, rank, 256). C_slab receives this rank's slab
 * as M x slab_cols row-major, slab_cols = ridge_slab_bounds' width for rank 0
 * (columns past n_slab are scratch). With gather_full_c != 0, the slabs of
 * all ranks are all-gathered over `nccl_comm` (an ncclComm_t of nranks ranks,
 * this rank = `rank`) into `slabs` (nranks x M x slab_cols FP16) and re-laid
 * out into C_full (M x N, ldc_full) on every rank (one rank: C_slab is
 * copied to C_full, no communicator needed). Everything is enqueued on
 * `stream`. NCCL is resolved at run time from the libnccl.so.2 already loaded
 * in the process (else loaded); RIDGE_ECOMM if it is absent or the collective
 * fails. Buffers are the caller's.
 */
int ridge_gemm_sharded(const ridge_tile_config* cfg, const void* A, const void* B_slab,
                       void* C_slab, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                       int32_t nranks, int32_t rank, int32_t gather_full_c, void* nccl_comm,
                       void* slabs, void* C_full, int64_t ldc_full, void* stream);

/*
 * The N-slab GEMM with the gather fused into the epilogue: rank `rank` of
 * `nranks` (<= 8) computes its slab C[:, n0:n0+n_slab] and its epilogue stores
 * every tile straight into all ranks' full M x N C buffers (c_full[r] for
 * r = 0..nranks-1, this rank's own included, all with pitch ldc), over NVLink
 * for the peers. c_full holds device pointers valid in this process (peers'
 * from ridge_ipc_open). When nccl_comm is given, the call is fenced on both
 * sides by a one-element all-reduce on `stream`: the one before the kernel is
 * an entry barrier (no rank starts writing into the others' C until every
 * rank has reached this call in its stream order, so work a rank enqueued on
 * `stream` before the call -- reading its previous C, say -- is finished
 * first), the one after it a completion barrier (when it is done on this
 * rank, every rank's tiles have landed in this rank's C). A rank that reads
 * its C on another stream or on the host must finish doing so before it makes
 * the next call. Without nccl_comm the caller provides both fences. No
 * counterpart in the reference; replaces ridge_gemm_sharded's NCCL
 * all-gather + re-layout with copies that overlap the GEMM.
 */
int ridge_gemm_sharded_p2p(const ridge_tile_config* cfg, const void* A, const void* B_slab,
                           int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                           int32_t nranks, int32_t rank, void* const* c_full, int64_t ldc,
                           void* nccl_comm, void* stream);

/*
 * Device memory another process on this node can map (CUDA IPC), for the
 * peer copies of C. ridge_device_alloc / ridge_device_free wrap cudaMalloc /
 * cudaFree (an IPC handle names a whole allocation); ridge_ipc_export writes
 * the handle (ridge_ipc_handle_bytes() bytes) of such an allocation;
 * ridge_ipc_open maps another process's handle here (peer access enabled);
 * ridge_ipc_close unmaps it.
 */
int64_t ridge_ipc_handle_bytes(void);
int ridge_device_alloc(int64_t bytes, void** ptr);
int ridge_device_free(void* ptr);
int ridge_ipc_export(const void* base, void* handle);
int ridge_ipc_open(const void* handle, void** ptr);
int ridge_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* RIDGE_B200_H */
