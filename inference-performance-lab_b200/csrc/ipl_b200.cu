// C ABI of the library (declared in include/ipl_b200.h): argument checks, kernel selection and
// launch. One translation unit holds every kernel so that the per-device fault word is a single
// symbol without relocatable device code.
#include "ipl_b200.h"

#include "fused_add_rms_norm.cuh"
#include "silu_and_mul.cuh"

#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace ipl {
namespace {

thread_local char t_last_error[512] = "";

ipl_status fail(ipl_status status, const char* fmt, ...) {
    va_list args;
    va_start(args, fmt);
    std::vsnprintf(t_last_error, sizeof(t_last_error), fmt, args);
    va_end(args);
    return status;
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    std::atomic<int> sm_count{0};
    std::atomic<int> max_smem_optin{0};
    std::atomic<uint32_t> smem_configured{0};  // bit per kernel instance given the shared-memory opt-in
};
DeviceInfo g_devices[kMaxDevices];

// SM count and opt-in shared memory of the current device, queried once per device.
ipl_status current_device(int* device, DeviceInfo** info) {
    cudaError_t err = cudaGetDevice(device);
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "failed to query the current CUDA device: %s", cudaGetErrorString(err));
    }
    if (*device < 0 || *device >= kMaxDevices) {
        return fail(IPL_ERROR_CUDA, "CUDA device index %d is out of range", *device);
    }
    DeviceInfo& d = g_devices[*device];
    if (d.sm_count.load(std::memory_order_acquire) == 0) {
        int sms = 0, smem = 0;
        err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, *device);
        if (err == cudaSuccess) {
            err = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, *device);
        }
        if (err != cudaSuccess) {
            return fail(IPL_ERROR_CUDA, "failed to read CUDA device properties: %s", cudaGetErrorString(err));
        }
        d.max_smem_optin.store(smem, std::memory_order_relaxed);
        d.sm_count.store(sms, std::memory_order_release);
    }
    *info = &d;
    return IPL_SUCCESS;
}

// Limits the plan queries plan with: the current device's, as the launch path reads them, so a
// query names the kernel a call on this device launches. Where no device can be queried (a host
// without a GPU), a B200's: 148 SMs, 232448 bytes of opt-in shared memory per block. Leaves
// neither this thread's last-error message nor CUDA's last error changed.
void plan_limits(int* sm_count, int* smem_limit) {
    char saved[sizeof(t_last_error)];
    std::memcpy(saved, t_last_error, sizeof(saved));
    int device = 0;
    DeviceInfo* info = nullptr;
    if (current_device(&device, &info) == IPL_SUCCESS) {
        *sm_count = info->sm_count.load(std::memory_order_relaxed);
        *smem_limit = info->max_smem_optin.load(std::memory_order_relaxed);
        return;
    }
    std::memcpy(t_last_error, saved, sizeof(saved));
    (void)cudaGetLastError();
    *sm_count = 148;
    *smem_limit = 232448;
}

template <typename Kernel, typename... Args>
cudaError_t launch(Kernel kernel, unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                   Args... args) {
    // Programmatic stream serialisation: the kernel may be scheduled while the previous kernel
    // in the stream drains; it orders its own global reads with griddepcontrol.wait.
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(block);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, args...);
}

// The same with the grid in thread-block clusters of `cluster` CTAs along x (grid a multiple of it).
template <typename Kernel, typename... Args>
cudaError_t launch_clustered(Kernel kernel, unsigned grid, unsigned cluster, unsigned block, size_t smem,
                             cudaStream_t stream, Args... args) {
    cudaLaunchAttribute attribute[2];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    attribute[1].id = cudaLaunchAttributeClusterDimension;
    attribute[1].val.clusterDim.x = cluster;
    attribute[1].val.clusterDim.y = 1;
    attribute[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(block);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    config.attrs = attribute;
    config.numAttrs = 2;
    return cudaLaunchKernelEx(&config, kernel, args...);
}

// ------------------------------------------------------------------------------------------
// add + RMSNorm / RMSNorm planning

enum class RmsFamily {
    kNone, kStaged, kWarpRow, kCtaRow, kStash, kStashV8, kShifted, kShiftedV8, kCluster, kRowwiseCached, kRowwiseTwoPass
};

struct RmsPlan {
    RmsFamily family = RmsFamily::kNone;
    int warps_per_row = 0;  // staged kernels: 1, 2, 4, 8 or 16
    int chunks_per_lane = 0;  // warp-, CTA-per-row and stash kernels: 16-byte chunks per thread (1, 2, 4 or 8)
    unsigned threads = 0;     // CTA-per-row and stash kernels: block size
    bool capped = false;      // stash kernel, rows of 16384 < H <= 20480: the 96-register instance
    int phase = 0;            // shifted kernel: elements from the 16-byte block to each row
    int64_t lookahead = 0;       // stash and shifted kernels: one resident wave, when rows exceed it
    int64_t lookahead_ctas = 0;  // ... and how many CTAs look one wave ahead
    int cluster = 0;             // cluster kernel: CTAs a row (2..8) ...
    int cluster_slice = 0;       // ... and the 16-byte chunks each owns
    unsigned grid = 0;
    size_t smem = 0;
    StagedParams staged = {};
};

// Kernel names as reported by the plan queries (static strings).
const char* rms_kernel_name(const RmsPlan& plan, int mode) {
    static const char* const kStagedNames[2][5] = {  // bf16 outputs only
        {"rmsnorm_staged_kernel<1>", "rmsnorm_staged_kernel<2>", "rmsnorm_staged_kernel<4>",
         "rmsnorm_staged_kernel<8>", "rmsnorm_staged_kernel<16>"},
        {"rmsnorm_staged_kernel<1, plain>", "rmsnorm_staged_kernel<2, plain>", "rmsnorm_staged_kernel<4, plain>",
         "rmsnorm_staged_kernel<8, plain>", "rmsnorm_staged_kernel<16, plain>"}};
    static const char* const kWarpNames[3][3] = {
        {"rmsnorm_warp_kernel<1>", "rmsnorm_warp_kernel<2>", "rmsnorm_warp_kernel<4>"},
        {"rmsnorm_warp_kernel<1, plain>", "rmsnorm_warp_kernel<2, plain>", "rmsnorm_warp_kernel<4, plain>"},
        {"rmsnorm_warp_kernel<1, fp8>", "rmsnorm_warp_kernel<2, fp8>", "rmsnorm_warp_kernel<4, fp8>"}};
    static const char* const kCtaNames[3][3] = {
        {"rmsnorm_cta_kernel<1>", "rmsnorm_cta_kernel<2>", "rmsnorm_cta_kernel<4>"},
        {"rmsnorm_cta_kernel<1, plain>", "rmsnorm_cta_kernel<2, plain>", "rmsnorm_cta_kernel<4, plain>"},
        {"rmsnorm_cta_kernel<1, fp8>", "rmsnorm_cta_kernel<2, fp8>", "rmsnorm_cta_kernel<4, fp8>"}};
    static const char* const kStashNames[3] = {"rmsnorm_stash_kernel<4>", "rmsnorm_stash_kernel<4, plain>",
                                               "rmsnorm_stash_kernel<4, fp8>"};
    static const char* const kStashWideNames[3] = {"rmsnorm_stash_kernel<8>", "rmsnorm_stash_kernel<8, plain>",
                                                   "rmsnorm_stash_kernel<8, fp8>"};
    static const char* const kClusterNames[3][3] = {
        {"rmsnorm_cluster_kernel<1>", "rmsnorm_cluster_kernel<2>", "rmsnorm_cluster_kernel<4>"},
        {"rmsnorm_cluster_kernel<1, plain>", "rmsnorm_cluster_kernel<2, plain>", "rmsnorm_cluster_kernel<4, plain>"},
        {"rmsnorm_cluster_kernel<1, fp8>", "rmsnorm_cluster_kernel<2, fp8>", "rmsnorm_cluster_kernel<4, fp8>"}};
    static const char* const kRowwiseNames[3][2] = {
        {"rmsnorm_rowwise_kernel<cached>", "rmsnorm_rowwise_kernel<two-pass>"},
        {"rmsnorm_rowwise_kernel<cached, plain>", "rmsnorm_rowwise_kernel<two-pass, plain>"},
        {"rmsnorm_rowwise_kernel<cached, fp8>", "rmsnorm_rowwise_kernel<two-pass, fp8>"}};
    int i = 0;
    switch (plan.family) {
        case RmsFamily::kNone: return "none";
        case RmsFamily::kStaged:
            while ((1 << i) < plan.warps_per_row) ++i;
            return mode == kModeFusedFp8 ? "invalid" : kStagedNames[mode][i];
        case RmsFamily::kWarpRow:
            while ((1 << i) < plan.chunks_per_lane) ++i;
            return kWarpNames[mode][i];
        case RmsFamily::kCtaRow:
            while ((1 << i) < plan.chunks_per_lane) ++i;
            return kCtaNames[mode][i];
        case RmsFamily::kStash:
            // Eight chunks a thread: rows longer than 16384 (capped: up to 20480, more than 256
            // rows, add+RMSNorm and fp8) and plain RMSNorm of many long rows.
            if (plan.capped) return mode == kModeFusedFp8 ? "rmsnorm_stash_kernel<8, fp8, capped>" : "rmsnorm_stash_kernel<8, capped>";
            return plan.chunks_per_lane == kStashWideChunks ? kStashWideNames[mode] : kStashNames[mode];
        case RmsFamily::kShifted: {
            static const char* const kShiftedNames[2][7] = {
                {"rmsnorm_shifted_kernel<1>", "rmsnorm_shifted_kernel<2>", "rmsnorm_shifted_kernel<3>",
                 "rmsnorm_shifted_kernel<4>", "rmsnorm_shifted_kernel<5>", "rmsnorm_shifted_kernel<6>",
                 "rmsnorm_shifted_kernel<7>"},
                {"rmsnorm_shifted_kernel<1, plain>", "rmsnorm_shifted_kernel<2, plain>",
                 "rmsnorm_shifted_kernel<3, plain>", "rmsnorm_shifted_kernel<4, plain>",
                 "rmsnorm_shifted_kernel<5, plain>", "rmsnorm_shifted_kernel<6, plain>",
                 "rmsnorm_shifted_kernel<7, plain>"}};
            return mode == kModeFusedFp8 ? "invalid" : kShiftedNames[mode][plan.phase - 1];
        }
        case RmsFamily::kCluster:
            while ((1 << i) < plan.chunks_per_lane) ++i;
            return kClusterNames[mode][i];
        case RmsFamily::kStashV8: {
            return mode == kModeFused ? "rmsnorm_stash_v8_kernel" : mode == kModeFusedFp8 ? "rmsnorm_stash_v8_kernel<fp8>"
                                                                                        : "invalid";
        }
        case RmsFamily::kShiftedV8: {
            static const char* const kShiftedV8Names[7] = {
                "rmsnorm_shifted_v8_kernel<1>", "rmsnorm_shifted_v8_kernel<2>", "rmsnorm_shifted_v8_kernel<3>",
                "rmsnorm_shifted_v8_kernel<4>", "rmsnorm_shifted_v8_kernel<5>", "rmsnorm_shifted_v8_kernel<6>",
                "rmsnorm_shifted_v8_kernel<7>"};
            return mode == kModeFused ? kShiftedV8Names[plan.phase - 1] : "invalid";
        }
        case RmsFamily::kRowwiseCached: return kRowwiseNames[mode][0];
        case RmsFamily::kRowwiseTwoPass: return kRowwiseNames[mode][1];
    }
    return "invalid";
}

// x, weight and (fused op) residual / (plain op) out: the three row pointers of a call.
ipl_status check_rms_args(const void* x, const void* other, const void* weight, int64_t rows, int64_t hidden,
                          double epsilon, bool residual) {
    if (rows < 0) return fail(IPL_ERROR_INVALID_VALUE, "number of rows must be non-negative");
    if (hidden <= 0) return fail(IPL_ERROR_INVALID_VALUE, "x must have a non-empty final dimension");
    if (!(epsilon > 0.0)) return fail(IPL_ERROR_INVALID_VALUE, "epsilon must be positive");
    if (hidden > INT_MAX) return fail(IPL_ERROR_TOO_LARGE, "hidden dimension is too large");
    if (rows > INT_MAX) return fail(IPL_ERROR_TOO_LARGE, "number of rows is too large");
    if (rows > 0 && (x == nullptr || other == nullptr || weight == nullptr)) {
        return fail(IPL_ERROR_INVALID_VALUE, residual ? "x, residual and weight must be non-null"
                                                      : "output, input and weight must be non-null");
    }
    const uintptr_t odd = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(other) |
                          reinterpret_cast<uintptr_t>(weight);
    if (odd & 1u) return fail(IPL_ERROR_INVALID_VALUE, "bfloat16 pointers must be 2-byte aligned");
    if (residual && rows > 0 && x == other) {
        return fail(IPL_ERROR_INVALID_VALUE, "x and residual must not alias");
    }
    return IPL_SUCCESS;
}

// CTAs of `threads` threads that the GPU holds at once when each thread may take `regs`
// registers (the cap the kernel's launch bound sets; allocation is in whole multiples of 8, which
// 64, 96 and 128 are): the register file, threads per SM and 32 CTAs per SM all bound it.
int64_t resident_ctas(int sm_count, int64_t threads, int64_t regs) {
    int64_t per_sm = kRegistersPerSm / (threads * regs);
    if (per_sm > kThreadsPerSm / threads) per_sm = kThreadsPerSm / threads;
    if (per_sm > 32) per_sm = 32;
    return static_cast<int64_t>(sm_count) * per_sm;
}

// The one-wave look-ahead of the stash and shifted kernels (prefetch_next_wave_row): every CTA
// looks ahead in a launch of up to four resident waves, the first wave only in a longer one.
constexpr int64_t kLookaheadAllWaves = 4;
void set_lookahead(RmsPlan& plan, int64_t rows, int64_t wave) {
    plan.lookahead = rows > wave ? wave : 0;
    plan.lookahead_ctas = rows > wave ? (rows <= kLookaheadAllWaves * wave ? rows : wave) : 0;
}

// The cluster kernel with `ctas` CTAs a row: each owns ceil(H / 8 / ctas) 16-byte chunks and
// stages its slice of gamma. Chunks a thread (1, 2 or 4): the most that leave the CTA at least
// 128 threads, more where 512 threads would not hold the slice. Measured against fewer chunks a
// thread over more threads: 512 x 65536 48.1 against 67.4 us, 2048 x 49152 -10 %.
void set_cluster(RmsPlan& plan, int64_t rows, int64_t hidden, int ctas) {
    const int64_t slice = (hidden / 8 + ctas - 1) / ctas;
    int per_thread = 1;
    while (per_thread < kStashChunks && (slice + 2 * per_thread - 1) / (2 * per_thread) >= 128) per_thread *= 2;
    while (per_thread < kStashChunks && (slice + per_thread - 1) / per_thread > kStashMaxThreads) per_thread *= 2;
    plan.family = RmsFamily::kCluster;
    plan.chunks_per_lane = per_thread;
    const int64_t threads = (slice + plan.chunks_per_lane - 1) / plan.chunks_per_lane;
    plan.threads = static_cast<unsigned>((threads + kWarpSize - 1) / kWarpSize * kWarpSize);
    plan.cluster = ctas;
    plan.cluster_slice = static_cast<int>(slice);
    plan.smem = static_cast<size_t>(slice) * 16u;
    plan.grid = static_cast<unsigned>(rows * ctas);
}

// CTAs a row for the cluster kernel (aligned rows, H % 8 == 0), or 0 where one CTA a row plans
// better. From cold-L2 sweeps on B200 (CUDA graph, add+RMSNorm and RMSNorm, 1-2048 rows x H
// 6144-131072, cluster sizes 2, 4 and 8 against the kernels planned before):
// * H > 32768 (up to 131072, 512 threads of four chunks in each of 8 CTAs): always, 8 CTAs a row.
//   The only other aligned kernel there is the rowwise one (2-byte accesses, the row read twice):
//   2.8-4.3x faster from 512 rows (512 x 65536 48.4 against 208 us), 9-45x for 1-64 rows;
//   8 CTAs were 1-12 % ahead of 4 at every size;
// * few long rows, where one CTA a row leaves SMs idle and each CTA's row takes long to load:
//   16384 < H <= 32768 up to 256 rows (RMSNorm 128): 1.06-2.2x against the stash kernel's
//   eight-chunk instance (8 x 32768 2.70 against 5.80 us); 8192 <= H <= 16384 up to 32 rows,
//   6144 <= H < 8192 up to 16: 1.04-1.56x against the CTA-per-row kernel (1 x 16384 2.10 against
//   3.28 us); H >= 12288 and more rows than SMs up to 256, where the CTA-per-row kernel needs a
//   second wave: 1.09-1.33x. Outside these ranges the cluster was level or up to 30 % slower;
// * cluster size: 8 CTAs for up to 16 rows; otherwise the most (8, 4, 2) that leave each CTA at
//   least 256 chunks and the launch at most 768 CTAs - the GPU starts CTAs at about one a
//   nanosecond, and a CTA of one chunk a thread costs more to start than it saves (192 x 16384:
//   4 CTAs a row 5.71 us, 8 CTAs 7.33).
int cluster_ctas_for(int64_t rows, int64_t hidden, int mode, int sm_count) {
    const int64_t chunks = hidden / 8;
    if (hidden > kStashMaxLongHidden) {
        const bool fits = chunks <= static_cast<int64_t>(kClusterMaxCtas) * kStashMaxThreads * kStashChunks;
        return fits && rows <= INT_MAX / kClusterMaxCtas ? kClusterMaxCtas : 0;
    }
    if (hidden < 6144) return 0;
    const bool use = hidden > kStashMaxHidden
                         ? rows <= (mode == kModePlain ? 128 : 256)
                         : rows <= (hidden >= 8192 ? 32 : 16) ||
                               (hidden >= 12288 && rows > sm_count && rows <= kCtaRowMaxRows);
    if (!use) return 0;
    if (rows <= 16) return kClusterMaxCtas;
    int ctas = kClusterMaxCtas;
    while (ctas > 2 && (chunks / ctas < 256 || rows * ctas > 768)) ctas /= 2;
    return ctas;
}

// Pure function of the arguments and two device limits. `other` is the residual (fused modes) or
// the output (plain mode); either must share x's offset modulo 16 bytes for the staged kernel.
// `out8` is the fp8 output of kModeFusedFp8, whose vector paths need 16-byte aligned rows
// (H % 8 == 0) and an 8-byte aligned output. `weight` matters only to the 256-bit stash kernel,
// which stages it with 16-byte copies.
RmsPlan plan_rms(const void* x, const void* other, const void* out8, const void* weight, int64_t rows,
                 int64_t hidden, int mode, int sm_count, int smem_limit) {
    RmsPlan plan;
    if (rows == 0) return plan;
    const bool residual = mode != kModePlain;
    const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
    const uintptr_t oa = reinterpret_cast<uintptr_t>(other);
    const bool fp8_vector_ok = mode != kModeFusedFp8 ||
                               (hidden % 8 == 0 && (xa & 15u) == 0 && (reinterpret_cast<uintptr_t>(out8) & 7u) == 0);
    const int chunks_max = static_cast<int>((hidden + 7) / 8 + 1);
    const int stage_bytes = (residual ? 2 : 1) * chunks_max * 16;
    const int row_phase = static_cast<int>((xa & 15u) >> 1);
    const StagedLayout fixed = staged_layout(0, stage_bytes, chunks_max);
    const int64_t room = static_cast<int64_t>(smem_limit) - fixed.total;
    int max_stages = room > 0 ? static_cast<int>(room / (stage_bytes + 2 * 8)) : 0;
    if (max_stages > kStagedMaxStages) max_stages = kStagedMaxStages;

    // Rows split over a thread-block cluster (cluster_ctas_for).
    if (hidden % 8 == 0 && ((xa | oa) & 15u) == 0 && fp8_vector_ok) {
        const int ctas = cluster_ctas_for(rows, hidden, mode, sm_count);
        if (ctas > 0) {
            set_cluster(plan, rows, hidden, ctas);
            return plan;
        }
    }
    // Add+RMSNorm (and its fp8 output) on rows of 1536 <= H <= 5120 (H % 16 == 0, x and residual
    // 32-byte aligned, weight and an fp8 output 16-byte aligned), 257-4096 of them: the stash
    // scheme with one 32-byte pair of chunks a thread (rmsnorm_stash_v8_kernel), every CTA looking
    // one resident wave ahead. Measured against the kernels below on B200 (cold L2, CUDA graph):
    // add+RMSNorm 1.02-1.21x the four-chunk stash instance (2048 x 3584 8.96 against 9.34 us,
    // 2000 x 3072 7.44 against 8.29) and the CTA-per-row kernel on its one-wave launches (300 x 3584
    // 2.72 against 3.06); the fp8 output 1.01-1.08x. Plain RMSNorm stays on the four-chunk stash
    // instance (0.96x at 2048 x 3584).
    if (mode != kModePlain && hidden % 16 == 0 && hidden >= kStashV8MinHidden && hidden <= kStashV8MaxHidden &&
        rows > kCtaRowMaxRows && rows <= kStashV8MaxRows && ((xa | oa) & 31u) == 0 &&
        (reinterpret_cast<uintptr_t>(weight) & 15u) == 0 &&
        (mode != kModeFusedFp8 || (reinterpret_cast<uintptr_t>(out8) & 15u) == 0)) {
        const int64_t threads = (hidden / 16 + kWarpSize - 1) / kWarpSize * kWarpSize;
        plan.family = RmsFamily::kStashV8;
        plan.chunks_per_lane = 2;
        plan.threads = static_cast<unsigned>(threads);
        plan.smem = static_cast<size_t>(hidden) * 2u;
        plan.grid = static_cast<unsigned>(rows);
        const int64_t wave = resident_ctas(sm_count, threads, 64);  // launch bound (512, 2): 64 registers
        plan.lookahead = rows > wave ? wave : 0;
        plan.lookahead_ctas = rows > wave ? rows : 0;  // every CTA: up to 4096 rows is a few waves
        return plan;
    }
    // Aligned rows (H % 8 == 0, 16-byte aligned, H <= 16384) have four kernels. The choice, from
    // cold-L2 sweeps on B200 against each other and vLLM's kernels (1..262144 rows, H 128..16384):
    // * up to 256 rows (decode batches), or with one chunk a thread (H <= 4096) as many rows as
    //   have their CTAs resident at once: a CTA per row with the row in registers - one memory
    //   round trip, no shared-memory hand-off. 3 CTAs of 448 threads an SM at H = 3584 (444 rows),
    //   888 rows at 2048, the fp8 op's 64 registers: 296 at 3584; at most 8 an SM (1184 rows).
    //   Measured 3-34 % under the other kernels there (H 128-4096; e.g. 384 x 3584 3.14 against
    //   3.43 us, 64 x 1024 1.65 against the warp kernel's 2.41), 10-37 % over them once a second
    //   wave is needed, and 13 % over with 10 CTAs an SM at 1480 x 1032;
    // * more rows of H <= 1024 that move under 7 KiB each (RMSNorm up to H = 1024, add+RMSNorm up
    //   to 768): a warp per row, eight rows a CTA. A CTA per row is held to the rate at which
    //   the GPU starts CTAs there (about one a nanosecond: 131072 rows took ~135 us at any width
    //   up to 512), 1.4-4x slower;
    // * otherwise a small CTA for every row whose threads keep their chunks in registers (stash
    //   kernel), up to H = 16384. It streams like a copy: add+RMSNorm 10.9 against the staged
    //   ring's 11.4 us at [2048, 3584], 2462 against 2657 us at 262144 x 8192 (106.5 % of the copy
    //   peak), 12-35 % ahead of the ring at H = 13312-16384; RMSNorm at or ahead of the ring at
    //   every size; the fp8 output 5-20 % ahead of it at all but one of 44 shapes; 6-18 % ahead of
    //   the warp kernel for add+RMSNorm rows of 1024 (8 KiB). The ring was 1-4 % ahead for
    //   add+RMSNorm at three resident shapes only (2048 x 2560, 1024 x 5120, 768 x 6144). RMSNorm of
    //   rows of 8192 and more, 4096+ rows: eight chunks a thread (4-10 % faster there, even with
    //   vLLM's kernel at 32768 x 8192; slower on fewer or shorter rows).
    const bool vector_rows = hidden % 8 == 0 && hidden <= kCtaRowMaxHidden && ((xa | oa) & 15u) == 0 && fp8_vector_ok;
    bool cta_one_wave = false;
    if (vector_rows && hidden <= 8 * kCtaRowMaxThreads) {  // one chunk a thread; t >= 32 (H >= 8)
        const int64_t t = (hidden / 8 + kWarpSize - 1) / kWarpSize * kWarpSize;
        const int64_t regs = mode == kModeFusedFp8 ? kCtaRowRegsFp8 : kCtaRowRegs;
        int64_t per_sm = kRegistersPerSm / (t * regs);
        if (per_sm > kThreadsPerSm / t) per_sm = kThreadsPerSm / t;
        if (per_sm > kCtaRowMaxResident) per_sm = kCtaRowMaxResident;
        cta_one_wave = rows <= static_cast<int64_t>(sm_count) * per_sm;
    }
    const bool few_rows = rows <= kCtaRowMaxRows || cta_one_wave;
    const int64_t row_bytes = hidden * (mode == kModePlain ? 4 : mode == kModeFusedFp8 ? 7 : 8);  // HBM bytes
    if (vector_rows && hidden <= kWarpRowMaxHidden && !few_rows && row_bytes < kStashMinRowBytes) {
        const int64_t per_lane = (hidden / 8 + kWarpSize - 1) / kWarpSize;
        plan.family = RmsFamily::kWarpRow;
        plan.chunks_per_lane = per_lane <= 1 ? 1 : per_lane <= 2 ? 2 : 4;
        const int64_t warps_per_cta = kWarpRowThreads / kWarpSize;
        const int64_t need = (rows + warps_per_cta - 1) / warps_per_cta;
        const int64_t cap = static_cast<int64_t>(sm_count) * 8;
        plan.grid = static_cast<unsigned>(need < cap ? need : cap);
        plan.smem = static_cast<size_t>(hidden) * 4u;
        return plan;
    }
    const int family_choice = few_rows ? 1 : hidden > kStashMaxHidden ? 3 : 2;  // 1 CTA per row, 2 stash, 3 staged
    // Rows of 16384 < H <= 32768: the stash kernel with eight chunks a thread (up to 512 threads;
    // add+RMSNorm and the fp8 op at 128 registers, one CTA an SM, or, up to H = 20480 and for more
    // than 256 rows, the instance capped at 96 registers, two an SM). 2-9x the two-pass row kernel that
    // served these rows before; against vLLM's kernel 0.8-1.03x its time.
    const bool long_rows = hidden % 8 == 0 && hidden > kCtaRowMaxHidden && hidden <= kStashMaxLongHidden &&
                           ((xa | oa) & 15u) == 0 && fp8_vector_ok;
    // Many rows off 16 bytes, x and residual (or out) alike: the stash kernel's scheme on the aligned
    // chunks that cover each row, bf16 outputs. Against the staged ring (cold, CUDA graph) 3-22 %
    // faster for add+RMSNorm at 15 of 20 shapes of 384-16384 rows x H 2048-8192 (2048 x 3584: 11.75
    // against 12.35 us), level at two, 7 % slower at 1024 x 4096; for RMSNorm 9-31 % faster at
    // H = 3584 and 7-12 % slower at 8192, hence its lower limit.
    const bool shifted_rows = hidden % 8 == 0 && hidden > kWarpRowMaxHidden && (xa & 15u) != 0 &&
                              (xa & 15u) == (oa & 15u) && rows > kCtaRowMaxRows &&
                              hidden <= (mode == kModeFused ? kShiftedMaxHidden
                                         : mode == kModePlain ? kShiftedPlainMaxHidden : 0);
    // Add+RMSNorm rows of 1536 <= H <= 4080 (H % 16 == 0: at most 256 threads, four CTAs an SM),
    // 257-4096 of them, x and residual at the same phase P in the first half of a 32-byte block
    // (the covering chunks pair up into 32-byte blocks), a 16-byte aligned weight: the shifted
    // scheme with 256-bit accesses, every CTA looking one resident wave ahead. Measured on B200
    // (cold L2, CUDA graph, library A/B on one box) against the shifted kernel: 2048 x 3584 10.57
    // against 10.98 us (every phase 1.04-1.05x), 300 x 3584 1.10x, 2048 x 2048 1.15x, 4096 x 2048
    // 1.06x, 1024 x 3584 level; at H = 5120 (352 threads, two CTAs an SM) 0.97x.
    if (mode == kModeFused && hidden % 16 == 0 && hidden >= kStashV8MinHidden && hidden <= kShiftedV8MaxHidden &&
        rows > kCtaRowMaxRows && rows <= kStashV8MaxRows && (xa & 15u) != 0 && (xa & 31u) == (oa & 31u) &&
        (xa & 31u) < 16u && (reinterpret_cast<uintptr_t>(weight) & 15u) == 0) {
        const int64_t threads = (hidden / 16 + 1 + kWarpSize - 1) / kWarpSize * kWarpSize;
        plan.family = RmsFamily::kShiftedV8;
        plan.chunks_per_lane = 2;
        plan.phase = static_cast<int>((xa & 15u) >> 1);
        plan.threads = static_cast<unsigned>(threads);
        plan.grid = static_cast<unsigned>(rows);
        const int64_t wave = resident_ctas(sm_count, threads, 64);  // launch bound (512, 2): 64 registers
        plan.lookahead = rows > wave ? wave : 0;
        plan.lookahead_ctas = rows > wave ? rows : 0;
        return plan;
    }
    if (shifted_rows) {
        const int64_t row_chunks = hidden / 8 + 1;
        const int64_t per_warp = static_cast<int64_t>(kStashChunks) * kWarpSize;
        int64_t threads = (row_chunks + per_warp - 1) / per_warp * kWarpSize;
        threads = threads < kStashMinThreads ? kStashMinThreads : threads;
        plan.family = RmsFamily::kShifted;
        plan.chunks_per_lane = kStashChunks;
        plan.phase = static_cast<int>((xa & 15u) >> 1);
        plan.threads = static_cast<unsigned>(threads);
        plan.grid = static_cast<unsigned>(rows < INT_MAX ? rows : INT_MAX);
        set_lookahead(plan, rows, resident_ctas(sm_count, threads, 64));  // launch bound (512, 2): 64 registers
        return plan;
    }
    // Many aligned rows: a small CTA for every row, each thread's chunks in registers.
    if ((vector_rows && family_choice == 2) || long_rows) {
        // Up to kStashChunks chunks a thread (H <= 16384 needs at most 512 threads).
        const int per_lane =
            long_rows || (mode == kModePlain && hidden >= 8192 && rows >= 4096) ? kStashWideChunks : kStashChunks;
        const int64_t row_chunks = hidden / 8;
        const int64_t per_warp = static_cast<int64_t>(per_lane) * kWarpSize;
        int64_t threads = (row_chunks + per_warp - 1) / per_warp * kWarpSize;
        threads = threads < kStashMinThreads ? kStashMinThreads : threads;
        plan.family = RmsFamily::kStash;
        plan.chunks_per_lane = per_lane;
        plan.capped = long_rows && mode != kModePlain && hidden <= kStashCappedMaxHidden && rows > kCtaRowMaxRows;
        plan.threads = static_cast<unsigned>(threads);
        plan.smem = per_lane == kStashChunks ? static_cast<size_t>(hidden) * 2u : 0;  // staged gamma
        plan.grid = static_cast<unsigned>(rows < INT_MAX ? rows : INT_MAX);
        // Registers a thread may take under each instance's launch bound: 64, the capped
        // instance 96, eight chunks a thread with a residual 128.
        const int64_t regs = plan.capped ? 96 : (per_lane == kStashWideChunks && mode != kModePlain) ? 128 : 64;
        set_lookahead(plan, rows, resident_ctas(sm_count, threads, regs));
        return plan;
    }
    // Few aligned rows: a CTA per row, values in registers.
    if (vector_rows && family_choice == 1) {
        const int64_t row_chunks = hidden / 8;
        const int64_t per_thread = (row_chunks + kCtaRowMaxThreads - 1) / kCtaRowMaxThreads;
        plan.family = RmsFamily::kCtaRow;
        plan.chunks_per_lane = per_thread <= 1 ? 1 : per_thread <= 2 ? 2 : 4;
        const int64_t threads = (row_chunks + plan.chunks_per_lane - 1) / plan.chunks_per_lane;
        plan.threads = static_cast<unsigned>((threads + kWarpSize - 1) / kWarpSize * kWarpSize);
        plan.grid = static_cast<unsigned>(rows < INT_MAX ? rows : INT_MAX);  // a CTA for every row
        return plan;
    }
    if ((xa & 15u) == (oa & 15u) && max_stages >= 2 && mode != kModeFusedFp8) {
        const int grid = static_cast<int>(rows < sm_count ? rows : sm_count);
        const int64_t rows_per_cta = (rows + grid - 1) / grid;
        // Ring depth S and consumer groups G (W = 16 / G warps per row), from a sweep of both on
        // B200 (2048..262144 rows, H 1024..8192):
        // * a CTA whose rows all fit in shared memory at once takes them all (S = its rows) and
        //   processes up to 8 at a time: the kernel is then bound by its start-up and drain, and
        //   having every row requested at the start shortens both;
        // * a CTA that streams more rows than fit keeps about 128 KB in flight with one stage per
        //   group (S = G): 4 x 32 KB rows at H = 8192 ran at 97 % of the copy peak, deeper rings
        //   at 91 %. The fp8 output's conversion makes pass 2 heavier: there half the groups, each
        //   of twice the warps, share the same ring (S = 2G), 3-7 % faster at 32768 rows.
        int stages;
        int groups;
        if (rows_per_cta <= max_stages) {
            stages = static_cast<int>(rows_per_cta);
            groups = stages >= 8 ? 8 : stages >= 4 ? 4 : stages >= 2 ? 2 : 1;
        } else {
            const int target = static_cast<int>((128 * 1024 + stage_bytes / 2) / stage_bytes);
            groups = 1;
            while (groups * 2 <= target && groups * 2 <= kStagedConsumerWarps && groups * 2 <= max_stages) {
                groups *= 2;
            }
            stages = groups;
        }
        plan.family = RmsFamily::kStaged;
        plan.warps_per_row = kStagedConsumerWarps / groups;
        plan.grid = static_cast<unsigned>(grid);
        plan.staged.rows = rows;
        plan.staged.hidden = static_cast<int>(hidden);
        plan.staged.chunks_max = chunks_max;
        plan.staged.stage_bytes = stage_bytes;
        plan.staged.stages = stages;
        plan.staged.row_phase = row_phase;
        plan.smem = staged_layout(stages, stage_bytes, chunks_max).total;
        return plan;
    }
    plan.family = hidden <= static_cast<int64_t>(kRowwiseThreads) * kRowwiseCachedPerThread
                      ? RmsFamily::kRowwiseCached
                      : RmsFamily::kRowwiseTwoPass;
    const int64_t cap = static_cast<int64_t>(sm_count) * 8;
    plan.grid = static_cast<unsigned>(rows < cap ? rows : cap);
    return plan;
}

WarpRowParams row_params(const RmsPlan& plan) {
    WarpRowParams w;
    w.x = plan.staged.x;
    w.residual = plan.staged.residual;
    w.out = plan.staged.out;
    w.out8 = plan.staged.out8;
    w.scale = plan.staged.scale;
    w.weight = plan.staged.weight;
    w.rows = plan.staged.rows;
    w.hidden = plan.staged.hidden;
    w.epsilon = plan.staged.epsilon;
    w.lookahead = plan.lookahead;
    w.lookahead_ctas = plan.lookahead_ctas;
    w.cluster_slice = plan.cluster_slice;
    return w;
}

const char* mode_label(int mode) {
    return mode == kModeFused ? "fused RMSNorm" : mode == kModePlain ? "RMSNorm" : "fused RMSNorm fp8";
}

// The stash kernel's four-chunk instances stage gamma in plan.smem bytes of dynamic shared
// memory (H * 2, at most 32 KB: under the default limit, no opt-in); the eight-chunk ones use none.
template <int kMode>
ipl_status launch_stash(const RmsPlan& plan, cudaStream_t stream, const WarpRowParams& w) {
    cudaError_t err;
    if constexpr (kMode != kModePlain) {
        if (plan.capped) {
            err = launch(rmsnorm_stash_kernel<kStashWideChunks, kMode, true>, plan.grid, plan.threads, 0, stream, w);
            if (err != cudaSuccess) {
                return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
            }
            return IPL_SUCCESS;
        }
    }
    err = plan.chunks_per_lane == kStashWideChunks
              ? launch(rmsnorm_stash_kernel<kStashWideChunks, kMode>, plan.grid, plan.threads, 0, stream, w)
              : launch(rmsnorm_stash_kernel<kStashChunks, kMode>, plan.grid, plan.threads, plan.smem, stream, w);
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
    }
    return IPL_SUCCESS;
}

template <int W, int kMode>
ipl_status launch_staged(const RmsPlan& plan, DeviceInfo* info, cudaStream_t stream) {
    auto kernel = rmsnorm_staged_kernel<W, kMode>;
    int bit = 0;
    while ((1 << bit) < W) ++bit;
    bit += 8 * kMode;
    if (!(info->smem_configured.load(std::memory_order_acquire) & (1u << bit))) {
        const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     info->max_smem_optin.load());
        if (err != cudaSuccess) {
            return fail(IPL_ERROR_CUDA, "%s kernel setup failed: %s", mode_label(kMode), cudaGetErrorString(err));
        }
        info->smem_configured.fetch_or(1u << bit, std::memory_order_acq_rel);
    }
    const cudaError_t err = launch(kernel, plan.grid, kStagedThreads, plan.smem, stream, plan.staged);
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
    }
    return IPL_SUCCESS;
}

template <int kMode>
ipl_status run_rms(uint16_t* x, uint16_t* residual, uint16_t* out, uint8_t* out8, const float* scale,
                   const uint16_t* weight, int64_t rows, int64_t hidden, double epsilon, cudaStream_t stream) {
    constexpr bool kResidual = kMode != kModePlain;
    int device = 0;
    DeviceInfo* info = nullptr;
    ipl_status st = current_device(&device, &info);
    if (st != IPL_SUCCESS) return st;
    RmsPlan plan = plan_rms(x, kResidual ? static_cast<const void*>(residual) : static_cast<const void*>(out), out8,
                            weight, rows, hidden, kMode, info->sm_count.load(std::memory_order_relaxed),
                            info->max_smem_optin.load(std::memory_order_relaxed));
    plan.staged.x = x;
    plan.staged.residual = residual;
    plan.staged.out = out;
    plan.staged.out8 = out8;
    plan.staged.scale = scale;
    plan.staged.weight = weight;
    plan.staged.rows = rows;
    plan.staged.hidden = static_cast<int>(hidden);
    plan.staged.epsilon = static_cast<float>(epsilon);
    switch (plan.family) {
        case RmsFamily::kStaged:
            if constexpr (kMode == kModeFusedFp8) {
                return fail(IPL_ERROR_CUDA, "%s: no staged plan exists for this mode", mode_label(kMode));
            } else {
                switch (plan.warps_per_row) {
                    case 1: return launch_staged<1, kMode>(plan, info, stream);
                    case 2: return launch_staged<2, kMode>(plan, info, stream);
                    case 4: return launch_staged<4, kMode>(plan, info, stream);
                    case 8: return launch_staged<8, kMode>(plan, info, stream);
                    default: return launch_staged<16, kMode>(plan, info, stream);
                }
            }
        case RmsFamily::kWarpRow: {
            const WarpRowParams w = row_params(plan);
            cudaError_t err = cudaSuccess;
            switch (plan.chunks_per_lane) {
                case 1: err = launch(rmsnorm_warp_kernel<1, kMode>, plan.grid, kWarpRowThreads, plan.smem, stream, w); break;
                case 2: err = launch(rmsnorm_warp_kernel<2, kMode>, plan.grid, kWarpRowThreads, plan.smem, stream, w); break;
                default: err = launch(rmsnorm_warp_kernel<4, kMode>, plan.grid, kWarpRowThreads, plan.smem, stream, w); break;
            }
            if (err != cudaSuccess) {
                return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
            }
            return IPL_SUCCESS;
        }
        case RmsFamily::kCtaRow: {
            const WarpRowParams w = row_params(plan);
            cudaError_t err = cudaSuccess;
            switch (plan.chunks_per_lane) {
                case 1: err = launch(rmsnorm_cta_kernel<1, kMode>, plan.grid, plan.threads, 0, stream, w); break;
                case 2: err = launch(rmsnorm_cta_kernel<2, kMode>, plan.grid, plan.threads, 0, stream, w); break;
                default: err = launch(rmsnorm_cta_kernel<4, kMode>, plan.grid, plan.threads, 0, stream, w); break;
            }
            if (err != cudaSuccess) {
                return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
            }
            return IPL_SUCCESS;
        }
        case RmsFamily::kStash: {
            const WarpRowParams w = row_params(plan);
            return launch_stash<kMode>(plan, stream, w);
        }
        case RmsFamily::kShifted: {
            if constexpr (kMode == kModeFusedFp8) {
                return fail(IPL_ERROR_CUDA, "%s: no shifted plan exists for this mode", mode_label(kMode));
            } else {
                const WarpRowParams w = row_params(plan);
                cudaError_t err = cudaSuccess;
                switch (plan.phase) {
                    case 1: err = launch(rmsnorm_shifted_kernel<kMode, 1>, plan.grid, plan.threads, 0, stream, w); break;
                    case 2: err = launch(rmsnorm_shifted_kernel<kMode, 2>, plan.grid, plan.threads, 0, stream, w); break;
                    case 3: err = launch(rmsnorm_shifted_kernel<kMode, 3>, plan.grid, plan.threads, 0, stream, w); break;
                    case 4: err = launch(rmsnorm_shifted_kernel<kMode, 4>, plan.grid, plan.threads, 0, stream, w); break;
                    case 5: err = launch(rmsnorm_shifted_kernel<kMode, 5>, plan.grid, plan.threads, 0, stream, w); break;
                    case 6: err = launch(rmsnorm_shifted_kernel<kMode, 6>, plan.grid, plan.threads, 0, stream, w); break;
                    default: err = launch(rmsnorm_shifted_kernel<kMode, 7>, plan.grid, plan.threads, 0, stream, w); break;
                }
                if (err != cudaSuccess) {
                    return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
                }
                return IPL_SUCCESS;
            }
        }
        case RmsFamily::kStashV8: {
            if constexpr (kMode == kModePlain) {
                return fail(IPL_ERROR_CUDA, "%s: no 256-bit stash plan exists for this mode", mode_label(kMode));
            } else {
                const WarpRowParams w = row_params(plan);
                const cudaError_t err =
                    launch(rmsnorm_stash_v8_kernel<kMode>, plan.grid, plan.threads, plan.smem, stream, w);
                if (err != cudaSuccess) {
                    return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
                }
                return IPL_SUCCESS;
            }
        }
        case RmsFamily::kCluster: {
            const WarpRowParams w = row_params(plan);
            const unsigned cluster = static_cast<unsigned>(plan.cluster);
            cudaError_t err = cudaSuccess;
            switch (plan.chunks_per_lane) {
                case 1: err = launch_clustered(rmsnorm_cluster_kernel<1, kMode>, plan.grid, cluster, plan.threads, plan.smem, stream, w); break;
                case 2: err = launch_clustered(rmsnorm_cluster_kernel<2, kMode>, plan.grid, cluster, plan.threads, plan.smem, stream, w); break;
                default: err = launch_clustered(rmsnorm_cluster_kernel<4, kMode>, plan.grid, cluster, plan.threads, plan.smem, stream, w); break;
            }
            if (err != cudaSuccess) {
                return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
            }
            return IPL_SUCCESS;
        }
        case RmsFamily::kShiftedV8: {
            if constexpr (kMode != kModeFused) {
                return fail(IPL_ERROR_CUDA, "%s: no 256-bit shifted plan exists for this mode", mode_label(kMode));
            } else {
                const WarpRowParams w = row_params(plan);
                cudaError_t err = cudaSuccess;
                switch (plan.phase) {
                    case 1: err = launch(rmsnorm_shifted_v8_kernel<1>, plan.grid, plan.threads, 0, stream, w); break;
                    case 2: err = launch(rmsnorm_shifted_v8_kernel<2>, plan.grid, plan.threads, 0, stream, w); break;
                    case 3: err = launch(rmsnorm_shifted_v8_kernel<3>, plan.grid, plan.threads, 0, stream, w); break;
                    case 4: err = launch(rmsnorm_shifted_v8_kernel<4>, plan.grid, plan.threads, 0, stream, w); break;
                    case 5: err = launch(rmsnorm_shifted_v8_kernel<5>, plan.grid, plan.threads, 0, stream, w); break;
                    case 6: err = launch(rmsnorm_shifted_v8_kernel<6>, plan.grid, plan.threads, 0, stream, w); break;
                    default: err = launch(rmsnorm_shifted_v8_kernel<7>, plan.grid, plan.threads, 0, stream, w); break;
                }
                if (err != cudaSuccess) {
                    return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
                }
                return IPL_SUCCESS;
            }
        }
        case RmsFamily::kRowwiseCached:
        case RmsFamily::kRowwiseTwoPass: {
            const cudaError_t err =
                plan.family == RmsFamily::kRowwiseCached
                    ? launch(rmsnorm_rowwise_kernel<true, kMode>, plan.grid, kRowwiseThreads, 0, stream,
                             static_cast<const uint16_t*>(x), residual, out, out8, scale, weight, rows,
                             static_cast<int>(hidden), plan.staged.epsilon)
                    : launch(rmsnorm_rowwise_kernel<false, kMode>, plan.grid, kRowwiseThreads, 0, stream,
                             static_cast<const uint16_t*>(x), residual, out, out8, scale, weight, rows,
                             static_cast<int>(hidden), plan.staged.epsilon);
            if (err != cudaSuccess) {
                return fail(IPL_ERROR_CUDA, "%s kernel launch failed: %s", mode_label(kMode), cudaGetErrorString(err));
            }
            return IPL_SUCCESS;
        }
        case RmsFamily::kNone:
            return IPL_SUCCESS;
    }
    return IPL_SUCCESS;
}

// ------------------------------------------------------------------------------------------
// SiLU-and-mul planning

enum class SiluKernel { kNone, kWave16, kVector32, kVector16, kScalar };

const char* silu_kernel_name(SiluKernel k) {
    switch (k) {
        case SiluKernel::kNone: return "none";
        case SiluKernel::kWave16: return "silu_wave_kernel";
        case SiluKernel::kVector32: return "silu_vector_kernel<32>";
        case SiluKernel::kVector16: return "silu_vector_kernel<16>";
        case SiluKernel::kScalar: return "silu_scalar_kernel";
    }
    return "invalid";
}

ipl_status check_silu_args(const void* output, const void* input, int64_t rows, int64_t inter) {
    if (rows < 0 || inter < 0) return fail(IPL_ERROR_INVALID_VALUE, "sizes must be non-negative");
    if (inter > (INT64_MAX / 4) || (inter > 0 && rows > INT64_MAX / (4 * inter))) {
        return fail(IPL_ERROR_TOO_LARGE, "input is too large");
    }
    if (rows * inter > 0 && (output == nullptr || input == nullptr)) {
        return fail(IPL_ERROR_INVALID_VALUE, "input and output must be non-null");
    }
    if ((reinterpret_cast<uintptr_t>(output) | reinterpret_cast<uintptr_t>(input)) & 1u) {
        return fail(IPL_ERROR_INVALID_VALUE, "bfloat16 pointers must be 2-byte aligned");
    }
    return IPL_SUCCESS;
}

SiluKernel plan_silu(const void* output, const void* input, int64_t rows, int64_t inter, int sm_count) {
    if (rows * inter == 0) return SiluKernel::kNone;
    const uintptr_t a = reinterpret_cast<uintptr_t>(output) | reinterpret_cast<uintptr_t>(input);
    const uint64_t packs32 = static_cast<uint64_t>(rows) * static_cast<uint64_t>(inter / 16);
    const uint64_t packs16 = static_cast<uint64_t>(rows) * static_cast<uint64_t>(inter / 8);
    // One 16-byte pack per thread in a single wave of two 1024-thread CTAs per SM, when the packs
    // fill more than one such CTA per SM.
    const uint64_t wave16 = static_cast<uint64_t>(sm_count) * 2 * kSiluWaveThreads;
    if (inter % 8 == 0 && (a & 15u) == 0 && packs16 > wave16 / 2 && packs16 <= wave16) return SiluKernel::kWave16;
    if (inter % 16 == 0 && (a & 31u) == 0 && packs32 <= UINT32_MAX) return SiluKernel::kVector32;
    if (inter % 8 == 0 && (a & 15u) == 0 && packs16 <= UINT32_MAX) return SiluKernel::kVector16;
    return SiluKernel::kScalar;
}

template <int kBytes>
cudaError_t launch_silu_vector(uint16_t* out, const uint16_t* in, int64_t rows, int64_t inter,
                               int sm_count, cudaStream_t stream) {
    SiluVectorParams p;
    p.out = out;
    p.in = in;
    p.intermediate = inter;
    const uint32_t per_row = static_cast<uint32_t>(inter / (kBytes / 2));
    p.total_packs = static_cast<uint32_t>(rows) * per_row;
    p.packs_per_row = make_fast_div32(per_row);
    // One wave: 8 CTAs of 256 threads per SM. Pick the smallest unroll that covers the work in
    // that wave, up to 4, then loop.
    const uint64_t wave = static_cast<uint64_t>(sm_count) * 8 * kSiluThreads;
    const uint64_t total = p.total_packs;
    if (total <= wave) {
        const unsigned grid = static_cast<unsigned>((total + kSiluThreads - 1) / kSiluThreads);
        return launch(silu_vector_kernel<kBytes, 1>, grid, kSiluThreads, 0, stream, p);
    }
    if (total <= 2 * wave) {
        const unsigned grid = static_cast<unsigned>((total + 2 * kSiluThreads - 1) / (2 * kSiluThreads));
        return launch(silu_vector_kernel<kBytes, 2>, grid, kSiluThreads, 0, stream, p);
    }
    const uint64_t need = (total + 4 * kSiluThreads - 1) / (4 * kSiluThreads);
    const unsigned grid = static_cast<unsigned>(need < wave / kSiluThreads ? need : wave / kSiluThreads);
    return launch(silu_vector_kernel<kBytes, 4>, grid, kSiluThreads, 0, stream, p);
}

ipl_status run_silu(void* output, const void* input, int64_t rows, int64_t inter, void* stream_ptr,
                    bool packed_contract) {
    ipl_status st = check_silu_args(output, input, rows, inter);
    if (st != IPL_SUCCESS) return st;
    if (rows * inter == 0) return IPL_SUCCESS;
    if (packed_contract) {
        if (inter % 8 != 0) return fail(IPL_ERROR_MISALIGNED, "the output width must be divisible by 8");
        if ((reinterpret_cast<uintptr_t>(output) | reinterpret_cast<uintptr_t>(input)) & 15u) {
            return fail(IPL_ERROR_MISALIGNED, "input and output must be 16-byte aligned");
        }
    }
    int device = 0;
    DeviceInfo* info = nullptr;
    st = current_device(&device, &info);
    if (st != IPL_SUCCESS) return st;
    const int sms = info->sm_count.load(std::memory_order_relaxed);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    auto* out = static_cast<uint16_t*>(output);
    const auto* in = static_cast<const uint16_t*>(input);
    cudaError_t err = cudaSuccess;
    switch (plan_silu(output, input, rows, inter, sms)) {
        case SiluKernel::kWave16: {
            SiluVectorParams p;
            p.out = out;
            p.in = in;
            p.intermediate = inter;
            const uint32_t per_row = static_cast<uint32_t>(inter / 8);
            p.total_packs = static_cast<uint32_t>(rows) * per_row;
            p.packs_per_row = make_fast_div32(per_row);
            const unsigned grid = (p.total_packs + kSiluWaveThreads - 1) / kSiluWaveThreads;
            err = launch(silu_wave_kernel, grid, kSiluWaveThreads, 0, stream, p);
            break;
        }
        case SiluKernel::kVector32:
            err = launch_silu_vector<32>(out, in, rows, inter, sms, stream);
            break;
        case SiluKernel::kVector16:
            err = launch_silu_vector<16>(out, in, rows, inter, sms, stream);
            break;
        case SiluKernel::kScalar: {
            const int64_t total = rows * inter;
            const int64_t cap = static_cast<int64_t>(sms) * 8;
            const int64_t need = (total + kSiluThreads - 1) / kSiluThreads;
            err = launch(silu_scalar_kernel, static_cast<unsigned>(need < cap ? need : cap), kSiluThreads, 0,
                         stream, out, in, rows, inter);
            break;
        }
        case SiluKernel::kNone:
            break;
    }
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "%s SiLU-and-multiply kernel launch failed: %s",
                    packed_contract ? "packed" : "scalar", cudaGetErrorString(err));
    }
    return IPL_SUCCESS;
}

}  // namespace
}  // namespace ipl

using namespace ipl;

extern "C" {

ipl_status ipl_fused_add_rms_norm_bf16(void* x, void* residual, const void* weight, int64_t rows,
                                       int64_t hidden_size, double epsilon, void* stream) {
    const ipl_status st = check_rms_args(x, residual, weight, rows, hidden_size, epsilon, true);
    if (st != IPL_SUCCESS || rows == 0) return st;
    return run_rms<kModeFused>(static_cast<uint16_t*>(x), static_cast<uint16_t*>(residual), static_cast<uint16_t*>(x),
                               nullptr, nullptr, static_cast<const uint16_t*>(weight), rows, hidden_size, epsilon,
                               static_cast<cudaStream_t>(stream));
}

ipl_status ipl_rms_norm_bf16(void* output, const void* input, const void* weight, int64_t rows,
                             int64_t hidden_size, double epsilon, void* stream) {
    const ipl_status st = check_rms_args(input, output, weight, rows, hidden_size, epsilon, false);
    if (st != IPL_SUCCESS || rows == 0) return st;
    return run_rms<kModePlain>(const_cast<uint16_t*>(static_cast<const uint16_t*>(input)), nullptr,
                               static_cast<uint16_t*>(output), nullptr, nullptr, static_cast<const uint16_t*>(weight),
                               rows, hidden_size, epsilon, static_cast<cudaStream_t>(stream));
}

ipl_status ipl_fused_add_rms_norm_static_fp8_quant(void* output, const void* input, void* residual,
                                                   const void* weight, const float* scale, int64_t rows,
                                                   int64_t hidden_size, double epsilon, void* stream) {
    ipl_status st = check_rms_args(input, residual, weight, rows, hidden_size, epsilon, true);
    if (st != IPL_SUCCESS || rows == 0) return st;
    if (output == nullptr || scale == nullptr) {
        return fail(IPL_ERROR_INVALID_VALUE, "output and scale must be non-null");
    }
    if (reinterpret_cast<uintptr_t>(scale) & 3u) {
        return fail(IPL_ERROR_INVALID_VALUE, "scale must be 4-byte aligned");
    }
    uint16_t* x = const_cast<uint16_t*>(static_cast<const uint16_t*>(input));
    return run_rms<kModeFusedFp8>(x, static_cast<uint16_t*>(residual), x, static_cast<uint8_t*>(output), scale,
                                  static_cast<const uint16_t*>(weight), rows, hidden_size, epsilon,
                                  static_cast<cudaStream_t>(stream));
}

ipl_status ipl_silu_and_mul_bf16(void* output, const void* input, int64_t rows, int64_t intermediate_size,
                                 void* stream) {
    return run_silu(output, input, rows, intermediate_size, stream, false);
}

ipl_status ipl_silu_and_mul_packed_bf16(void* output, const void* input, int64_t rows,
                                        int64_t intermediate_size, void* stream) {
    return run_silu(output, input, rows, intermediate_size, stream, true);
}

const char* ipl_last_error(void) { return t_last_error; }

const char* ipl_status_string(ipl_status status) {
    switch (status) {
        case IPL_SUCCESS: return "IPL_SUCCESS";
        case IPL_ERROR_INVALID_VALUE: return "IPL_ERROR_INVALID_VALUE";
        case IPL_ERROR_MISALIGNED: return "IPL_ERROR_MISALIGNED";
        case IPL_ERROR_TOO_LARGE: return "IPL_ERROR_TOO_LARGE";
        case IPL_ERROR_CUDA: return "IPL_ERROR_CUDA";
    }
    return "IPL_UNKNOWN_STATUS";
}

int ipl_abi_version(void) { return IPL_ABI_VERSION; }

ipl_status ipl_device_fault_flags(int device, uint32_t* flags) {
    if (flags == nullptr) return fail(IPL_ERROR_INVALID_VALUE, "flags must be non-null");
    int previous = 0;
    cudaError_t err = cudaGetDevice(&previous);
    if (err == cudaSuccess) err = cudaSetDevice(device);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpyFromSymbol(flags, g_fault_word, sizeof(uint32_t));
    cudaSetDevice(previous);
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "failed to read the device fault word: %s", cudaGetErrorString(err));
    }
    return IPL_SUCCESS;
}

ipl_status ipl_clear_device_fault_flags(int device) {
    int previous = 0;
    const uint32_t zero = 0;
    cudaError_t err = cudaGetDevice(&previous);
    if (err == cudaSuccess) err = cudaSetDevice(device);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_fault_word, &zero, sizeof(uint32_t));
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    cudaSetDevice(previous);
    if (err != cudaSuccess) {
        return fail(IPL_ERROR_CUDA, "failed to clear the device fault word: %s", cudaGetErrorString(err));
    }
    return IPL_SUCCESS;
}

const char* ipl_fused_add_rms_norm_plan(const void* x, const void* residual, const void* weight, int64_t rows,
                                        int64_t hidden_size) {
    if (check_rms_args(x, residual, weight, rows, hidden_size, 1.0, true) != IPL_SUCCESS) return "invalid";
    int sms = 0, smem = 0;
    plan_limits(&sms, &smem);
    return rms_kernel_name(plan_rms(x, residual, nullptr, weight, rows, hidden_size, kModeFused, sms, smem), kModeFused);
}

const char* ipl_rms_norm_plan(const void* output, const void* input, const void* weight, int64_t rows,
                              int64_t hidden_size) {
    if (check_rms_args(input, output, weight, rows, hidden_size, 1.0, false) != IPL_SUCCESS) return "invalid";
    int sms = 0, smem = 0;
    plan_limits(&sms, &smem);
    return rms_kernel_name(plan_rms(input, output, nullptr, weight, rows, hidden_size, kModePlain, sms, smem), kModePlain);
}

const char* ipl_fused_add_rms_norm_static_fp8_quant_plan(const void* output, const void* input, const void* residual,
                                                         const void* weight, int64_t rows, int64_t hidden_size) {
    if (check_rms_args(input, residual, weight, rows, hidden_size, 1.0, true) != IPL_SUCCESS || output == nullptr) {
        return "invalid";
    }
    int sms = 0, smem = 0;
    plan_limits(&sms, &smem);
    return rms_kernel_name(plan_rms(input, residual, output, weight, rows, hidden_size, kModeFusedFp8, sms, smem),
                           kModeFusedFp8);
}

const char* ipl_silu_and_mul_plan(const void* output, const void* input, int64_t rows,
                                  int64_t intermediate_size) {
    if (check_silu_args(output, input, rows, intermediate_size) != IPL_SUCCESS) return "invalid";
    int sms = 0, smem = 0;
    plan_limits(&sms, &smem);
    return silu_kernel_name(plan_silu(output, input, rows, intermediate_size, sms));
}

}  // extern "C"
