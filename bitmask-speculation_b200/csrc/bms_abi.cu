// C-ABI entry points (include/bms_b200.h) and launch configuration.
//
// The library is a plain shared object built by nvcc for sm_100a; it links the
// CUDA runtime and nothing else, takes raw device pointers and a cudaStream_t,
// and allocates no memory.  Launch choices:
//  * rows whose logits and masks start on 16-byte boundaries stream through the
//    bulk-copy (TMA) pipeline; other rows use the plain-load variant of the same
//    kernel;
//  * the cluster size C (CTAs sharing one row) and the number of persistent
//    clusters are chosen from the device's occupancy so that the slowest CTA
//    streams as few chunks as possible: many rows -> C = 1 with every SM busy,
//    few rows -> up to 16 CTAs per row merging through distributed shared memory.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/bms_b200.h"
#include "select.cuh"

namespace bms {
namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof g_error, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear a non-sticky error so later calls start clean
    return fail(BMS_ERROR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define BMS_CUDA(call, what)                                  \
    do {                                                      \
        const cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, (what));  \
    } while (0)

struct DeviceGuard {
    int prev = -1, want = -1;
    cudaError_t enter(int device) {
        want = device;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return e;
        if (prev != device) return cudaSetDevice(device);
        return cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0 && prev != want) cudaSetDevice(prev);
    }
};

int check_device(int device) {
    int n = 0;
    BMS_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(BMS_ERROR_INVALID_ARGUMENT, "invalid CUDA device %d", device);
    return BMS_SUCCESS;
}

// Every pointer the kernels touch must be device (or managed) memory of `device`.
int check_ptr(const void* p, int device, const char* name, size_t align) {
    if (p == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "%s must not be NULL", name);
    if (reinterpret_cast<uintptr_t>(p) % align != 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "%s must be %zu-byte aligned", name, align);
    cudaPointerAttributes a;
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(BMS_ERROR_INVALID_ARGUMENT, "%s is not a CUDA pointer", name);
    }
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "%s must be CUDA device memory", name);
    if (a.device != device)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "%s is on device %d, expected device %d", name, a.device, device);
    return BMS_SUCCESS;
}

#define BMS_CHECK(expr)                      \
    do {                                     \
        const int rc_ = (expr);              \
        if (rc_ != BMS_SUCCESS) return rc_;  \
    } while (0)

int elem_bytes(int dtype) { return dtype == BMS_FLOAT32 ? 4 : 2; }

int check_dtype(int dtype) {
    if (dtype != BMS_FLOAT32 && dtype != BMS_BFLOAT16 && dtype != BMS_FLOAT16)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "logits must be float32, bfloat16 or float16 (dtype code %d)", dtype);
    return BMS_SUCCESS;
}

int check_vocab(int64_t vocab) {
    if (vocab <= 0 || vocab > 2147483647LL) return fail(BMS_ERROR_INVALID_ARGUMENT, "invalid vocabulary size");
    return BMS_SUCCESS;
}

// ---------------------------------------------------------------- launch override (tests)
int g_force_cluster = 0;
int g_force_clusters = 0;

// ---------------------------------------------------------------- per-device kernel setup
constexpr int kMaxDevices = 64;
constexpr int kClusterSizes[] = {1, 2, 4, 8, 16};

struct KernelInfo {
    bool ready = false;
    int sms = 0;
    int max_clusters[5] = {0, 0, 0, 0, 0};  // resident clusters for each cluster size
    int flat_ctas = 0;                      // resident CTAs of the flat-schedule variant (sampler, bulk)
};

std::mutex g_mutex;

template <typename T, bool kSample, bool kBulk, int kStages>
int kernel_info(int device, KernelInfo*& out) {
    static KernelInfo table[kMaxDevices];
    std::lock_guard<std::mutex> lock(g_mutex);
    KernelInfo& info = table[device];
    if (!info.ready) {
        auto kernel = select_rows_kernel<T, kSample, kBulk, kStages>;
        const size_t smem = select_smem_bytes<T, kSample>(kStages);
        BMS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                 "cudaFuncSetAttribute(smem)");
        BMS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                 "cudaFuncSetAttribute(cluster)");
        BMS_CUDA(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device), "sm count");
        if constexpr (kSample && kBulk) {
            auto flat = select_rows_kernel<T, true, true, kStages, true>;
            BMS_CUDA(cudaFuncSetAttribute(flat, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                     "cudaFuncSetAttribute(smem)");
            int per_sm = 0;
            BMS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, flat, kThreads, smem), "flat occupancy");
            info.flat_ctas = per_sm * info.sms;
        }
        for (int i = 0; i < 5; ++i) {
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kClusterSizes[i];
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.gridDim = dim3(kClusterSizes[i] * info.sms);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = smem;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
            if (e != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
            info.max_clusters[i] = n;
        }
        if (info.max_clusters[0] <= 0) return fail(BMS_ERROR_CUDA, "selection kernel cannot be resident on device %d", device);
        info.ready = true;
    }
    out = &info;
    return BMS_SUCCESS;
}

int cluster_index(int c) {
    for (int i = 0; i < 5; ++i)
        if (kClusterSizes[i] == c) return i;
    return 0;
}

// Every rank's exchange area, passed by value to the merge kernel.
struct ExchangeAreas {
    uint8_t* a[kMaxExchangeRanks];
};

struct Plan {
    int cluster;
    int clusters;
    int64_t segment;
};

// Per-row cost of the row-end work (finalizer merge, cluster all-gather, index recovery or the
// sampling walk) in units of one streamed chunk, by cluster size; measured on B200 at
// V = 248,320 (2,304 rows: C = 1 / 2 / 4 took 194 / 203 / 258 us for the argmax and 301 / 374 /
// 620 us for the sampler).
constexpr double kRowCostArgmax[5] = {1.1, 2.4, 3.6, 5.0, 7.0};
constexpr double kRowCostSampler[5] = {5.0, 8.0, 12.0, 16.0, 20.0};

// Choose the cluster size that minimises the streaming plus row-end work of the busiest CTA.
// Clusters only pay while most SMs would idle: from one row per two SMs on, one-CTA clusters
// are as fast or faster (measured on B200 with one- and two-CTA clusters: 148 rows 13.3 / 16.4
// us for the argmax and 29.5 / 36.6 us for the sampler, 100 rows 13.1 / 14.3 and 29.3 / 32.2 us).
Plan plan_launch(const KernelInfo& info, int64_t rows, int64_t vocab, int tokens_per_chunk, int max_chunks,
                 bool sampler, bool single) {
    Plan best{0, 0, 0};
    double best_cost = 0.0;
    for (int i = 0; i < 5; ++i) {
        const int c = kClusterSizes[i];
        if (single ? c != 1 : (g_force_cluster ? c != g_force_cluster : (c > 1 && 2 * rows >= info.sms))) continue;
        const int resident = info.max_clusters[i];
        if (resident <= 0) continue;
        const int64_t seg = ((vocab + c - 1) / c + 31) / 32 * 32;
        const int64_t chunks = (seg + tokens_per_chunk - 1) / tokens_per_chunk;
        if (max_chunks > 0 && chunks > max_chunks) continue;
        int64_t clusters = rows < resident ? rows : resident;
        if (g_force_clusters) clusters = g_force_clusters < rows ? g_force_clusters : rows;
        const int64_t waves = (rows + clusters - 1) / clusters;
        const double overhead = sampler ? kRowCostSampler[i] : kRowCostArgmax[i];
        const double cost = static_cast<double>(waves) * (static_cast<double>(chunks) + overhead);
        if (best.cluster == 0 || cost < best_cost - 1e-9) {
            best = Plan{c, static_cast<int>(clusters), seg};
            best_cost = cost;
        }
    }
    return best;
}

std::atomic<uint32_t> g_epoch{0};

// Dynamic schedule (a workspace is given, at least 1.5x as many rows as resident one-CTA
// clusters, rows of at most kWsChunks chunks, no forced cluster size): one-CTA clusters fill
// every resident slot and take tickets -- whole rows first, then half-row blocks of the last
// rows (half as many as CTAs), whose pieces are merged through the workspace; the blocks absorb
// the spread of the CTAs' finishing times.  Smaller batches keep the fixed schedule: measured on
// B200 at V = 248,320 (256 to 1,500 rows), splitting them gained no bandwidth for the argmax and
// less than the merges cost for the sampler, while 2,304 rows gained 1-3%.  With a forced CTA
// count (test hook) every batch takes this path, split rows included.
template <typename T, bool kSample, bool kBulk, int kStages>
bool launch_dynamic(SelectParams& p, const KernelInfo& info, cudaLaunchConfig_t& cfg) {
    constexpr int kTPC = Layout<T>::kTokensPerChunk;
    const int64_t n = (p.vocab + kTPC - 1) / kTPC;
    if (p.ws == nullptr || p.partials != nullptr || g_force_cluster != 0 || n > kWsChunks) return false;
    int64_t grid = info.max_clusters[0];
    if (g_force_clusters > 0 && g_force_clusters < grid) grid = g_force_clusters;
    else if (!p.dynamic_always && 2 * p.rows < 3 * grid) return false;
    int64_t split, block;
    if (p.rows <= grid) {
        split = p.rows;
        block = (split * n + grid - 1) / grid;
    } else {
        split = grid / 2 > 1 ? grid / 2 : 1;
        block = (n + 1) / 2;
    }
    if (split > p.ws_rows) split = p.ws_rows;
    block = block < 4 ? 4 : block > kWsChunks ? kWsChunks : block;
    const int64_t split_chunks = split * n;
    p.whole_rows = p.rows - split;
    p.block = static_cast<int32_t>(block);
    p.tickets = p.whole_rows + (split_chunks + block - 1) / block;
    p.segment = (p.vocab + 31) / 32 * 32;
    uint32_t e = ++g_epoch;
    if (e == 0) e = ++g_epoch;
    p.epoch = e;
    const int64_t ctas = p.tickets < grid ? p.tickets : grid;
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    return true;
}

// Flat schedule of sampler batches with fewer than 1.5 rows per resident CTA (a workspace with
// the flat-record area is given, rows of at most kWsChunks chunks, no forced launch shape).  The
// batch's chunks, in row-major order, are taken as tickets by one-CTA clusters filling every
// resident slot, every ticket from the counter (a CTA that starts late owns no block); tickets
// shrink by tier -- one block per CTA of about 60 % of its even share, one of about 20 %, then
// blocks of two chunks (single chunks when the batch has no more chunks than CTAs) -- so that
// most chunks stream in long pieces and SMs streaming at different speeds still finish together.
// Consumer warps store one record per (chunk, warp) granule to the workspace and hand nothing over
// at a piece boundary; a second launch (flat_merge_kernel) merges and walks every row in parallel.
//
// Measured on B200 (configuration-2 rows, fp16, 31 chunks per row, CUDA events, back to back),
// flat against the fixed schedule: 8 / 64 / 148 / 200 / 256 / 300 rows 12.8 / 19.1 / 28.2 / 33.3 /
// 39.0 / 42.5 us against 15.9 / 28.7 / 29.5 / 38.9 / 39.2 / 50.1 us; 480 / 600 rows 58.6 / 69.2 us
// against 64.5 / 76.4 us on a two-launch split schedule.  A batch of one row per resident CTA
// streams faster on the fixed schedule (444 rows: 50.9 against 55.9 us): up to one row per
// resident CTA the flat schedule runs where its cost, about 13.2 us + 0.47 us x chunks / SMs, is
// below the fixed schedule's, about 18.6 us + 0.34 us x chunks per row x ceil(rows / SMs).
constexpr int64_t kFlatTierPct[2] = {60, 20};
constexpr int64_t kFlatSmallBlock = 2;

template <typename T, bool kSample, bool kBulk, int kStages>
bool launch_flat(SelectParams& p, const KernelInfo& info, cudaLaunchConfig_t& cfg) {
    constexpr int kTPC = Layout<T>::kTokensPerChunk;
    const int64_t n = (p.vocab + kTPC - 1) / kTPC;
    const int64_t grid = info.flat_ctas;
    if (!kSample || !kBulk || grid <= 0 || p.ws == nullptr || !p.ws_flat || p.partials != nullptr || p.dynamic_always ||
        g_force_cluster != 0 || g_force_clusters != 0 || n > kWsChunks || p.rows > p.ws_rows || 2 * p.rows >= 3 * grid)
        return false;
    const int64_t chunks = p.rows * n;
    const int64_t sms = info.sms;
    if (p.rows <= grid && 2 * p.rows >= sms) {
        const double flat_us = 13.2 + 0.47 * static_cast<double>(chunks) / static_cast<double>(sms);
        const double fixed_us = 18.6 + 0.34 * static_cast<double>(n) * static_cast<double>((p.rows + sms - 1) / sms);
        if (fixed_us <= flat_us) return false;
    }
    const int64_t small = chunks <= grid ? 1 : kFlatSmallBlock;
    int64_t rem = chunks, tickets = 0;
    for (int i = 0; i < 2; ++i) {
        int64_t b = chunks * kFlatTierPct[i] / (100 * grid);
        if (b < small) b = small;
        int64_t t = rem / b;
        if (t > grid) t = grid;
        p.tier_block[i] = static_cast<int32_t>(b);
        p.tier_tickets[i] = t;
        rem -= t * b;
        tickets += t;
    }
    tickets += (rem + small - 1) / small;
    p.flat = 1;
    p.whole_rows = 0;
    p.block = static_cast<int32_t>(small);
    p.tickets = tickets;
    p.segment = (p.vocab + 31) / 32 * 32;
    uint32_t e = ++g_epoch;
    if (e == 0) e = ++g_epoch;
    p.epoch = e;
    cfg.gridDim = dim3(static_cast<unsigned>(tickets < grid ? tickets : grid));
    return true;
}

template <typename T, bool kSample, bool kBulk, int kStages>
int launch_select_t(SelectParams p, int device, cudaStream_t stream) {
    KernelInfo* info = nullptr;
    BMS_CHECK((kernel_info<T, kSample, kBulk, kStages>(device, info)));
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t cfg = {};
        if (launch_flat<T, kSample, kBulk, kStages>(p, *info, cfg)) {
            if constexpr (kSample && kBulk) {
                cfg.blockDim = dim3(kThreads);
                cfg.dynamicSmemBytes = select_smem_bytes<T, kSample>(kStages);
                cfg.stream = stream;
                const bool full = static_cast<int>(cfg.gridDim.x) >= info->flat_ctas;
                cfg.attrs = pdl;
                cfg.numAttrs = full ? 1 : 0;
                BMS_CUDA(cudaLaunchKernelEx(&cfg, select_rows_kernel<T, true, true, kStages, true>, p), "selection launch");
                cudaLaunchConfig_t mcfg = {};
                const int64_t cap = static_cast<int64_t>(info->sms) * 8;
                mcfg.gridDim = dim3(static_cast<unsigned>(p.rows < cap ? p.rows : cap));
                mcfg.blockDim = dim3(kFlatMergeWarps * 32);
                mcfg.stream = stream;
                mcfg.attrs = pdl;
                mcfg.numAttrs = 1;
                BMS_CUDA(cudaLaunchKernelEx(&mcfg, flat_merge_kernel<T>, p), "flat merge launch");
                return BMS_SUCCESS;
            }
        }
    }
    {
        cudaLaunchConfig_t cfg = {};
        if (launch_dynamic<T, kSample, kBulk, kStages>(p, *info, cfg)) {
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = select_smem_bytes<T, kSample>(kStages);
            cfg.stream = stream;
            const bool full = static_cast<int>(cfg.gridDim.x) >= info->max_clusters[0];
            cfg.attrs = pdl;
            cfg.numAttrs = full ? 1 : 0;
            BMS_CUDA(cudaLaunchKernelEx(&cfg, select_rows_kernel<T, kSample, kBulk, kStages>, p), "selection launch");
            return BMS_SUCCESS;
        }
        p.ws = nullptr;
    }
    const Plan plan = plan_launch(*info, p.rows, p.vocab, Layout<T>::kTokensPerChunk, kSample ? kMaxChunksSampler : 0,
                                  kSample, p.partials != nullptr);
    if (plan.cluster == 0)
        return fail(BMS_ERROR_UNSUPPORTED, "vocabulary of %lld tokens exceeds the %s limit", static_cast<long long>(p.vocab),
                    kSample ? "sampler" : "selection");
    p.segment = plan.segment;
    cudaLaunchConfig_t cfg = {};
    // Programmatic dependent launch: CTAs may be dispatched and initialise their barriers while
    // the previous grid in the stream finishes its row-end work (the previous grid signals once
    // all its CTAs streamed their last chunk; this one waits for its completion before touching
    // memory).  A launch without a cluster dimension is a grid of one-CTA clusters.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = plan.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(plan.cluster * plan.clusters));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = select_smem_bytes<T, kSample>(kStages);
    cfg.stream = stream;
    // A grid that fills every resident slot, or one of at most one CTA per SM, hides its launch
    // behind its predecessor's row-end work.  Grids in between, dispatched early into the slots
    // their predecessor leaves free, would be spread unevenly over the SMs (measured on B200:
    // 256 sampler rows 48 instead of 40 us).
    const bool full = plan.clusters >= info->max_clusters[cluster_index(plan.cluster)] ||
                      plan.cluster * plan.clusters <= info->sms;
    cfg.attrs = full ? attr : attr + 1;
    cfg.numAttrs = (full ? 1 : 0) + (plan.cluster > 1 ? 1 : 0);
    BMS_CUDA(cudaLaunchKernelEx(&cfg, select_rows_kernel<T, kSample, kBulk, kStages>, p), "selection launch");
    return BMS_SUCCESS;
}

// Ring depth: 4 stages for the argmax (3 CTAs/SM fit), 3 for the sampler, whose granule tables
// also live in shared memory (3 CTAs/SM as well).
template <bool kSample>
constexpr int bulk_stages() { return kSample ? 3 : 4; }

template <typename T, bool kSample>
int launch_select_dtype(SelectParams p, int device, cudaStream_t stream) {
    const int eb = sizeof(T);
    const bool bulk = reinterpret_cast<uintptr_t>(p.logits) % 16 == 0 && reinterpret_cast<uintptr_t>(p.masks) % 16 == 0 &&
                      (p.vocab * eb) % 16 == 0 && (p.logit_stride * eb) % 16 == 0 && p.mask_stride % 4 == 0;
    if (bulk) return launch_select_t<T, kSample, true, bulk_stages<kSample>()>(p, device, stream);
    return launch_select_t<T, kSample, false, 1>(p, device, stream);
}

template <bool kSample>
int launch_select(int dtype, const SelectParams& p, int device, cudaStream_t stream) {
    if (p.rows == 0) return BMS_SUCCESS;
    switch (dtype) {
        case BMS_FLOAT32: return launch_select_dtype<float, kSample>(p, device, stream);
        case BMS_BFLOAT16: return launch_select_dtype<__nv_bfloat16, kSample>(p, device, stream);
        default: return launch_select_dtype<__half, kSample>(p, device, stream);
    }
}

// ---------------------------------------------------------------- popcount / density / budget
__device__ int32_t policy_budget(const bms_policy& P, double d) {
    if (P.kind == 0) {
        if (d < P.low_density) return P.max_budget;
        if (d < P.high_density) return (P.min_budget + P.max_budget) / 2;
        return P.min_budget;
    }
    if (d < P.low_density) return P.max_budget;
    if (d > P.high_density) return P.min_budget;
    const double span = static_cast<double>(P.max_budget - P.min_budget);
    const double frac = __ddiv_rn(__dsub_rn(d, P.low_density), __dsub_rn(P.high_density, P.low_density));
    return P.max_budget - static_cast<int32_t>(floor(__dmul_rn(span, frac)));
}

// One CTA per row (grid-stride): popcount with the padding bits of the last word cleared.
__global__ void __launch_bounds__(256) count_rows_kernel(const int32_t* __restrict__ masks, int64_t rows, int64_t vocab,
                                                         bms_policy policy, int64_t* __restrict__ counts,
                                                         double* __restrict__ density, int32_t* __restrict__ budget) {
    __shared__ uint32_t part[8];
    const int64_t words = (vocab + 31) / 32;
    const int tail = static_cast<int>(vocab % 32);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const int32_t* m = masks + row * words;
        uint32_t c = 0;
        for (int64_t w = threadIdx.x; w < words; w += blockDim.x) {
            uint32_t bits = static_cast<uint32_t>(m[w]);
            if (w == words - 1 && tail != 0) bits &= (1u << tail) - 1u;
            c += __popc(bits);
        }
        c = __reduce_add_sync(0xFFFFFFFFu, c);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t total = 0;
            for (int i = 0; i < 8; ++i) total += part[i];
            if (counts) counts[row] = total;
            const double d = __ddiv_rn(static_cast<double>(total), static_cast<double>(vocab));
            if (density) density[row] = d;
            if (budget) budget[row] = policy_budget(policy, d);
        }
        __syncthreads();
    }
}

// Token-ID lists to packed mask rows, one CTA per list (grid-stride): the row is cleared, then the
// listed tokens' bits are set (atomicOr: a list may repeat IDs or be unsorted).  List l is
// ids[offsets[l], offsets[l + 1]), clamped to [0, n_ids) so that no offsets can reach outside
// `ids`; IDs outside [0, vocab) set nothing and flag the list in `bad` (nullable).
__global__ void __launch_bounds__(256) expand_lists_kernel(const int32_t* __restrict__ ids, int64_t n_ids,
                                                           const int32_t* __restrict__ offsets, int64_t lists,
                                                           int64_t vocab, int32_t* __restrict__ out,
                                                           int32_t* __restrict__ bad) {
    const int64_t words = (vocab + 31) / 32;
    for (int64_t l = blockIdx.x; l < lists; l += gridDim.x) {
        uint32_t* row = reinterpret_cast<uint32_t*>(out) + l * words;
        for (int64_t w = threadIdx.x; w < words; w += blockDim.x) row[w] = 0u;
        __syncthreads();  // the cleared words before any bit of this CTA is set
        int64_t b = offsets[l], e = offsets[l + 1];
        b = b < 0 ? 0 : b > n_ids ? n_ids : b;
        e = e < b ? b : e > n_ids ? n_ids : e;
        int flag = 0;
        for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
            const int64_t t = ids[i];
            if (t >= 0 && t < vocab) atomicOr(row + (t >> 5), 1u << (t & 31));
            else flag = 1;
        }
        flag = __syncthreads_or(flag);
        if (bad != nullptr && threadIdx.x == 0) bad[l] = flag;
    }
}

// Gap-stream expansion (bms_expand_token_gaps): row l of `out` ([rows, ceil(vocab / 32)] words)
// becomes the packed mask of the token IDs coded by the byte stream
// bytes[offsets[l], offsets[l + 1]) (clamped to [0, n_bytes]); starting before token 0, a byte b > 0
// advances b tokens and allows the token reached, a byte 0 advances 255 tokens and allows nothing.
// Tokens at or past `vocab` set nothing and flag the row in `bad` (nullable).
//
// One CTA per row builds the row's bitmap in shared memory: the stream is read in tiles of 4,096
// bytes (thread t takes bytes [16t, 16t + 16) of a tile, so that every warp load covers 512
// contiguous bytes), a block scan of the threads' summed advances gives each thread its starting
// token, and the bits go in with shared-memory atomicOr; the finished row is written out with
// coalesced word stores.  Rows whose bitmap does not fit kGapSmemBytes use expand_gaps_atomic_kernel.
constexpr int kGapThreads = 256;
constexpr int kGapTile = 16 * kGapThreads;
constexpr int64_t kGapSmemBytes = 160 * 1024;

__global__ void __launch_bounds__(kGapThreads) expand_gaps_kernel(const uint8_t* __restrict__ bytes, int64_t n_bytes,
                                                                  const int32_t* __restrict__ offsets, int64_t rows,
                                                                  int64_t vocab, int32_t* __restrict__ out,
                                                                  int32_t* __restrict__ bad) {
    extern __shared__ uint32_t sbits[];
    __shared__ long long warp_sums[kGapThreads / 32];
    const int64_t words = (vocab + 31) / 32;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    for (int64_t l = blockIdx.x; l < rows; l += gridDim.x) {
        for (int64_t w = tid; w < words; w += kGapThreads) sbits[w] = 0u;
        int64_t b = offsets[l], e = offsets[l + 1];
        b = b < 0 ? 0 : b > n_bytes ? n_bytes : b;
        e = e < b ? b : e > n_bytes ? n_bytes : e;
        __syncthreads();  // the cleared bitmap before any bit is set
        long long base = -1;  // token reached before the tile
        int flag = 0;
        for (int64_t t0 = b; t0 < e; t0 += kGapTile) {
            const int64_t s0 = t0 + 16 * static_cast<int64_t>(tid);
            uint32_t c[16];
            long long local = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const bool in = s0 + j < e;
                c[j] = in ? static_cast<uint32_t>(bytes[s0 + j]) : 1u;
                local += in ? (c[j] ? c[j] : 255u) : 0u;
            }
            long long v = local;  // block inclusive scan: warps, then the warp totals
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long n = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += n;
            }
            if (lane == 31) warp_sums[wid] = v;
            __syncthreads();
            long long pos = base + v - local, total = 0;
#pragma unroll
            for (int w = 0; w < kGapThreads / 32; ++w) {
                const long long ws = warp_sums[w];
                if (w < wid) pos += ws;
                total += ws;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                if (s0 + j >= e) break;
                pos += c[j] ? c[j] : 255u;
                if (c[j]) {
                    if (pos < vocab) atomicOr(&sbits[pos >> 5], 1u << (pos & 31));
                    else flag = 1;
                }
            }
            base += total;
            __syncthreads();  // every thread read warp_sums before the next tile writes it
        }
        flag = __syncthreads_or(flag);  // also: every bit is set
        int32_t* row = out + l * words;
        for (int64_t w = tid; w < words; w += kGapThreads) row[w] = static_cast<int32_t>(sbits[w]);
        if (bad != nullptr && tid == 0) bad[l] = flag;
        __syncthreads();  // the bitmap is read out before the next row clears it
    }
}

// The same expansion for bitmaps larger than kGapSmemBytes: each thread decodes one contiguous
// segment of the stream, a block scan of the segment advances gives every segment's starting
// token, and the bits go into the cleared row with global atomicOr.
__global__ void __launch_bounds__(256) expand_gaps_atomic_kernel(const uint8_t* __restrict__ bytes, int64_t n_bytes,
                                                          const int32_t* __restrict__ offsets, int64_t rows,
                                                          int64_t vocab, int32_t* __restrict__ out,
                                                          int32_t* __restrict__ bad) {
    __shared__ long long warp_sums[8];
    const int64_t words = (vocab + 31) / 32;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    for (int64_t l = blockIdx.x; l < rows; l += gridDim.x) {
        uint32_t* row = reinterpret_cast<uint32_t*>(out) + l * words;
        for (int64_t w = tid; w < words; w += blockDim.x) row[w] = 0u;
        int64_t b = offsets[l], e = offsets[l + 1];
        b = b < 0 ? 0 : b > n_bytes ? n_bytes : b;
        e = e < b ? b : e > n_bytes ? n_bytes : e;
        const int64_t per = (e - b + blockDim.x - 1) / blockDim.x;
        const int64_t s0 = b + tid * per < e ? b + tid * per : e;
        const int64_t s1 = s0 + per < e ? s0 + per : e;
        long long local = 0;
        for (int64_t i = s0; i < s1; ++i) {
            const uint32_t c = bytes[i];
            local += c ? c : 255u;
        }
        long long v = local;  // inclusive scan: warps, then the 8 warp totals
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long n = __shfl_up_sync(0xFFFFFFFFu, v, o);
            if (lane >= o) v += n;
        }
        if (lane == 31) warp_sums[wid] = v;
        __syncthreads();  // also orders the cleared words before any bit is set
        long long pos = -1 + v - local;
        for (int w = 0; w < wid; ++w) pos += warp_sums[w];
        int flag = 0;
        for (int64_t i = s0; i < s1; ++i) {
            const uint32_t c = bytes[i];
            pos += c ? c : 255u;
            if (c) {
                if (pos < vocab) atomicOr(row + (pos >> 5), 1u << (pos & 31));
                else flag = 1;
            }
        }
        flag = __syncthreads_or(flag);
        if (bad != nullptr && tid == 0) bad[l] = flag;
    }
}

// ---------------------------------------------------------------- stochastic speculative acceptance
// Row normaliser of a sampler partial (one rank covering the whole row): the partial's reference
// max M and the row's mass S relative to it, or a status code for rows that cannot be sampled
// (the sampler's codes and priority, merge_sampler_ranks).
struct RowNorm {
    float M;
    double S;
    int32_t code;
    double invS;  // 1 / S, so that each weight costs a multiply, not a division
};

__device__ __forceinline__ RowNorm row_norm(const GatherSlot& g) {
    const float kInf = __int_as_float(0x7F800000);
    RowNorm r{__uint_as_float(g.a), g.s, kOk, g.s > 0.0 ? 1.0 / g.s : 0.0};
    r.code = (g.c & kFlagAbort) ? kTimeout : (g.c & kFlagNaN) ? kNaN : (r.M == kInf) ? kPosInf : (g.b == 0u) ? kEmpty
             : (r.M == -kInf || !(r.S > 0.0)) ? kNoMass : kOk;
    return r;
}

// Unnormalised weight of logit x in a row of maximum M: 2^((x - M) log2(e) / T) (fp32).  x == M
// gives exactly 1 whatever the scale.
__device__ __forceinline__ float spec_exp(float x, float M, float sc) {
    const float d = x - M;
    return ptx::ex2(d == 0.0f ? 0.0f : fminf(d * sc, 126.0f));
}

// Weight of logit x relative to a row normaliser: 2^((x - M) log2(e) / T) / S (fp32 exponential,
// fp64 quotient).  x == M gives exactly 1 / S whatever the scale.
__device__ __forceinline__ double spec_weight(float x, const RowNorm& n, float sc) {
    return static_cast<double>(spec_exp(x, n.M, sc)) * n.invS;
}

// Weights of tokens [a, a + 8) of the sampled row in the row's own units -- inverse-CDF sampling
// needs only relative masses: e_t = 2^((x - M_t) sc), or in the residual pass max(0, e_t - ratio
// e_q) with ratio = S_t / S_q (then p - q = that / S_t).  fp32 throughout, two tokens per f32x2
// instruction: ratio is split into rhi + rlo and applied by two FMAs, whose roundings are relative
// to the residual itself, so p - q stays accurate to about 1e-7 even where p and q nearly cancel.
// Tokens outside the mask or past the vocabulary weigh 0 (selected, so whatever a masked logit
// gives never enters a sum); a valid token has x <= M (M is the row's masked maximum), so its
// exponent needs no clamp, and the host keeps sc finite, so x == M gives exactly 1.
template <bool kRes>
__device__ __forceinline__ void row_weights8(int64_t a, int64_t vocab, uint32_t bits, const float (&xt)[8],
                                             const float (&xq)[8], float Mt, float Mq, float sc, float rhi,
                                             float rlo, float (&w)[8]) {
    if (a + 8 > vocab) bits &= a < vocab ? (1u << (vocab - a)) - 1u : 0u;
    const uint64_t sc2 = ptx::pack2(sc, sc), nmt = ptx::pack2(-Mt, -Mt);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        float t0, t1;
        ptx::unpack2(ptx::mul2(ptx::add2(ptx::pack2(xt[i], xt[i + 1]), nmt), sc2), t0, t1);
        float e0 = ptx::ex2(t0), e1 = ptx::ex2(t1);
        if constexpr (kRes) {
            float q0, q1;
            ptx::unpack2(ptx::mul2(ptx::add2(ptx::pack2(xq[i], xq[i + 1]), ptx::pack2(-Mq, -Mq)), sc2), q0, q1);
            const uint64_t eq = ptx::pack2(ptx::ex2(q0), ptx::ex2(q1));
            const uint64_t r = ptx::fma2(ptx::pack2(-rlo, -rlo), eq,
                                         ptx::fma2(ptx::pack2(-rhi, -rhi), eq, ptx::pack2(e0, e1)));
            ptx::unpack2(r, e0, e1);
            e0 = fmaxf(0.0f, e0);
            e1 = fmaxf(0.0f, e1);
        }
        w[i] = ((bits >> i) & 1u) ? e0 : 0.0f;
        w[i + 1] = ((bits >> (i + 1)) & 1u) ? e1 : 0.0f;
    }
}

// ((w0 + w1) + (w2 + w3)) + ((w4 + w5) + (w6 + w7)), the two halves side by side.
__device__ __forceinline__ float sum8(const float (&w)[8]) {
    const uint64_t h = ptx::add2(ptx::add2(ptx::pack2(w[0], w[4]), ptx::pack2(w[1], w[5])),
                                 ptx::add2(ptx::pack2(w[2], w[6]), ptx::pack2(w[3], w[7])));
    float lo, hi;
    ptx::unpack2(h, lo, hi);
    return lo + hi;
}

// Tokens [a, a + 8) of a row as floats (0 past `vocab`): one or two 16-byte loads when the row is
// 16-byte aligned (`vec`), else scalar loads.  No branch on the mask, so the loads of several
// calls can be in flight together.
template <typename T>
__device__ __forceinline__ void load8(const T* row, int64_t a, int64_t vocab, bool vec, float (&x)[8]) {
    using E = Elem<T>;
    if (vec && a + 8 <= vocab) {
        if constexpr (E::kBytes == 2) {
            const uint4 r = __ldg(reinterpret_cast<const uint4*>(row + a));
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                x[2 * i] = E::lo(w[i]);
                x[2 * i + 1] = E::hi(w[i]);
            }
        } else {
            const float4 p0 = __ldg(reinterpret_cast<const float4*>(row + a));
            const float4 p1 = __ldg(reinterpret_cast<const float4*>(row + a) + 1);
            x[0] = p0.x; x[1] = p0.y; x[2] = p0.z; x[3] = p0.w;
            x[4] = p1.x; x[5] = p1.y; x[6] = p1.z; x[7] = p1.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = a + i < vocab ? E::load(row, a + i) : 0.0f;
    }
}

// Tokens [a, a + 8) of a 16-byte aligned row as raw 16-byte vectors: issuing the loads of several
// tiles before any of them is decoded keeps them in flight together.
template <typename T>
struct Pack8 {
    uint4 w[Elem<T>::kBytes / 2];
};

template <typename T>
__device__ __forceinline__ void fetch8(const T* row, int64_t a, Pack8<T>& p) {
    const uint4* src = reinterpret_cast<const uint4*>(row + a);
#pragma unroll
    for (int i = 0; i < Elem<T>::kBytes / 2; ++i) p.w[i] = __ldg(src + i);
}

template <typename T>
__device__ __forceinline__ void unpack8(const Pack8<T>& p, float (&x)[8]) {
    using E = Elem<T>;
#pragma unroll
    for (int i = 0; i < E::kBytes / 2; ++i) {
        float v[E::kVec];
        E::decode(p.w[i], v);
#pragma unroll
        for (int k = 0; k < E::kVec; ++k) x[i * E::kVec + k] = v[k];
    }
}

// Online normaliser of a row's valid tokens, 8 consecutive logits at a time: m is the lane's running
// maximum, s the mass 2^((x - m) sc) of its tokens so far (fp64; each group of 8 summed in fp32
// first).  Invalid tokens enter as -inf.  A NaN or +inf valid logit leaves s meaningless; the row's
// status reports it.
__device__ __forceinline__ void norm_update8(const float (&x)[8], uint32_t bits, float sc, float& m, double& s) {
    const float kInf = __int_as_float(0x7F800000);
    float v[8];
    float tmax = -kInf;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = ((bits >> i) & 1u) ? x[i] : -kInf;
        tmax = fmaxf(tmax, v[i]);
    }
    if (tmax > m) {
        s *= static_cast<double>(ptx::ex2((m - tmax) * sc));
        m = tmax;
    }
    if (m > -kInf && m < kInf) {
        const uint64_t sc2 = ptx::pack2(sc, sc), nm = ptx::pack2(-m, -m);
        float w[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            float t0, t1;
            ptx::unpack2(ptx::mul2(ptx::add2(ptx::pack2(v[i], v[i + 1]), nm), sc2), t0, t1);
            w[i] = ptx::ex2(t0);
            w[i + 1] = ptx::ex2(t1);
        }
        s += static_cast<double>(sum8(w));
    }
}

// Merge of two (maximum, mass relative to it) parts of a row into (m, s).
__device__ __forceinline__ void norm_merge(float& m, double& s, float m2, double s2, float sc) {
    const float kInf = __int_as_float(0x7F800000);
    const float M = fmaxf(m, m2);
    const double a = m > -kInf ? s * static_cast<double>(ptx::ex2((m - M) * sc)) : 0.0;
    const double b = m2 > -kInf ? s2 * static_cast<double>(ptx::ex2((m2 - M) * sc)) : 0.0;
    m = M;
    s = a + b;
}

// Acceptance tests of one sequence (one warp, 32 drafts per pass): the first position j whose
// draft is rejected (u_i q_i(d_i) >= p_i(d_i), a token outside the mask or a row that cannot be
// sampled), or L when all L drafts are accepted, and the status of that position's rows.
template <typename T>
__device__ void accept_prefix(const T* __restrict__ target, const T* __restrict__ draft,
                              const int32_t* __restrict__ masks, int64_t seq, int64_t rows_per_seq, int64_t vocab,
                              const int64_t* __restrict__ proposals, int32_t L, const GatherSlot* __restrict__ tpart,
                              const GatherSlot* __restrict__ qpart, const double* __restrict__ u_accept, float sc,
                              int lane, int32_t& j_out, int32_t& code_out) {
    using E = Elem<T>;
    const int64_t K = rows_per_seq - 1, words = (vocab + 31) / 32;
    int32_t j = -1, code = kOk;
    if (L < 0 || L > K) {
        j = 0;
        code = kBadLength;
    }
    for (int64_t i0 = 0; j < 0 && i0 < L; i0 += 32) {
        const int64_t i = i0 + lane;
        bool stop = false;
        int32_t c = kOk;
        if (i < L) {
            const int64_t trow = seq * rows_per_seq + i, qrow = seq * K + i;
            const RowNorm tn = row_norm(tpart[trow]), qn = row_norm(qpart[qrow]);
            c = tn.code != kOk ? tn.code : qn.code;
            const int64_t d = proposals[seq * K + i];
            bool ok = false;
            if (c == kOk && d >= 0 && d < vocab &&
                ((static_cast<uint32_t>(masks[trow * words + (d >> 5)]) >> (d & 31)) & 1u)) {
                const double p = spec_weight(E::load(target, trow * vocab + d), tn, sc);
                const double q = spec_weight(E::load(draft, qrow * vocab + d), qn, sc);
                ok = q > 0.0 && u_accept[seq * K + i] * q < p;
            }
            stop = c != kOk || !ok;
        }
        const uint32_t ballot = __ballot_sync(0xFFFFFFFFu, stop);
        if (ballot) {
            const int f = __ffs(ballot) - 1;
            j = static_cast<int32_t>(i0 + f);
            code = __shfl_sync(0xFFFFFFFFu, c, f);
        }
    }
    j_out = j < 0 ? L : j;
    code_out = code;
}

constexpr int kAcceptCluster = 8;  // CTAs per sequence at most (a portable cluster)
// Acceptance CTAs have kAccWarps warps.  Streamed, each CTA's range of the sampled row arrives in
// chunks of kAccRowBytes per row (target, and the draft in the residual pass; two 256-token tiles
// per warp of 16-bit logits, one of fp32) plus the chunk's mask words, kAccStages chunks in flight
// by 1-D bulk copies.
constexpr int kAccWarps = 16;  // 2 CTAs per SM (64 registers streamed): 32 warps
constexpr int kAccThreads = 32 * kAccWarps;
constexpr int kAccStages = 3;
constexpr int kAccRowBytes = 1024 * kAccWarps;
constexpr int kAccStageBytes = 2 * kAccRowBytes + kAccRowBytes / 16;

// Speculative sampling for S sequences, one cluster of kAcceptCluster CTAs each.  Sequence s has
// lengths[s] = L drafts proposals[s, i] drawn from the draft's masked softmax q_i (draft row
// s * (R - 1) + i), and target rows s * R + i giving p_i (R = rows per sequence, both under mask row
// s * R + i).  Draft i is accepted iff u_i q_i(d_i) < p_i(d_i) (probability min(1, p / q)); at the
// first rejection j the replacement is drawn by inverse CDF with v_s from max(0, p_j - q_j)
// normalised, and after L acceptances the bonus from p_L -- so every emitted token is distributed
// as the target's masked softmax.  A replacement distribution that rounds to zero mass falls back to
// p_j.  Outputs: the accepted length, the drawn token, its kind (0 replacement, 1 bonus, 2 fallback
// for L = 0) and a status, nonzero when a row the procedure consumed cannot be sampled.
//
// Every CTA of the cluster (1, 2, 4 or 8 CTAs, chosen by the host from the batch size) runs the
// (cheap) acceptance tests itself; the sampled row is split into one contiguous range of 256-token
// tiles per CTA.  Each CTA sums its tiles (a warp per tile, 8 consecutive tokens per lane) -- with
// kStream, from shared-memory stages that thread 0 fills with 1-D bulk copies (kAccStages chunks in
// flight, so the bytes in flight cost no registers); without (rows or mask rows not 16-byte
// aligned), from global memory, four tiles' loads per warp issued together.  It pushes its total
// to every CTA of the cluster (st.shared::cluster) and, after a cluster barrier, every CTA knows
// the mass before its range and the total; the CTA whose range holds v * total (or, after
// rounding, the last CTA with mass) scans its tile sums, walks the tile and pushes the token to
// every CTA.  Every CTA of a cluster takes the same path and the same barriers (uniform decisions
// from the same pushed values), so the hardware cluster barriers always complete.  A stage wait
// that gives up (bounded, about a second) latches an abort: the CTA pushes the flag with its total,
// the cluster reports kTimeout for the sequence, and the CTA lets its copies land before it exits.
//
// kLazy (streamed only; tpart and qpart unused): the row normalisers are computed here, only for the
// positions the procedure consumes.  For i = 0, 1, ... the cluster streams target row i and draft
// row i (only the target row at i = L), each CTA keeping an online (max, mass) per lane, reduces
// them per CTA and exchanges them over distributed shared memory (identical merges in every CTA),
// and tests draft i -- stopping at the first rejection, so a round reads the rows up to the first
// rejection plus the sampled row again, not all 2K + 1 rows.  Thread 0 reads the test's inputs
// (the draft token, its mask bit, both logits, the uniform) while the rows stream.  The statuses
// follow the sampler partials: NaN anywhere in the row, a +inf valid logit, no valid token, no
// finite mass.
template <typename T, bool kStream, bool kLazy = false>
__global__ void __launch_bounds__(kAccThreads, kStream ? 2 : 1) speculative_accept_kernel(
    const T* __restrict__ target, const T* __restrict__ draft, const int32_t* __restrict__ masks, int64_t seqs,
    int64_t rows_per_seq, int64_t vocab, const int64_t* __restrict__ proposals, const int32_t* __restrict__ lengths,
    const GatherSlot* __restrict__ tpart, const GatherSlot* __restrict__ qpart, const double* __restrict__ u_accept,
    const double* __restrict__ u_resample, float sc, int32_t* __restrict__ accept_len, int64_t* __restrict__ token,
    int32_t* __restrict__ kind, int32_t* __restrict__ status) {
    __shared__ double sums[kAccWarps];
    extern __shared__ __align__(128) uint8_t accept_smem[];  // [kStream: stages] [this CTA's tile sums]
    double* tile_sums = reinterpret_cast<double*>(accept_smem + (kStream ? kAccStages * kAccStageBytes : 0));
    __shared__ __align__(8) uint64_t s_full[kAccStages];  // a stage's chunk has landed
    __shared__ __align__(8) uint64_t s_empty[kAccStages]; // every warp has read a stage's chunk
    __shared__ uint32_t s_issued[kAccStages];             // chunks issued into each stage
    __shared__ int32_t s_abort;                           // a stage wait gave up (latched)
    __shared__ uint4 s_rank[kAcceptCluster];   // per CTA of the cluster: its mass (two words), positive
    __shared__ uint4 s_pick;                   // the owning CTA's token (two words)
    __shared__ int32_t s_j, s_code, s_last, s_cut_past, s_claim;
    __shared__ int64_t s_token, s_tile;
    __shared__ double s_prefix;
    // kLazy: per CTA of the cluster its normalisers {Mt, count, flags, Mq}, {St, Sq}, by pass parity
    // (see npass below); the draft test's inputs by pass parity; per-warp partial normalisers.
    __shared__ uint4 s_norm[kLazy ? 2 : 1][kAcceptCluster][2];
    __shared__ double s_tu[2];
    __shared__ float s_txt[2], s_txq[2];
    __shared__ int32_t s_tbit[2];
    __shared__ float s_wm[2][kAccWarps];
    __shared__ double s_ws[2][kAccWarps];
    __shared__ uint32_t s_wcnt[kAccWarps], s_wfl[kAccWarps];
    static_assert(!kLazy || kStream, "lazy normalisers stream their rows");
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t crank = ptx::cluster_ctarank(), csize = ptx::cluster_nctarank();
    const int64_t K = rows_per_seq - 1, words = (vocab + 31) / 32;
    const int64_t ntiles = (vocab + 255) / 256;
    const int64_t per_rank = (ntiles + csize - 1) / csize;
    const int64_t r0 = min(ntiles, static_cast<int64_t>(crank) * per_rank), r1 = min(ntiles, r0 + per_rank);
    const int64_t nt = r1 - r0;  // tiles of this CTA
    // 16-byte loads need 16-byte aligned rows (row starts at multiples of vocab elements).
    const bool vec = (reinterpret_cast<uintptr_t>(target) % 16 == 0) && (reinterpret_cast<uintptr_t>(draft) % 16 == 0) &&
                     ((vocab * sizeof(T)) % 16 == 0);
    if (tid == 0) {
        for (int s = 0; s < kAccStages; ++s) {
            ptx::mbar_init(ptx::smem_addr(&s_full[s]), 1);
            ptx::mbar_init(ptx::smem_addr(&s_empty[s]), kAccWarps);
            s_issued[s] = 0;
        }
        s_abort = 0;
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    uint32_t gbase = 0;  // chunks this CTA has streamed so far (every thread counts them alike)
    // kLazy: normaliser passes so far, over all sequences.  Pass n uses slot n & 1 of s_norm and of
    // the test inputs: a peer's push for pass n + 2 follows pass n + 1's cluster barrier, which every
    // thread reaches only after reading pass n's slot -- also when a sequence ends without a
    // sampling pass (and its two cluster barriers) before the next sequence's first push.
    uint32_t npass = 0;
    // kStream: streams this CTA's tokens [r0 * 256, min(r1 * 256, V)) of a target row -- with
    // `with_q` also of a draft row -- and their mask words through the stages, kTok tokens a chunk
    // (chunk c in stage (gbase + c) % kAccStages), and calls consume(stage, t0, ntc) in every warp
    // for every chunk (ntc = the chunk's 256-token tiles).  Every chunk starts on a tile; its byte
    // counts are multiples of 16 (the host streams only rows of a multiple of 16 bytes and mask rows
    // of a multiple of 4 words).  Thread 0 refills a stage once all warps have read its previous
    // chunk (the warps run up to kAccStages - 1 chunks apart; a warp ahead waits only on a full
    // barrier of a chunk already issued).  A wait that gives up latches s_abort.
    constexpr int64_t kTok = kAccRowBytes / sizeof(T);
    constexpr int kPerWarp = static_cast<int>(kTok / 256 / kAccWarps);  // tiles per warp and chunk: 2 (16-bit), 1
    static_assert(kPerWarp * 256 * kAccWarps == kTok, "a chunk is whole tiles per warp");
    auto stream_pass = [&](const T* rt, const T* rq, const int32_t* mr, bool with_q, auto&& consume) {
        const int64_t A = r0 * 256, B = min(r1 * 256, vocab);
        const int64_t n = B > A ? (B - A + kTok - 1) / kTok : 0;
        auto issue = [&](int64_t c) {
            const uint32_t G = gbase + static_cast<uint32_t>(c), st = G % kAccStages, use = G / kAccStages;
            if (use > 0 && !wait_bounded(ptx::smem_addr(&s_empty[st]), (use - 1u) & 1u, &s_abort)) return;
            const int64_t t0 = A + c * kTok, t1 = min(B, t0 + kTok);
            const uint32_t tb = static_cast<uint32_t>((t1 - t0) * static_cast<int64_t>(sizeof(T)));
            const uint32_t mb = static_cast<uint32_t>(((t1 + 31) / 32 - t0 / 32) * 4);
            const uint32_t bar = ptx::smem_addr(&s_full[st]);
            const uint32_t dst = ptx::smem_addr(accept_smem + st * kAccStageBytes);
            ptx::mbar_arrive_expect_tx(bar, tb * (with_q ? 2u : 1u) + mb);
            ptx::bulk_load(dst, rt + t0, tb, bar);
            if (with_q) ptx::bulk_load(dst + kAccRowBytes, rq + t0, tb, bar);
            ptx::bulk_load(dst + 2 * kAccRowBytes, mr + t0 / 32, mb, bar);
            ++s_issued[st];
        };
        if (tid == 0 && !s_abort)
            for (int64_t c = 0; c < n && c < kAccStages; ++c) issue(c);
        for (int64_t c = 0; c < n; ++c) {
            const uint32_t G = gbase + static_cast<uint32_t>(c), st = G % kAccStages;
            if (wait_bounded(ptx::smem_addr(&s_full[st]), (G / kAccStages) & 1u, &s_abort)) {
                const int64_t t0 = A + c * kTok;
                consume(static_cast<const uint8_t*>(accept_smem + st * kAccStageBytes), t0,
                        (min(B, t0 + kTok) - t0 + 255) / 256);
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(ptx::smem_addr(&s_empty[st]));
            if (tid == 0 && c + kAccStages < n && !s_abort) issue(c + kAccStages);
        }
        gbase += static_cast<uint32_t>(n);
    };
    for (int64_t seq = ptx::cluster_id_x(); seq < seqs; seq += ptx::ncluster_x()) {
        const int32_t L = lengths[seq];
        int32_t j = -1, code = kOk;
        RowNorm tn{0.0f, 1.0, kOk, 1.0}, qn{0.0f, 1.0, kOk, 1.0};
        bool residual0;
        if constexpr (kLazy) {
            const float kInf = __int_as_float(0x7F800000);
            if (L < 0 || L > K) {
                j = 0;
                code = kBadLength;
            }
            for (int32_t i = 0; j < 0; ++i) {
                const bool with_q = i < L;  // position L: the bonus row, target only
                const int slot = static_cast<int>(npass++ & 1u);
                const int64_t ti = seq * rows_per_seq + i, qi = seq * K + i;
                if (tid == 32 && with_q) {  // draft i's test inputs, read while the rows stream
                    const int64_t d = proposals[qi];
                    int32_t bit = 0;
                    float xt = 0.0f, xq = 0.0f;
                    if (d >= 0 && d < vocab) {
                        bit = static_cast<int32_t>((static_cast<uint32_t>(masks[ti * words + (d >> 5)]) >> (d & 31)) & 1u);
                        xt = Elem<T>::load(target, ti * vocab + d);
                        xq = Elem<T>::load(draft, qi * vocab + d);
                    }
                    s_tbit[slot] = bit;
                    s_txt[slot] = xt;
                    s_txq[slot] = xq;
                    s_tu[slot] = u_accept[qi];
                }
                float mt = -kInf, mq = -kInf;
                double stl = 0.0, sql = 0.0;
                uint32_t cnt = 0u;
                typename Elem<T>::NanAcc nant = Elem<T>::nan_init(), nanq = Elem<T>::nan_init();
                bool tnan = false, qnan = false;  // NaN among the row's last partial group
                stream_pass(target + ti * vocab, draft + qi * vocab, masks + ti * words, with_q,
                            [&](const uint8_t* stage, int64_t t0, int64_t ntc) {
#pragma unroll
                    for (int k = 0; k < kPerWarp; ++k) {
                        const int64_t tl = wid + kAccWarps * k;
                        const int64_t off = tl * 256 + 8 * lane, a = t0 + off;
                        if (tl < ntc && a < vocab) {
                            uint32_t bits =
                                (reinterpret_cast<const uint32_t*>(stage + 2 * kAccRowBytes)[off >> 5] >> (off & 31)) & 0xFFu;
                            const bool tail = a + 8 > vocab;
                            if (tail) bits &= (1u << (vocab - a)) - 1u;
                            cnt += __popc(bits);
                            Pack8<T> pk;
                            float x[8];
#pragma unroll
                            for (int w = 0; w < Elem<T>::kBytes / 2; ++w)
                                pk.w[w] = reinterpret_cast<const uint4*>(stage + off * sizeof(T))[w];
                            unpack8<T>(pk, x);
                            if (!tail) {
#pragma unroll
                                for (int w = 0; w < Elem<T>::kBytes / 2; ++w) Elem<T>::nan_update(nant, pk.w[w]);
                            } else {
                                for (int e = 0; e < 8; ++e) tnan |= a + e < vocab && x[e] != x[e];
                            }
                            norm_update8(x, bits, sc, mt, stl);
                            if (with_q) {
#pragma unroll
                                for (int w = 0; w < Elem<T>::kBytes / 2; ++w)
                                    pk.w[w] = reinterpret_cast<const uint4*>(stage + kAccRowBytes + off * sizeof(T))[w];
                                unpack8<T>(pk, x);
                                if (!tail) {
#pragma unroll
                                    for (int w = 0; w < Elem<T>::kBytes / 2; ++w) Elem<T>::nan_update(nanq, pk.w[w]);
                                } else {
                                    for (int e = 0; e < 8; ++e) qnan |= a + e < vocab && x[e] != x[e];
                                }
                                norm_update8(x, bits, sc, mq, sql);
                            }
                        }
                    }
                });
                // Lanes -> warp -> CTA (the same merge order in every thread), then every CTA's
                // normalisers to every CTA of the cluster.
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) {
                    norm_merge(mt, stl, __shfl_xor_sync(0xFFFFFFFFu, mt, o), __shfl_xor_sync(0xFFFFFFFFu, stl, o), sc);
                    norm_merge(mq, sql, __shfl_xor_sync(0xFFFFFFFFu, mq, o), __shfl_xor_sync(0xFFFFFFFFu, sql, o), sc);
                }
                cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
                const uint32_t wfl = (__any_sync(0xFFFFFFFFu, tnan || Elem<T>::has_nan(nant)) ? 1u : 0u) |
                                     (__any_sync(0xFFFFFFFFu, qnan || Elem<T>::has_nan(nanq)) ? 2u : 0u);
                if (lane == 0) {
                    s_wm[0][wid] = mt;
                    s_ws[0][wid] = stl;
                    s_wm[1][wid] = mq;
                    s_ws[1][wid] = sql;
                    s_wcnt[wid] = cnt;
                    s_wfl[wid] = wfl;
                }
                __syncthreads();
                if (tid < static_cast<int>(csize)) {
                    float Mt = s_wm[0][0], Mq = s_wm[1][0];
                    double St = s_ws[0][0], Sq = s_ws[1][0];
                    uint32_t ccnt = s_wcnt[0], cfl = s_wfl[0];
                    for (int w = 1; w < kAccWarps; ++w) {
                        norm_merge(Mt, St, s_wm[0][w], s_ws[0][w], sc);
                        norm_merge(Mq, Sq, s_wm[1][w], s_ws[1][w], sc);
                        ccnt += s_wcnt[w];
                        cfl |= s_wfl[w];
                    }
                    if (s_abort) cfl |= 4u;
                    uint32_t sw[4];
                    memcpy(&sw[0], &St, 8);
                    memcpy(&sw[2], &Sq, 8);
                    const uint32_t peer = static_cast<uint32_t>(tid);
                    ptx::st_cluster_v4(ptx::mapa(ptx::smem_addr(&s_norm[slot][crank][0]), peer), __float_as_uint(Mt),
                                       ccnt, cfl, __float_as_uint(Mq));
                    ptx::st_cluster_v4(ptx::mapa(ptx::smem_addr(&s_norm[slot][crank][1]), peer), sw[0], sw[1], sw[2],
                                       sw[3]);
                }
                ptx::cluster_arrive();
                ptx::cluster_wait();
                {
                    float Mt = -kInf, Mq = -kInf;
                    double St = 0.0, Sq = 0.0;
                    uint32_t rcnt = 0u, rfl = 0u;
                    for (uint32_t q = 0; q < csize; ++q) {
                        const uint4 h = s_norm[slot][q][0], v = s_norm[slot][q][1];
                        double a, b;
                        const uint32_t va[2] = {v.x, v.y}, vb[2] = {v.z, v.w};
                        memcpy(&a, va, 8);
                        memcpy(&b, vb, 8);
                        norm_merge(Mt, St, __uint_as_float(h.x), a, sc);
                        norm_merge(Mq, Sq, __uint_as_float(h.w), b, sc);
                        rcnt += h.y;
                        rfl |= h.z;
                    }
                    auto make_norm = [&](float M, double S, bool nan) -> RowNorm {
                        RowNorm r{M, S, kOk, S > 0.0 ? 1.0 / S : 0.0};
                        r.code = (rfl & 4u) ? kTimeout : nan ? kNaN : (M == kInf) ? kPosInf : (rcnt == 0u) ? kEmpty
                                 : (M == -kInf || !(S > 0.0)) ? kNoMass : kOk;
                        return r;
                    };
                    tn = make_norm(Mt, St, (rfl & 1u) != 0u);
                    qn = make_norm(Mq, Sq, (rfl & 2u) != 0u);
                }
                if (!with_q) {
                    j = i;
                    code = tn.code;
                    break;
                }
                const int32_t c = tn.code != kOk ? tn.code : qn.code;
                bool ok = false;
                if (c == kOk && s_tbit[slot]) {
                    const double p = spec_weight(s_txt[slot], tn, sc), q = spec_weight(s_txq[slot], qn, sc);
                    ok = q > 0.0 && s_tu[slot] * q < p;
                }
                if (!ok) {
                    j = i;
                    code = c;
                }
            }
            residual0 = code == kOk && j < L;
        } else {
            if (wid == 0) {
                int32_t jw, cw;
                accept_prefix<T>(target, draft, masks, seq, rows_per_seq, vocab, proposals, L, tpart, qpart, u_accept,
                                 sc, lane, jw, cw);
                if (lane == 0) {
                    s_j = jw;
                    s_code = cw;
                }
            }
            __syncthreads();
            j = s_j;
            code = s_code;
            residual0 = code == kOk && j < L;
            if (code == kOk) {
                tn = row_norm(tpart[seq * rows_per_seq + j]);
                code = tn.code;
                if (residual0) qn = row_norm(qpart[seq * K + j]);  // usable: its acceptance test ran
            }
        }
        const int64_t trow = seq * rows_per_seq + j;
        const double ratio = residual0 && code == kOk ? tn.S / qn.S : 0.0;  // S_t / S_q, in [1/V, V]
        const float rhi = static_cast<float>(ratio), rlo = static_cast<float>(ratio - static_cast<double>(rhi));
        const T* trow_p = target + trow * vocab;
        const T* qrow_p = draft + (seq * K + (residual0 ? j : 0)) * vocab;
        const int32_t* mrow = masks + trow * words;
        const double cut_u = u_resample[seq];
        int64_t chosen = -1;
        for (int pass = 0; pass < 2 && code == kOk && chosen < 0; ++pass) {
            const bool residual = residual0 && pass == 0;
            // Weight sum of tokens [a, a + 8) from their decoded logits (mask bits `bits`).
            auto weights8 = [&](int64_t a, uint32_t bits, const float (&xt)[8], const float (&xq)[8], float (&w)[8]) {
                if (residual) row_weights8<true>(a, vocab, bits, xt, xq, tn.M, qn.M, sc, rhi, rlo, w);
                else row_weights8<false>(a, vocab, bits, xt, xq, tn.M, qn.M, sc, rhi, rlo, w);
            };
            auto weigh8 = [&](int64_t a, uint32_t bits, const float (&xt)[8], const float (&xq)[8]) -> double {
                float w[8];
                weights8(a, bits, xt, xq, w);
                return static_cast<double>(sum8(w));
            };
            if constexpr (kStream) {
                const int64_t A = r0 * 256;
                stream_pass(trow_p, qrow_p, mrow, residual, [&](const uint8_t* stage, int64_t t0, int64_t ntc) {
                    // fp32 lane sum of tile tl of the chunk (tokens past the vocabulary weigh 0).
                    auto lane_tile = [&](int64_t tl) -> float {
                        const int64_t off = tl * 256 + 8 * lane;
                        const uint32_t word = reinterpret_cast<const uint32_t*>(stage + 2 * kAccRowBytes)[off >> 5];
                        Pack8<T> pk;
                        float xt[8], xq[8] = {}, w[8];
#pragma unroll
                        for (int i = 0; i < Elem<T>::kBytes / 2; ++i)
                            pk.w[i] = reinterpret_cast<const uint4*>(stage + off * sizeof(T))[i];
                        unpack8<T>(pk, xt);
                        if (residual) {
#pragma unroll
                            for (int i = 0; i < Elem<T>::kBytes / 2; ++i)
                                pk.w[i] = reinterpret_cast<const uint4*>(stage + kAccRowBytes + off * sizeof(T))[i];
                            unpack8<T>(pk, xq);
                        }
                        weights8(t0 + off, (word >> (off & 31)) & 0xFFu, xt, xq, w);
                        return sum8(w);
                    };
                    // A full chunk has kPerWarp tiles per warp: both computed in one unrolled block
                    // (independent work to interleave), then one fp32 butterfly for both sums --
                    // after the xor-16 step the low half-warp holds tile wid's pairs, the high half
                    // tile wid + kAccWarps's.
                    float sk[kPerWarp];
                    if (ntc * 256 == kTok && t0 + kTok <= vocab) {
#pragma unroll
                        for (int k = 0; k < kPerWarp; ++k) sk[k] = lane_tile(wid + kAccWarps * k);
                    } else {
#pragma unroll
                        for (int k = 0; k < kPerWarp; ++k) {
                            const int64_t tl = wid + kAccWarps * k;
                            sk[k] = tl < ntc && t0 + tl * 256 + 8 * lane < vocab ? lane_tile(tl) : 0.0f;
                        }
                    }
                    const int64_t tbase = (t0 - A) / 256;
                    if constexpr (kPerWarp == 2) {
                        const bool high = (lane & 16) != 0;
                        float v = high ? sk[1] : sk[0];
                        v += __shfl_xor_sync(0xFFFFFFFFu, high ? sk[0] : sk[1], 16);
#pragma unroll
                        for (int o = 8; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                        if (lane == 0 && wid < ntc) tile_sums[tbase + wid] = v;
                        if (lane == 16 && wid + kAccWarps < ntc) tile_sums[tbase + wid + kAccWarps] = v;
                    } else {
                        float v = sk[0];
#pragma unroll
                        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                        if (lane == 0 && wid < ntc) tile_sums[tbase + wid] = v;
                    }
                });
            } else {
                // This CTA's tile sums, kBatch tiles per warp and iteration (64 bytes a lane and row in
                // flight): every raw 16-byte load of the batch is issued before the first weight is
                // computed.  Rows that are not 16-byte aligned and the row's last partial group take
                // load8's scalar loads instead.
                constexpr int kBatch = Elem<T>::kBytes == 2 ? 4 : 2;
                for (int64_t lt = wid; lt < nt; lt += kAccWarps * kBatch) {
                    Pack8<T> pt[kBatch], pq[kBatch];
                    uint32_t bits[kBatch];
                    bool fast[kBatch];
#pragma unroll
                    for (int q = 0; q < kBatch; ++q) {
                        const int64_t a = (r0 + lt + kAccWarps * q) * 256 + 8 * lane;
                        const bool live = lt + kAccWarps * q < nt && a < vocab;
                        bits[q] = live ? (static_cast<uint32_t>(mrow[a >> 5]) >> (a & 31)) & 0xFFu : 0u;
                        fast[q] = live && vec && a + 8 <= vocab;
                        if (fast[q]) {
                            fetch8<T>(trow_p, a, pt[q]);
                            if (residual) fetch8<T>(qrow_p, a, pq[q]);
                        }
                    }
                    double v[kBatch];
#pragma unroll
                    for (int q = 0; q < kBatch; ++q) {
                        const int64_t a = (r0 + lt + kAccWarps * q) * 256 + 8 * lane;
                        float xt[8], xq[8] = {};
                        v[q] = 0.0;
                        if (fast[q]) {
                            unpack8<T>(pt[q], xt);
                            if (residual) unpack8<T>(pq[q], xq);
                            v[q] = weigh8(a, bits[q], xt, xq);
                        } else if (bits[q]) {
                            load8<T>(trow_p, a, vocab, vec, xt);
                            if (residual) load8<T>(qrow_p, a, vocab, vec, xq);
                            v[q] = weigh8(a, bits[q], xt, xq);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < kBatch; ++q) {
#pragma unroll
                        for (int o = 16; o >= 1; o >>= 1) v[q] += __shfl_xor_sync(0xFFFFFFFFu, v[q], o);
                        if (lane == 0 && lt + kAccWarps * q < nt) tile_sums[lt + kAccWarps * q] = v[q];
                    }
                }
            }
            if (tid == 0) {
                s_tile = -1;
                s_token = -1;
                s_last = -1;
                s_claim = 0;
                s_cut_past = 0;
            }
            __syncthreads();
            // Scan of this CTA's tile sums in order: thread tid owns tiles [tid * per, (tid + 1) * per).
            const int64_t per = (nt + kAccThreads - 1) / kAccThreads;
            const int64_t a0 = min(nt, tid * per), a1 = min(nt, a0 + per);
            double local = 0.0;
            for (int64_t t = a0; t < a1; ++t) local += tile_sums[t];
            double v = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double n = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += n;
            }
            if (lane == 31) sums[wid] = v;
            __syncthreads();
            const bool aborted = kStream && s_abort != 0;  // every stage wait has ended by now
            double before = 0.0, ctotal = 0.0;
            for (int w = 0; w < kAccWarps; ++w) {
                if (w < wid) before += sums[w];
                ctotal += sums[w];
            }
            // This CTA's mass to every CTA of the cluster, then the cluster's prefix and total.
            if (tid < static_cast<int>(csize)) {
                uint32_t lo, hi;
                memcpy(&lo, &ctotal, 4);
                memcpy(&hi, reinterpret_cast<const uint8_t*>(&ctotal) + 4, 4);
                ptx::st_cluster_v4(ptx::mapa(ptx::smem_addr(&s_rank[crank]), static_cast<uint32_t>(tid)), lo, hi,
                                   ctotal > 0.0 ? 1u : 0u, aborted ? 1u : 0u);
            }
            ptx::cluster_arrive();
            ptx::cluster_wait();
            auto rank_mass = [&](uint32_t q) -> double {
                const uint4 r = s_rank[q];
                const uint64_t bits = (static_cast<uint64_t>(r.y) << 32) | r.x;
                return __longlong_as_double(static_cast<long long>(bits));
            };
            double rbefore = 0.0, total = 0.0;
            int last_pos = -1;
            bool any_abort = false;
            for (uint32_t q = 0; q < csize; ++q) {
                const double m = rank_mass(q);
                if (q < crank) rbefore += m;
                if (s_rank[q].z) last_pos = static_cast<int>(q);
                any_abort |= s_rank[q].w != 0u;
                total += m;
            }
            // The CTA whose range holds the cut (the masses before it summed in the same order as
            // rbefore), else -- rounding put the cut past the last mass -- the last CTA with mass.
            const double cut = cut_u * total;
            int owner = -1;
            bool past = false;
            {
                double acc = 0.0;
                for (uint32_t q = 0; q < csize; ++q) {
                    const double m = rank_mass(q);
                    if (owner < 0 && m > 0.0 && cut < acc + m) owner = static_cast<int>(q);
                    acc += m;
                }
            }
            if (owner < 0 && last_pos >= 0) {
                owner = last_pos;
                past = true;
            }
            if (any_abort) {  // a CTA's stream gave up: the sequence reports a timeout
                owner = -1;
                code = kTimeout;
            }
            if (static_cast<int>(crank) == owner) {
                // This CTA holds the cut: its tile, by the scan of its tile sums (masses before it:
                // rbefore + the scan), or its last tile with mass when the cut lies past it.
                const double incl = rbefore + before + v;
                if (local > 0.0) {
                    atomicMax(&s_last, tid);
                    if (!past && cut >= incl - local && cut < incl) {
                        double acc = incl - local;
                        int64_t pick = -1;
                        double pick_prefix = 0.0;
                        for (int64_t t = a0; t < a1; ++t) {
                            if (tile_sums[t] > 0.0) {
                                pick = t;
                                pick_prefix = acc;
                                if (cut < acc + tile_sums[t]) break;
                                acc += tile_sums[t];
                            }
                        }
                        if (atomicExch(&s_claim, 1) == 0) {  // rounding may let two segments claim
                            s_tile = pick;
                            s_prefix = pick_prefix;
                        }
                    }
                }
                __syncthreads();
                if (s_tile < 0 && tid == s_last) {
                    int64_t pick = -1;
                    double acc = incl - local;
                    double pick_prefix = 0.0;
                    for (int64_t t = a0; t < a1; ++t)
                        if (tile_sums[t] > 0.0) {
                            pick = t;
                            pick_prefix = acc;
                            acc += tile_sums[t];
                        }
                    s_tile = pick;
                    s_prefix = pick_prefix;
                    s_cut_past = 1;
                }
                __syncthreads();
                if (wid == 0 && s_tile >= 0) {
                    // Each lane's 8 tokens of the tile, decoded once: the lane sums and the walk.
                    const int64_t a = (r0 + s_tile) * 256 + 8 * lane;
                    float xt[8] = {}, xq[8] = {};
                    uint32_t bits = 0u;
                    if (a < vocab) {
                        bits = (static_cast<uint32_t>(mrow[a >> 5]) >> (a & 31)) & 0xFFu;
                        load8<T>(trow_p, a, vocab, vec, xt);
                        if (residual) load8<T>(qrow_p, a, vocab, vec, xq);
                    }
                    float w[8];
                    weights8(a, bits, xt, xq, w);
                    const double ls = static_cast<double>(sum8(w));
                    double li = ls;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const double n = __shfl_up_sync(0xFFFFFFFFu, li, o);
                        if (lane >= o) li += n;
                    }
                    const bool cut_past = s_cut_past != 0;
                    const uint32_t pos = __ballot_sync(0xFFFFFFFFu, ls > 0.0);
                    const uint32_t hit = __ballot_sync(0xFFFFFFFFu, !cut_past && ls > 0.0 && cut < s_prefix + li);
                    const int Lw = hit ? __ffs(hit) - 1 : (pos ? 31 - __clz(pos) : -1);
                    if (lane == Lw) {
                        double acc = s_prefix + li - ls;
                        int64_t pick = -1;
                        bool done = false;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            if (done || !(w[i] > 0.0f)) continue;
                            pick = a + i;
                            if (hit && cut < acc + static_cast<double>(w[i])) done = true;
                            else acc += static_cast<double>(w[i]);
                        }
                        s_token = pick;
                    }
                }
                __syncthreads();
                // The token to every CTA of the cluster (-1 if the walk found no weight).
                if (tid < static_cast<int>(csize)) {
                    const int64_t tkn = s_token;
                    uint32_t lo, hi;
                    memcpy(&lo, &tkn, 4);
                    memcpy(&hi, reinterpret_cast<const uint8_t*>(&tkn) + 4, 4);
                    ptx::st_cluster_v4(ptx::mapa(ptx::smem_addr(&s_pick), static_cast<uint32_t>(tid)), lo, hi, 0u, 0u);
                }
            }
            ptx::cluster_arrive();
            ptx::cluster_wait();
            if (owner >= 0) {
                const uint4 r = s_pick;
                const uint32_t w2[2] = {r.x, r.y};
                memcpy(&chosen, w2, 8);
            }
        }
        if (code == kOk && chosen < 0) code = kNoMass;
        if (crank == 0 && tid == 0) {
            accept_len[seq] = j;
            status[seq] = code;
            token[seq] = code == kOk ? chosen : -1;
            kind[seq] = j < L ? 0 : (L > 0 ? 1 : 2);
        }
        __syncthreads();
    }
    // Copies still in flight after an abort land before the CTA exits, and no CTA exits while a
    // peer can still write into its shared memory.
    if (kStream && tid == 0)
        for (int st = 0; st < kAccStages; ++st)
            if (s_issued[st] > 0) drain_wait(ptx::smem_addr(&s_full[st]), (s_issued[st] - 1u) & 1u);
    ptx::cluster_arrive();
    ptx::cluster_wait();
}

// Dynamic shared memory of the acceptance kernel: the streamed variant's stages, then one double
// per 256-token tile of a CTA's range.
constexpr size_t kAcceptSmemLimit = 200 * 1024;

size_t accept_smem_bytes(int64_t vocab, int csize, bool stream) {
    const int64_t ntiles = (vocab + 255) / 256;
    return (stream ? static_cast<size_t>(kAccStages) * kAccStageBytes : 0) +
           static_cast<size_t>((ntiles + csize - 1) / csize) * sizeof(double);
}

// Resident clusters of the acceptance kernel for 1, 2, 4 and 8 CTAs per cluster (0 where the
// shared memory does not fit), cached per device and type for the last vocabulary size seen.
struct AcceptInfo {
    int64_t vocab = -1;
    int clusters[4] = {0, 0, 0, 0};
};

template <typename T, bool kStream, bool kLazy = false>
int accept_info(int device, int64_t vocab, AcceptInfo& out) {
    static AcceptInfo table[kMaxDevices];
    int sms = 0;
    BMS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "sm count");
    std::lock_guard<std::mutex> lock(g_mutex);
    AcceptInfo& info = table[device];
    if (info.vocab != vocab) {
        auto kernel = speculative_accept_kernel<T, kStream, kLazy>;
        size_t most = 0;  // the largest size that fits: the function's dynamic shared memory limit
        for (int i = 0; i < 4; ++i) {
            const size_t smem = accept_smem_bytes(vocab, 1 << i, kStream);
            if (smem <= kAcceptSmemLimit) most = std::max(most, smem);
        }
        if (most > 48 * 1024)
            BMS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(most)),
                     "cudaFuncSetAttribute(smem)");
        for (int i = 0; i < 4; ++i) {
            const int c = 1 << i;
            const size_t smem = accept_smem_bytes(vocab, c, kStream);
            int n = 0;
            if (smem <= kAcceptSmemLimit) {
                cudaLaunchConfig_t cfg = {};
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = c;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.gridDim = dim3(c * sms);
                cfg.blockDim = dim3(kAccThreads);
                cfg.dynamicSmemBytes = smem;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    n = 0;
                }
            }
            info.clusters[i] = n;
        }
        info.vocab = vocab;
    }
    out = info;
    return BMS_SUCCESS;
}

// Longest-prefix acceptance, one warp per sequence: lane i looks at row i of a 32-row window,
// a ballot finds the first row where the reference stops (a failed status, a draft mismatch,
// or the bonus row), and per-row budgets follow.  Launched as a programmatic dependent of
// the selection kernel: the wait below is the grid dependency, not a spin.
__global__ void __launch_bounds__(256) verify_epilogue_kernel(
    const int64_t* __restrict__ row_tokens, const int64_t* __restrict__ row_counts, const int32_t* __restrict__ row_status,
    int64_t seqs, int64_t rows_per_seq, int64_t vocab, const int64_t* __restrict__ proposals,
    const int32_t* __restrict__ lengths, bms_policy policy, int32_t* __restrict__ row_budget,
    int32_t* __restrict__ accept_len, int64_t* __restrict__ token, int32_t* __restrict__ kind,
    int32_t* __restrict__ seq_status) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int64_t first_thread = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t threads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t k_max = rows_per_seq - 1;
    for (int64_t s = first_thread >> 5; s < seqs; s += threads >> 5) {
        const int64_t base = s * rows_per_seq;
        const int32_t len = lengths[s];
        int32_t a = -1, ss = 0, kd = 0;
        int64_t tk = -1;
        if (len < 0 || len > k_max) {
            a = 0;
            ss = kBadLength;
        }
        for (int64_t w0 = 0; a < 0 && w0 <= len; w0 += 32) {
            const int64_t i = w0 + lane;
            bool stop = false, miss = false;
            int32_t st = 0;
            int64_t tok = -1;
            if (i <= len) {
                st = row_status[base + i];
                tok = row_tokens[base + i];
                miss = i < len && tok != proposals[s * k_max + i];
                stop = st != 0 || miss || i == len;
            }
            const uint32_t ballot = __ballot_sync(0xFFFFFFFFu, stop);
            if (ballot) {
                const int f = __ffs(ballot) - 1;
                const int32_t fst = __shfl_sync(0xFFFFFFFFu, st, f);
                const int64_t ftok = __shfl_sync(0xFFFFFFFFu, tok, f);
                const bool fmiss = __shfl_sync(0xFFFFFFFFu, miss, f);
                a = static_cast<int32_t>(w0 + f);
                if (fst != 0) {
                    ss = fst;  // a consumed row failed: the reference raises here
                } else {
                    tk = ftok;  // correction at the first mismatch, else bonus / fallback
                    kd = fmiss ? 0 : (len > 0 ? 1 : 2);
                }
            }
        }
        if (lane == 0) {
            accept_len[s] = a;
            token[s] = tk;
            kind[s] = kd;
            seq_status[s] = ss;
        }
    }
    if (row_budget != nullptr && row_counts != nullptr) {
        for (int64_t r = first_thread; r < seqs * rows_per_seq; r += threads)
            row_budget[r] = policy_budget(policy, __ddiv_rn(static_cast<double>(row_counts[r]), static_cast<double>(vocab)));
    }
}

// Merge of vocabulary-shard partials, one warp per row (grid-stride).  partials is [shards, rows]
// in shard order.  The sampler's owner walk re-reads this rank's shard (the same device functions
// as the single-GPU cluster merge, so both produce identical bits).
template <typename T, bool kSample>
__global__ void __launch_bounds__(128) shard_merge_kernel(
    const GatherSlot* __restrict__ partials, int32_t shards, int32_t shard, int64_t rows, double temperature,
    double inv, float scale2, const double* __restrict__ uniforms, const uint8_t* __restrict__ logits,
    const int32_t* __restrict__ masks, int64_t mask_words, int64_t vocab_shard, int64_t token_offset,
    const uint8_t* __restrict__ granules, int64_t granule_stride, int64_t* __restrict__ tokens,
    int64_t* __restrict__ counts, int32_t* __restrict__ status) {
    __shared__ float walk[4][32][33];
    __shared__ double fac[4][kConsumerWarps];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + wib; row < rows; row += nwarps) {
        if constexpr (!kSample) {
            const bool in = lane < shards;
            const GatherSlot g = in ? partials[lane * rows + row] : GatherSlot{0u, 0u, 0u, 0u, 0.0, 0.0};
            const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, g.a);
            const uint32_t lo = __reduce_max_sync(0xFFFFFFFFu, (in && g.a == hi) ? g.b : 0u);
            const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, g.c);
            const uint32_t fl = __reduce_or_sync(0xFFFFFFFFu, g.d);
            if (lane == 0) {
                const int32_t code = argmax_status(fl, total);
                status[row] = code;
                tokens[row] = code == kOk ? static_cast<int64_t>(0xFFFFFFFFu - lo) : -1;
                if (counts) counts[row] = total;
            }
        } else {
            const SampleMerge mg = merge_sampler_ranks(partials + row, rows, static_cast<uint32_t>(shards), uniforms[row],
                                                       temperature, inv, 0u, lane);
            int64_t token = -1;
            int32_t code = mg.code;
            if (mg.code == kOk && mg.owner == shard) {
                const uint8_t* rec = granules + row * granule_stride;
                const bool has = lane < kConsumerWarps;
                const float wmax = has ? reinterpret_cast<const float*>(rec + SamplerRecord::kWarpMaxOffset)[lane] : 0.0f;
                const double wmass = has ? reinterpret_cast<const double*>(rec + SamplerRecord::kWarpMassOffset)[lane] : 0.0;
                // The shard's own max, as its finalizer used it for the warp factors.
                const float seg_m = __uint_as_float(partials[static_cast<int64_t>(shard) * rows + row].a);
                const double wf = (has && wmass > 0.0) ? warp_factor(wmax, seg_m, temperature, inv) : 0.0;
                const int nchunks = static_cast<int>((vocab_shard + Layout<T>::kTokensPerChunk - 1) / Layout<T>::kTokensPerChunk);
                const uint8_t* lrow = logits + static_cast<size_t>(row) * static_cast<size_t>(vocab_shard) * sizeof(T);
                const int32_t* mrow = masks + static_cast<size_t>(row) * static_cast<size_t>(mask_words) + (token_offset >> 5);
                const int64_t chosen = sampler_owner_walk<T>(
                    reinterpret_cast<const double*>(rec + SamplerRecord::kGranuleOffset), kConsumerWarps, 1,
                    nchunks * kConsumerWarps, wf,
                    wmass, has, mg, temperature, inv, scale2, 0, vocab_shard, lrow, mrow, walk[wib], fac[wib], lane);
                token = chosen >= 0 ? token_offset + chosen : -1;
                if (chosen < 0) code = kNoMass;
            }
            if (lane == 0) {
                // Only the owner knows the token; the others report -1 (combine ranks with a max).
                status[row] = code;
                tokens[row] = token;
                if (counts) counts[row] = mg.total;
            }
        }
    }
}

// Merge of a peer-memory exchange step (argmax partials), one warp per row (grid-stride) over
// this rank's area: waits (bounded) until every rank published the step, merges exactly like
// shard_merge_kernel, then the last CTA tells every rank that this rank's slot of the step is
// free again.  A wait that gives up reports status 7 for the CTA's rows, and so does a row whose
// partial from some rank carries another step's epoch tag (ranks that passed different row counts).
__global__ void __launch_bounds__(128) exchange_merge_kernel(ExchangeAreas areas, int32_t ranks, int32_t rank,
                                                             int64_t rows_cap, uint32_t epoch, int64_t rows,
                                                             int64_t* __restrict__ tokens, int64_t* __restrict__ counts,
                                                             int32_t* __restrict__ status) {
    __shared__ int32_t gave_up;
    ExchangeHeader* own = reinterpret_cast<ExchangeHeader*>(areas.a[rank]);
    // An empty step has no partials to wait for (its selection launches nothing).
    if (threadIdx.x == 0) gave_up = (rows == 0 || wait_flags_at_least(own->ready, ranks, epoch)) ? 0 : 1;
    __syncthreads();
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + wib; row < rows; row += nwarps) {
        if (gave_up) {
            if (lane == 0) {
                status[row] = kTimeout;
                tokens[row] = -1;
                if (counts) counts[row] = 0;
            }
            continue;
        }
        const bool in = lane < ranks;
        GatherSlot g{0u, 0u, 0u, 0u, 0.0, 0.0};
        uint32_t tag = epoch;
        if (in) {  // written by peer GPUs: read through L2
            const uint4* src = reinterpret_cast<const uint4*>(exchange_slot(areas.a[rank], ranks, rows_cap, epoch, lane) + row);
            const uint4 x = __ldcg(src), y = __ldcg(src + 1);
            g.a = x.x;
            g.b = x.y;
            g.c = x.z;
            g.d = x.w;
            tag = y.z;  // low word of the slot's epoch tag (GatherSlot::pad)
        }
        const bool stale = __any_sync(0xFFFFFFFFu, tag != epoch);
        const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, g.a);
        const uint32_t lo = __reduce_max_sync(0xFFFFFFFFu, (in && g.a == hi) ? g.b : 0u);
        const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, g.c);
        const uint32_t fl = __reduce_or_sync(0xFFFFFFFFu, g.d) | (stale ? kFlagAbort : 0u);
        if (lane == 0) {
            const int32_t code = argmax_status(fl, total);
            status[row] = code;
            tokens[row] = code == kOk ? static_cast<int64_t>(0xFFFFFFFFu - lo) : -1;
            if (counts) counts[row] = total;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ptx::fence_acq_rel_sys();
        const uint32_t before = atomicAdd(&own->merge_done, 1u);
        if (before + 1u == gridDim.x) {
            atomicExch(&own->merge_done, 0u);
            ptx::fence_acq_rel_sys();
            for (int q = 0; q < ranks; ++q)
                ptx::st_release_sys(&reinterpret_cast<ExchangeHeader*>(areas.a[q])->consumed[rank], epoch);
        }
    }
}

// 1 / T for the device's exponent arguments, or 0 where it is not finite (they then divide by T).
double inverse_temperature(double temperature) {
    const double inv = temperature > 0.0 ? 1.0 / temperature : 0.0;
    return std::isfinite(inv) ? inv : 0.0;
}

float sampler_scale2(double temperature) {
    float scf = static_cast<float>(2.0 * 1.4426950408889634 / temperature);
    const float tiny = 1.40129846e-45f;
    if (!(scf >= tiny)) scf = tiny;
    return scf;
}

int64_t granule_bytes(int dtype, int64_t vocab_shard) {
    const int64_t tpc = kChunkBytes / elem_bytes(dtype);
    return SamplerRecord::bytes(static_cast<int>((vocab_shard + tpc - 1) / tpc));
}

int check_policy(const bms_policy* policy) {
    if (policy == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "policy must not be NULL when budgets are requested");
    const bms_policy& P = *policy;
    if (P.kind != 0 && P.kind != 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "unknown policy kind %d", P.kind);
    if (!(std::isfinite(P.low_density) && std::isfinite(P.high_density)) || P.low_density < 0 || P.high_density > 1 ||
        !(P.low_density < P.high_density))
        return fail(BMS_ERROR_INVALID_ARGUMENT, "density thresholds must be finite, within [0, 1] and increasing");
    if (P.min_budget < 1 || P.max_budget < P.min_budget)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "budgets must satisfy 1 <= min_budget <= max_budget");
    return BMS_SUCCESS;
}

int sm_count(int device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return n;
}

int select_common(int dtype, const void* logits, const int32_t* masks, int64_t rows, int64_t vocab, int device) {
    BMS_CHECK(check_dtype(dtype));
    BMS_CHECK(check_vocab(vocab));
    if (rows < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows must be nonnegative");
    BMS_CHECK(check_device(device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(logits, device, "logits", static_cast<size_t>(elem_bytes(dtype))));
    BMS_CHECK(check_ptr(masks, device, "masks", 4));
    return BMS_SUCCESS;
}

// Split-row capacity of a device's workspace: every row of a batch on the flat schedule (fewer
// than 1.5 rows per resident CTA, at most 3 CTAs per SM).
int64_t workspace_rows(int device) { return 5ll * sm_count(device); }

int attach_workspace(SelectParams& p, void* ws, int64_t bytes, int device) {
    if (ws == nullptr) return BMS_SUCCESS;
    const int64_t need = ws_bytes(workspace_rows(device));
    if (bytes < need)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "workspace of %lld bytes is smaller than bms_workspace_bytes() = %lld",
                    static_cast<long long>(bytes), static_cast<long long>(need));
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    BMS_CHECK(check_ptr(ws, device, "workspace", 256));
    p.ws = static_cast<uint8_t*>(ws);
    p.ws_rows = workspace_rows(device);
    p.ws_flat = 1;
    return BMS_SUCCESS;
}

// Workspace of bms_masked_reduce_batch_noalloc: a file-scope device array (one instance per
// device), so that entry point allocates nothing.  Split-row capacity kStaticWsRows (the dynamic
// schedule splits at most that many rows), about 1.8 MB.
constexpr int64_t kStaticWsRows = 256;
constexpr int64_t kStaticWsBytes = ws_split_bytes(kStaticWsRows);
static __device__ __align__(256) uint8_t g_static_ws[kStaticWsBytes];
void* g_static_ws_ptr[kMaxDevices] = {};  // guarded by g_mutex

// Device address of this device's static workspace (the device must be current).  The first call
// per device resolves the symbol and clears the counters on `stream` -- setup that must not run
// under stream capture; later calls only return the cached address.
int static_workspace(int device, cudaStream_t stream, void*& out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_static_ws_ptr[device] == nullptr) {
        void* ptr = nullptr;
        BMS_CUDA(cudaGetSymbolAddress(&ptr, g_static_ws), "cudaGetSymbolAddress(static workspace)");
        // Header and row counters start at zero (pieces carry launch epochs); every call leaves
        // them at zero again.
        BMS_CUDA(cudaMemsetAsync(ptr, 0, static_cast<size_t>(ws_pieces_offset(kStaticWsRows)), stream),
                 "clearing the static workspace");
        g_static_ws_ptr[device] = ptr;
    }
    out = g_static_ws_ptr[device];
    return BMS_SUCCESS;
}

SelectParams base_params(const void* logits, const int32_t* masks, int64_t rows, int64_t vocab) {
    SelectParams p = {};
    p.logits = logits;
    p.masks = masks;
    p.rows = rows;
    p.vocab = vocab;
    p.logit_stride = vocab;
    p.mask_stride = (vocab + 31) / 32;
    p.token_offset = 0;
    return p;
}

}  // namespace
}  // namespace bms

using namespace bms;

extern "C" {

const char* bms_last_error(void) { return g_error; }

int bms_runtime_version(int32_t* version) {
    if (version == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "version must not be NULL");
    int v = 0;
    BMS_CUDA(cudaRuntimeGetVersion(&v), "cudaRuntimeGetVersion");
    *version = v;
    return BMS_SUCCESS;
}

int bms_set_launch_override(int32_t cluster, int32_t clusters) {
    if (cluster != 0 && cluster != 1 && cluster != 2 && cluster != 4 && cluster != 8 && cluster != 16)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "cluster override must be 0, 1, 2, 4, 8 or 16");
    if (clusters < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "clusters override must be nonnegative");
    g_force_cluster = cluster;
    g_force_clusters = clusters;
    return BMS_SUCCESS;
}

int64_t bms_workspace_bytes(int32_t device) {
    if (check_device(device) != BMS_SUCCESS) return -1;
    return ws_bytes(workspace_rows(device));
}

int bms_masked_reduce_batch(const void* logits, int32_t dtype, const int32_t* masks, int64_t rows, int64_t vocab,
                            int64_t* tokens, int64_t* counts, int32_t* status, void* workspace,
                            int64_t workspace_bytes, int32_t device, void* stream) {
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab, device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(tokens, device, "tokens", 8));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    SelectParams p = base_params(logits, masks, rows, vocab);
    BMS_CHECK(attach_workspace(p, workspace, workspace_bytes, device));
    p.tokens = tokens;
    p.counts = counts;
    p.status = status;
    return launch_select<false>(dtype, p, device, static_cast<cudaStream_t>(stream));
}

int bms_masked_reduce_batch_noalloc(const void* logits, int32_t dtype, const int32_t* masks, int64_t rows,
                                    int64_t vocab, int64_t* tokens, int64_t* counts, int32_t* status, int32_t device,
                                    void* stream) {
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab, device));
    if (rows == 0) return BMS_SUCCESS;
    const int64_t tpc = dtype == BMS_FLOAT32 ? Layout<float>::kTokensPerChunk : Layout<__half>::kTokensPerChunk;
    if (vocab > kWsChunks * tpc)
        return fail(BMS_ERROR_UNSUPPORTED, "vocabulary of %lld tokens exceeds the %lld-token rows the static workspace splits",
                    static_cast<long long>(vocab), static_cast<long long>(kWsChunks * tpc));
    BMS_CHECK(check_ptr(tokens, device, "tokens", 8));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    BMS_CHECK(static_workspace(device, s, ws));
    SelectParams p = base_params(logits, masks, rows, vocab);
    p.ws = static_cast<uint8_t*>(ws);
    p.ws_rows = kStaticWsRows;
    p.dynamic_always = 1;
    p.tokens = tokens;
    p.counts = counts;
    p.status = status;
    return launch_select<false>(dtype, p, device, s);
}

int bms_masked_argmax(const void* logits, int32_t dtype, const int32_t* mask, int64_t vocab, int64_t* token,
                      int32_t* status, int32_t device, void* stream) {
    return bms_masked_reduce_batch(logits, dtype, mask, 1, vocab, token, nullptr, status, nullptr, 0, device, stream);
}

int bms_masked_sample_batch(const void* logits, int32_t dtype, const int32_t* masks, int64_t rows, int64_t vocab,
                            double temperature, const double* uniforms, int64_t* tokens, int64_t* counts,
                            int32_t* status, void* workspace, int64_t workspace_bytes, int32_t device, void* stream) {
    if (!std::isfinite(temperature) || temperature < 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "temperature must be finite and nonnegative");
    if (temperature == 0)  // csrc/sample.cu:120: zero temperature is the masked argmax
        return bms_masked_reduce_batch(logits, dtype, masks, rows, vocab, tokens, counts, status, workspace,
                                       workspace_bytes, device, stream);
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab, device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(uniforms, device, "uniforms", 8));
    BMS_CHECK(check_ptr(tokens, device, "tokens", 8));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    SelectParams p = base_params(logits, masks, rows, vocab);
    BMS_CHECK(attach_workspace(p, workspace, workspace_bytes, device));
    p.tokens = tokens;
    p.counts = counts;
    p.status = status;
    p.uniforms = uniforms;
    p.temperature = temperature;
    p.inv_temperature = inverse_temperature(temperature);
    // 2*log2(e)/T in float; +inf for tiny T, clamped to the smallest denormal for huge T so
    // that -inf logits still map to zero weight.
    p.scale2 = sampler_scale2(temperature);
    p.scale = static_cast<float>(1.4426950408889634 / temperature);
    return launch_select<true>(dtype, p, device, static_cast<cudaStream_t>(stream));
}

int bms_masked_sample(const void* logits, int32_t dtype, const int32_t* mask, int64_t vocab, double temperature,
                      const double* uniform, int64_t* token, int32_t* status, int32_t device, void* stream) {
    return bms_masked_sample_batch(logits, dtype, mask, 1, vocab, temperature, uniform, token, nullptr, status, nullptr,
                                   0, device, stream);
}

int bms_mask_budget(const int32_t* masks, int64_t rows, int64_t vocab, const bms_policy* policy, int64_t* counts,
                    double* density, int32_t* budget, int32_t device, void* stream) {
    BMS_CHECK(check_vocab(vocab));
    if (rows < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows must be nonnegative");
    bms_policy P = {0, 1, 8, 0, 0.005, 0.02};
    if (budget) {
        BMS_CHECK(check_policy(policy));
        P = *policy;
    }
    BMS_CHECK(check_device(device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(masks, device, "masks", 4));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    if (density) BMS_CHECK(check_ptr(density, device, "density", 8));
    if (budget) BMS_CHECK(check_ptr(budget, device, "budget", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
    const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
    count_rows_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(masks, rows, vocab, P, counts, density, budget);
    BMS_CUDA(cudaGetLastError(), "popcount launch");
    return BMS_SUCCESS;
}

int bms_speculative_accept(const void* target_logits, const void* draft_logits, int32_t dtype, const int32_t* masks,
                           int64_t seqs, int64_t rows_per_seq, int64_t vocab, const int64_t* proposals,
                           const int32_t* lengths, const bms_partial* target_partials, const bms_partial* draft_partials,
                           double temperature, const double* accept_uniforms, const double* resample_uniforms,
                           int32_t* accept_len, int64_t* token, int32_t* kind, int32_t* status, int32_t device,
                           void* stream) {
    if (!std::isfinite(temperature) || !(temperature > 0))
        return fail(BMS_ERROR_INVALID_ARGUMENT, "temperature must be finite and positive");
    if (seqs < 0 || rows_per_seq < 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "invalid sequence shape");
    BMS_CHECK(check_dtype(dtype));
    BMS_CHECK(check_vocab(vocab));
    BMS_CHECK(check_device(device));
    if (seqs == 0) return BMS_SUCCESS;
    const size_t eb = static_cast<size_t>(elem_bytes(dtype));
    BMS_CHECK(check_ptr(target_logits, device, "target_logits", eb));
    BMS_CHECK(check_ptr(masks, device, "masks", 4));
    BMS_CHECK(check_ptr(lengths, device, "lengths", 4));
    // No partials: the kernel computes the consumed positions' normalisers itself (lazy).
    const bool lazy = target_partials == nullptr;
    if (lazy && draft_partials != nullptr)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "target_partials and draft_partials must both be given or both be NULL");
    if (!lazy) BMS_CHECK(check_ptr(target_partials, device, "target_partials", 16));
    BMS_CHECK(check_ptr(resample_uniforms, device, "resample_uniforms", 8));
    if (rows_per_seq > 1) {
        BMS_CHECK(check_ptr(draft_logits, device, "draft_logits", eb));
        BMS_CHECK(check_ptr(proposals, device, "proposals", 8));
        if (!lazy) BMS_CHECK(check_ptr(draft_partials, device, "draft_partials", 16));
        BMS_CHECK(check_ptr(accept_uniforms, device, "accept_uniforms", 8));
    }
    BMS_CHECK(check_ptr(accept_len, device, "accept_len", 4));
    BMS_CHECK(check_ptr(token, device, "token", 8));
    BMS_CHECK(check_ptr(kind, device, "kind", 4));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    // log2(e) / T, kept finite (so that a token at the row maximum weighs exactly 1 at any T).
    const float sc = static_cast<float>(std::min(1.4426950408889634 / temperature, 3.0e38));
    // CTAs per sequence, c in {1, 2, 4, 8}, by a cost model: the resident clusters take the
    // sequences in ceil(seqs / resident) rounds, each costing sigma + 1 / c -- streaming the sampled
    // rows split c ways, plus the serial part of a sequence (the acceptance tests, its rows' norms,
    // the first chunk's latency, two cluster barriers, the walk) that every CTA of the cluster
    // waits through.  sigma = kAcceptSerialBytes / row bytes: measured on B200 at V = 248,320 bf16,
    // one CTA streams a sequence's target and draft rows in about 70 us and the serial part takes
    // about 15 us, as long as streaming 109 KB of one row.
    // Rows stream through shared memory when every bulk copy can be 16-byte aligned and sized.
    const auto aligned = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    const bool streamed = aligned(target_logits) && aligned(draft_logits) && aligned(masks) &&
                        (vocab * static_cast<int64_t>(eb)) % 16 == 0 && ((vocab + 31) / 32) % 4 == 0;
    if (lazy && !streamed)
        return fail(BMS_ERROR_UNSUPPORTED,
                    "without partials, rows must be 16-byte aligned multiples of 16 bytes and mask rows multiples "
                    "of 4 words");
    AcceptInfo ai;
#define BMS_SPEC_INFO(T)                                                                                      \
    BMS_CHECK((lazy ? accept_info<T, true, true>(device, vocab, ai)                                         \
                    : streamed ? accept_info<T, true>(device, vocab, ai) : accept_info<T, false>(device, vocab, ai)))
    if (dtype == BMS_FLOAT32) BMS_SPEC_INFO(float);
    else if (dtype == BMS_BFLOAT16) BMS_SPEC_INFO(__nv_bfloat16);
    else BMS_SPEC_INFO(__half);
#undef BMS_SPEC_INFO
    constexpr double kAcceptSerialBytes = 109000.0;
    const double sigma = kAcceptSerialBytes / (static_cast<double>(vocab) * static_cast<double>(eb));
    int ci = -1;
    double best = 0.0;
    for (int i = 0; i < 4; ++i) {
        if (ai.clusters[i] <= 0) continue;
        const double rounds = static_cast<double>((seqs + ai.clusters[i] - 1) / ai.clusters[i]);
        const double cost = rounds * (sigma + 1.0 / static_cast<double>(1 << i));
        if (ci < 0 || cost < best) {
            ci = i;
            best = cost;
        }
    }
    if (ci < 0) return fail(BMS_ERROR_UNSUPPORTED, "vocabulary too large for the acceptance kernel");
    // Lazy normalisers: a sequence's positions run one after another, so its chain of passes, not
    // the rounds, sets the time -- 8 CTAs per sequence when every cluster is resident at once, else
    // 4 (measured on B200, 256 sequences x K = 8, V = 248,320 bf16: 1 / 2 / 4 / 8 CTAs 793 / 656 /
    // 543 / 727 us with a mean accepted run of 2.6, 335 / 297 / 266 / 374 us with 0.36).
    if (lazy) {
        if (ai.clusters[3] > 0 && seqs <= ai.clusters[3]) ci = 3;
        else if (ai.clusters[2] > 0) ci = 2;
    }
    for (int i = 0; i < 4; ++i)  // the tests' launch override (1, 2, 4 or 8 CTAs per sequence)
        if (g_force_cluster == (1 << i) && ai.clusters[i] > 0) ci = i;
    const int csize = 1 << ci;
    const int64_t clusters = std::min<int64_t>(seqs, g_force_clusters > 0 ? g_force_clusters : ai.clusters[ci]);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * csize));
    cfg.blockDim = dim3(kAccThreads);
    cfg.dynamicSmemBytes = accept_smem_bytes(vocab, csize, streamed);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto tp = reinterpret_cast<const GatherSlot*>(target_partials);
    auto qp = reinterpret_cast<const GatherSlot*>(draft_partials);
#define BMS_SPEC_S(T, S, LZ)                                                                                \
    cudaLaunchKernelEx(&cfg, speculative_accept_kernel<T, S, LZ>, static_cast<const T*>(target_logits),        \
                       static_cast<const T*>(draft_logits), masks, seqs, rows_per_seq, vocab, proposals, lengths, tp, \
                       qp, accept_uniforms, resample_uniforms, sc, accept_len, token, kind, status)
#define BMS_SPEC(T) \
    (lazy ? BMS_SPEC_S(T, true, true) : streamed ? BMS_SPEC_S(T, true, false) : BMS_SPEC_S(T, false, false))
    cudaError_t launched;
    if (dtype == BMS_FLOAT32) launched = BMS_SPEC(float);
    else if (dtype == BMS_BFLOAT16) launched = BMS_SPEC(__nv_bfloat16);
    else launched = BMS_SPEC(__half);
#undef BMS_SPEC
#undef BMS_SPEC_S
    BMS_CUDA(launched, "speculative acceptance launch");
    return BMS_SUCCESS;
}

int bms_expand_token_lists(const int32_t* ids, int64_t n_ids, const int32_t* offsets, int64_t lists, int64_t vocab,
                           int32_t* out, int32_t* bad, int32_t device, void* stream) {
    BMS_CHECK(check_vocab(vocab));
    if (lists < 0 || n_ids < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "lists and n_ids must be nonnegative");
    BMS_CHECK(check_device(device));
    if (lists == 0) return BMS_SUCCESS;
    if (n_ids > 0) BMS_CHECK(check_ptr(ids, device, "ids", 4));
    BMS_CHECK(check_ptr(offsets, device, "offsets", 4));
    BMS_CHECK(check_ptr(out, device, "out", 4));
    if (bad) BMS_CHECK(check_ptr(bad, device, "bad", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
    const unsigned grid = static_cast<unsigned>(lists < cap ? lists : cap);
    expand_lists_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(ids, n_ids, offsets, lists, vocab, out, bad);
    BMS_CUDA(cudaGetLastError(), "token-list expansion launch");
    return BMS_SUCCESS;
}

int bms_expand_token_gaps(const uint8_t* bytes, int64_t n_bytes, const int32_t* offsets, int64_t rows, int64_t vocab,
                          int32_t* out, int32_t* bad, int32_t device, void* stream) {
    BMS_CHECK(check_vocab(vocab));
    if (rows < 0 || n_bytes < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows and n_bytes must be nonnegative");
    BMS_CHECK(check_device(device));
    if (rows == 0) return BMS_SUCCESS;
    if (n_bytes > 0) BMS_CHECK(check_ptr(bytes, device, "bytes", 1));
    BMS_CHECK(check_ptr(offsets, device, "offsets", 4));
    BMS_CHECK(check_ptr(out, device, "out", 4));
    if (bad) BMS_CHECK(check_ptr(bad, device, "bad", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
    const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
    const int64_t smem = (vocab + 31) / 32 * 4;
    if (smem <= kGapSmemBytes) {
        if (smem > 48 * 1024)
            BMS_CUDA(cudaFuncSetAttribute(expand_gaps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kGapSmemBytes)),
                     "cudaFuncSetAttribute(gap expansion smem)");
        expand_gaps_kernel<<<grid, kGapThreads, static_cast<size_t>(smem), static_cast<cudaStream_t>(stream)>>>(
            bytes, n_bytes, offsets, rows, vocab, out, bad);
    } else {
        expand_gaps_atomic_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(bytes, n_bytes, offsets, rows,
                                                                                         vocab, out, bad);
    }
    BMS_CUDA(cudaGetLastError(), "gap-stream expansion launch");
    return BMS_SUCCESS;
}

int bms_mask_count(const int32_t* mask, int64_t vocab, int64_t* count, int32_t device, void* stream) {
    if (count == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "count must not be NULL");
    return bms_mask_budget(mask, 1, vocab, nullptr, count, nullptr, nullptr, device, stream);
}

int bms_verify_batch(const void* logits, int32_t dtype, const int32_t* masks, int64_t seqs, int64_t rows_per_seq,
                     int64_t vocab, const int64_t* proposals, const int32_t* lengths, const bms_policy* policy,
                     int64_t* row_tokens, int64_t* row_counts, int32_t* row_status, int32_t* row_budget,
                     int32_t* accept_len, int64_t* token, int32_t* kind, int32_t* seq_status,
                     const int32_t* mask_rows, int64_t mask_table_rows, void* workspace, int64_t workspace_bytes,
                     int32_t device, void* stream) {
    if (seqs < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "seqs must be nonnegative");
    if (rows_per_seq < 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows_per_seq must be at least 1");
    if (seqs > INT64_MAX / rows_per_seq) return fail(BMS_ERROR_INVALID_ARGUMENT, "batch too large");
    bms_policy P = {0, 1, 8, 0, 0.005, 0.02};
    if (row_budget) {
        if (row_counts == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "row_budget requires row_counts");
        BMS_CHECK(check_policy(policy));
        P = *policy;
    }
    const int64_t rows = seqs * rows_per_seq;
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab, device));
    if (seqs == 0) return BMS_SUCCESS;
    if (rows_per_seq > 1) BMS_CHECK(check_ptr(proposals, device, "proposals", 8));
    BMS_CHECK(check_ptr(lengths, device, "lengths", 4));
    BMS_CHECK(check_ptr(row_tokens, device, "row_tokens", 8));
    if (row_counts) BMS_CHECK(check_ptr(row_counts, device, "row_counts", 8));
    BMS_CHECK(check_ptr(row_status, device, "row_status", 4));
    if (row_budget) BMS_CHECK(check_ptr(row_budget, device, "row_budget", 4));
    BMS_CHECK(check_ptr(accept_len, device, "accept_len", 4));
    BMS_CHECK(check_ptr(token, device, "token", 8));
    BMS_CHECK(check_ptr(kind, device, "kind", 4));
    BMS_CHECK(check_ptr(seq_status, device, "seq_status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    if (mask_rows != nullptr) {
        if (mask_table_rows < 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "mask_table_rows must be at least 1");
        BMS_CHECK(check_ptr(mask_rows, device, "mask_rows", 4));
    }
    SelectParams p = base_params(logits, masks, rows, vocab);
    BMS_CHECK(attach_workspace(p, workspace, workspace_bytes, device));
    p.mask_rows = mask_rows;
    p.mask_table_rows = mask_table_rows;
    p.tokens = row_tokens;
    p.counts = row_counts;
    p.status = row_status;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    BMS_CHECK(launch_select<false>(dtype, p, device, s));
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 4;
    const int64_t need_seq = (seqs + 7) / 8;   // one warp per sequence
    const int64_t need_row = (rows + 255) / 256;
    int64_t need = need_seq > need_row ? need_seq : need_row;
    const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BMS_CUDA(cudaLaunchKernelEx(&cfg, verify_epilogue_kernel, row_tokens, static_cast<const int64_t*>(row_counts),
                                static_cast<const int32_t*>(row_status), seqs, rows_per_seq, vocab, proposals, lengths,
                                P, row_budget, accept_len, token, kind, seq_status),
             "verification epilogue launch");
    return BMS_SUCCESS;
}

int64_t bms_shard_granule_bytes(int32_t dtype, int64_t vocab_shard) {
    if (check_dtype(dtype) != BMS_SUCCESS || vocab_shard <= 0) return -1;
    return granule_bytes(dtype, vocab_shard);
}

int bms_shard_partials(const void* logits, int32_t dtype, const int32_t* masks, int64_t mask_words, int64_t rows,
                       int64_t vocab_shard, int64_t token_offset, double temperature, bms_partial* partials,
                       void* granules, int64_t granule_stride, int32_t device, void* stream) {
    return bms_shard_partials_indexed(logits, dtype, masks, mask_words, nullptr, 0, rows, vocab_shard, token_offset,
                                      temperature, partials, granules, granule_stride, device, stream);
}

int bms_shard_partials_indexed(const void* logits, int32_t dtype, const int32_t* masks, int64_t mask_words,
                               const int32_t* mask_rows, int64_t mask_table_rows, int64_t rows, int64_t vocab_shard,
                               int64_t token_offset, double temperature, bms_partial* partials, void* granules,
                               int64_t granule_stride, int32_t device, void* stream) {
    if (!std::isfinite(temperature) || temperature < 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "temperature must be finite and nonnegative");
    if (token_offset < 0 || token_offset % 32 != 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "token_offset must be a nonnegative multiple of 32");
    BMS_CHECK(check_vocab(vocab_shard));
    if (token_offset + vocab_shard > 2147483647LL) return fail(BMS_ERROR_INVALID_ARGUMENT, "vocabulary exceeds int32");
    if (mask_words < (token_offset + vocab_shard + 31) / 32)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "mask_words must cover token_offset + vocab_shard");
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab_shard, device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(partials, device, "partials", 16));
    const bool sample = temperature != 0;
    if (sample) {
        BMS_CHECK(check_ptr(granules, device, "granules", 16));
        if (granule_stride < granule_bytes(dtype, vocab_shard) || granule_stride % 16 != 0)
            return fail(BMS_ERROR_INVALID_ARGUMENT, "granule_stride must be a multiple of 16 of at least %lld bytes",
                        static_cast<long long>(granule_bytes(dtype, vocab_shard)));
    }
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    if (mask_rows != nullptr) {
        if (mask_table_rows < 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "mask_table_rows must be at least 1");
        BMS_CHECK(check_ptr(mask_rows, device, "mask_rows", 4));
    }
    SelectParams p = base_params(logits, masks, rows, vocab_shard);
    p.mask_rows = mask_rows;
    p.mask_table_rows = mask_table_rows;
    p.mask_stride = mask_words;
    p.mask_word_offset = token_offset / 32;
    p.token_offset = token_offset;
    p.partials = reinterpret_cast<GatherSlot*>(partials);
    if (!sample) return launch_select<false>(dtype, p, device, static_cast<cudaStream_t>(stream));
    p.granule_out = static_cast<uint8_t*>(granules);
    p.granule_stride = granule_stride;
    p.temperature = temperature;
    p.inv_temperature = inverse_temperature(temperature);
    p.scale2 = sampler_scale2(temperature);
    p.scale = static_cast<float>(1.4426950408889634 / temperature);
    return launch_select<true>(dtype, p, device, static_cast<cudaStream_t>(stream));
}

int bms_shard_merge(const bms_partial* partials, int32_t shards, int32_t shard, int64_t rows, double temperature,
                    const double* uniforms, const void* logits, int32_t dtype, const int32_t* masks, int64_t mask_words,
                    int64_t vocab_shard, int64_t token_offset, const void* granules, int64_t granule_stride,
                    int64_t* tokens, int64_t* counts, int32_t* status, int32_t device, void* stream) {
    if (shards < 1 || shards > 32) return fail(BMS_ERROR_INVALID_ARGUMENT, "shards must be in [1, 32]");
    if (shard < 0 || shard >= shards) return fail(BMS_ERROR_INVALID_ARGUMENT, "shard must be in [0, shards)");
    if (rows < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows must be nonnegative");
    if (!std::isfinite(temperature) || temperature < 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "temperature must be finite and nonnegative");
    BMS_CHECK(check_device(device));
    if (rows == 0) return BMS_SUCCESS;
    BMS_CHECK(check_ptr(partials, device, "partials", 16));
    BMS_CHECK(check_ptr(tokens, device, "tokens", 8));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    const bool sample = temperature != 0;
    if (sample) {
        BMS_CHECK(check_dtype(dtype));
        BMS_CHECK(check_vocab(vocab_shard));
        if (token_offset < 0 || token_offset % 32 != 0 || mask_words < (token_offset + vocab_shard + 31) / 32)
            return fail(BMS_ERROR_INVALID_ARGUMENT, "invalid shard token_offset / mask_words");
        BMS_CHECK(check_ptr(uniforms, device, "uniforms", 8));
        BMS_CHECK(check_ptr(logits, device, "logits", static_cast<size_t>(elem_bytes(dtype))));
        BMS_CHECK(check_ptr(masks, device, "masks", 4));
        BMS_CHECK(check_ptr(granules, device, "granules", 16));
        if (granule_stride < granule_bytes(dtype, vocab_shard))
            return fail(BMS_ERROR_INVALID_ARGUMENT, "granule_stride too small");
    }
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
    const int64_t need = (rows + 3) / 4;
    const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const GatherSlot* parts = reinterpret_cast<const GatherSlot*>(partials);
    const float sc2 = sample ? sampler_scale2(temperature) : 0.0f;
    const double inv = inverse_temperature(temperature);
    const uint8_t* lg = static_cast<const uint8_t*>(logits);
    const uint8_t* gr = static_cast<const uint8_t*>(granules);
    if (!sample) {
        shard_merge_kernel<float, false><<<grid, 128, 0, s>>>(parts, shards, shard, rows, 0.0, 0.0, 0.0f, nullptr, nullptr,
                                                              nullptr, 0, 0, 0, nullptr, 0, tokens, counts, status);
    } else if (dtype == BMS_FLOAT32) {
        shard_merge_kernel<float, true><<<grid, 128, 0, s>>>(parts, shards, shard, rows, temperature, inv, sc2, uniforms, lg,
                                                             masks, mask_words, vocab_shard, token_offset, gr,
                                                             granule_stride, tokens, counts, status);
    } else if (dtype == BMS_BFLOAT16) {
        shard_merge_kernel<__nv_bfloat16, true><<<grid, 128, 0, s>>>(parts, shards, shard, rows, temperature, inv, sc2,
                                                                     uniforms, lg, masks, mask_words, vocab_shard,
                                                                     token_offset, gr, granule_stride, tokens, counts,
                                                                     status);
    } else {
        shard_merge_kernel<__half, true><<<grid, 128, 0, s>>>(parts, shards, shard, rows, temperature, inv, sc2, uniforms, lg,
                                                              masks, mask_words, vocab_shard, token_offset, gr,
                                                              granule_stride, tokens, counts, status);
    }
    BMS_CUDA(cudaGetLastError(), "shard merge launch");
    return BMS_SUCCESS;
}

// ---------------------------------------------------------------- peer-memory shard exchange
static_assert(sizeof(bms_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");

int64_t bms_exchange_bytes(int32_t ranks, int64_t rows_cap) {
    if (ranks < 1 || ranks > kMaxExchangeRanks || rows_cap < 1) return -1;
    return exchange_bytes(ranks, rows_cap);
}

int bms_exchange_create(int32_t device, int32_t ranks, int64_t rows_cap, void** area, bms_ipc_handle* handle) {
    if (area == nullptr || handle == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "area and handle must not be NULL");
    if (ranks < 1 || ranks > kMaxExchangeRanks) return fail(BMS_ERROR_INVALID_ARGUMENT, "ranks must be in [1, 8]");
    if (rows_cap < 1) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows_cap must be positive");
    BMS_CHECK(check_device(device));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    void* p = nullptr;
    const size_t bytes = static_cast<size_t>(exchange_bytes(ranks, rows_cap));
    BMS_CUDA(cudaMalloc(&p, bytes), "exchange area allocation");
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(BMS_ERROR_CUDA, "exchange area export: %s", cudaGetErrorString(e));
    }
    memcpy(handle->bytes, &h, sizeof(h));
    *area = p;
    return BMS_SUCCESS;
}

int bms_exchange_open(int32_t device, const bms_ipc_handle* handle, void** area) {
    if (area == nullptr || handle == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "area and handle must not be NULL");
    BMS_CHECK(check_device(device));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->bytes, sizeof(h));
    void* p = nullptr;
    BMS_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "exchange area mapping");
    *area = p;
    return BMS_SUCCESS;
}

int bms_exchange_close(int32_t device, void* area) {
    if (area == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "area must not be NULL");
    BMS_CHECK(check_device(device));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    BMS_CUDA(cudaIpcCloseMemHandle(area), "exchange area unmapping");
    return BMS_SUCCESS;
}

int bms_exchange_destroy(int32_t device, void* area) {
    if (area == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "area must not be NULL");
    BMS_CHECK(check_device(device));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    BMS_CUDA(cudaFree(area), "exchange area release");
    return BMS_SUCCESS;
}

namespace {
int check_exchange(void* const* areas, int32_t ranks, int32_t rank, int64_t rows_cap, uint32_t epoch, int64_t rows,
                   int device) {
    if (areas == nullptr) return fail(BMS_ERROR_INVALID_ARGUMENT, "areas must not be NULL");
    if (ranks < 1 || ranks > kMaxExchangeRanks) return fail(BMS_ERROR_INVALID_ARGUMENT, "ranks must be in [1, 8]");
    if (rank < 0 || rank >= ranks) return fail(BMS_ERROR_INVALID_ARGUMENT, "rank must be in [0, ranks)");
    if (rows_cap < 1 || rows > rows_cap) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows exceed the exchange area's rows_cap");
    if (epoch == 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "epoch must be at least 1");
    for (int q = 0; q < ranks; ++q)
        if (areas[q] == nullptr || reinterpret_cast<uintptr_t>(areas[q]) % 256 != 0)
            return fail(BMS_ERROR_INVALID_ARGUMENT, "exchange areas must be non-NULL and 256-byte aligned");
    return check_ptr(areas[rank], device, "this rank's exchange area", 256);
}
}  // namespace

int bms_shard_partials_exchange(const void* logits, int32_t dtype, const int32_t* masks, int64_t mask_words,
                                int64_t rows, int64_t vocab_shard, int64_t token_offset, void* const* areas,
                                int32_t ranks, int32_t rank, int64_t rows_cap, uint32_t epoch, int32_t device,
                                void* stream) {
    if (token_offset < 0 || token_offset % 32 != 0)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "token_offset must be a nonnegative multiple of 32");
    BMS_CHECK(check_vocab(vocab_shard));
    if (token_offset + vocab_shard > 2147483647LL) return fail(BMS_ERROR_INVALID_ARGUMENT, "vocabulary exceeds int32");
    if (mask_words < (token_offset + vocab_shard + 31) / 32)
        return fail(BMS_ERROR_INVALID_ARGUMENT, "mask_words must cover token_offset + vocab_shard");
    BMS_CHECK(select_common(dtype, logits, masks, rows, vocab_shard, device));
    BMS_CHECK(check_exchange(areas, ranks, rank, rows_cap, epoch, rows, device));
    if (rows == 0) return BMS_SUCCESS;
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    SelectParams p = base_params(logits, masks, rows, vocab_shard);
    p.mask_stride = mask_words;
    p.mask_word_offset = token_offset / 32;
    p.token_offset = token_offset;
    for (int q = 0; q < ranks; ++q) {
        p.xarea[q] = static_cast<uint8_t*>(areas[q]);
        p.xpeer[q] = exchange_slot(p.xarea[q], ranks, rows_cap, epoch, rank);
    }
    p.partials = p.xpeer[rank];
    p.xranks = ranks;
    p.xrank = rank;
    p.xepoch = epoch;
    return launch_select<false>(dtype, p, device, static_cast<cudaStream_t>(stream));
}

int bms_shard_merge_exchange(void* const* areas, int32_t ranks, int32_t rank, int64_t rows_cap, uint32_t epoch,
                             int64_t rows, int64_t* tokens, int64_t* counts, int32_t* status, int32_t device,
                             void* stream) {
    if (rows < 0) return fail(BMS_ERROR_INVALID_ARGUMENT, "rows must be nonnegative");
    BMS_CHECK(check_device(device));
    BMS_CHECK(check_exchange(areas, ranks, rank, rows_cap, epoch, rows, device));
    BMS_CHECK(check_ptr(tokens, device, "tokens", 8));
    if (counts) BMS_CHECK(check_ptr(counts, device, "counts", 8));
    BMS_CHECK(check_ptr(status, device, "status", 4));
    DeviceGuard guard;
    BMS_CUDA(guard.enter(device), "cudaSetDevice");
    ExchangeAreas a{};
    for (int q = 0; q < ranks; ++q) a.a[q] = static_cast<uint8_t*>(areas[q]);
    // Every step launches at least one CTA: its last CTA releases this rank's slot even for an
    // empty batch.
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
    const int64_t need = rows > 0 ? (rows + 3) / 4 : 1;
    const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
    exchange_merge_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(a, ranks, rank, rows_cap, epoch, rows,
                                                                                 tokens, counts, status);
    BMS_CUDA(cudaGetLastError(), "exchange merge launch");
    return BMS_SUCCESS;
}

}  // extern "C"
