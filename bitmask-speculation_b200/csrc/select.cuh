// Masked selection over packed grammar masks: one persistent streaming kernel
// for (a) fused masked argmax + valid count + NaN status and (b) masked
// online-softmax sampling by inverse CDF.
//
// Semantics follow the reference implementation of karthikeyansura/bitmask-
// speculation: csrc/reduce.cuh:19-62 (larger value wins, ties go to the lower
// token ID, NaN anywhere in the row fails it, padding bits of the last word are
// ignored), csrc/argmax.cu:77-98 (status 0 ok, 1 no valid token, 2 NaN; token -1
// on error) and csrc/sample.cu:24-112 / kernels/reference.py:10-52 (weights
// exp((x - max) / T), first token whose running mass exceeds u * total, status
// 3 bad uniform, 4 no finite mass, 5 valid +inf).
//
// Structure (B200 / sm_100a):
//  * A cluster of C CTAs owns one row at a time; CTA rank r streams tokens
//    [r*L, (r+1)*L) of the row.  Each cluster walks a contiguous block of rows
//    (persistent grid).
//  * One producer warp moves 16 KB chunks of logits plus their mask words from
//    HBM into a ring of shared-memory stages with 1-D bulk copies (TMA engine)
//    completing on mbarriers; eight consumer warps reduce them.  Rows whose
//    addresses are not 16-byte aligned use the same kernel with the consumer
//    warps loading the chunk themselves (kBulk = false).
//  * Consumer warp w of a chunk owns a contiguous 2 KB slice; each lane reads
//    16-byte vectors and the mask bits covering them from shared memory.
//  * Consumer warps only stream: at the end of a row each warp reduces its own
//    partial with redux.sync and hands it to a finalizer warp through a
//    double-buffered shared-memory slot guarded by mbarriers, then starts the
//    next row.  The finalizer merges the eight warp partials, recovers the
//    argmax index by re-reading the one 2 KB warp slice that holds the first
//    maximum, all-gathers the CTA partials across the cluster through
//    distributed shared memory (st.shared::cluster + remote mbarrier arrive)
//    and writes the row's outputs -- overlapped with the next row's streaming.
//    Argmax keys are (order-preserving float bits << 32 | ~index): a max merge.
//  * The sampler records one (reference, mass) pair per (chunk, warp) "granule"
//    in shared memory during the single streaming pass (fp32 MUFU ex2 weights;
//    the warp's reference max is raised only when a weight would exceed 2^20);
//    the finalizer merges ranks in fixed order in fp64, then re-reads only the
//    granule that holds u * total and walks it with exact fp64 weights
//    exp((x - M) / T).
//  * With a caller workspace the work can also arrive as tickets: whole rows
//    and split pieces merged through the workspace (dynamic schedule), or, for
//    small sampler batches, blocks of chunks whose granule records go straight
//    to the workspace for a second launch to merge (flat schedule, kFlat).
//  * Every wait is bounded (about one second, %globaltimer); on expiry the CTA
//    stops waiting, reports status 7 for its rows and still completes the
//    cluster protocol, so no wait can hang the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>
#include <type_traits>

#include "ptx.cuh"

namespace bms {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;       // bulk-copy issue
constexpr int kFinalizerWarp = kConsumerWarps + 1;  // per-row merge, index recovery, sampling walk
constexpr int kThreads = kConsumerThreads + 64;
constexpr int kChunkBytes = 16384;               // logits bytes per stage
constexpr int kWarpBytes = kChunkBytes / kConsumerWarps;
constexpr int kVecsPerLane = kWarpBytes / 16 / 32;  // 16-byte vectors per lane per chunk
constexpr int kMaxCluster = 16;
constexpr int kMaxChunksSampler = 64;  // granule table capacity (chunks per segment)
constexpr int kMaxExchangeRanks = 8;   // ranks of a peer-memory shard exchange
constexpr uint64_t kTimeoutNs = 1000000000ull;
// Sampler: a lane mass above 2^20 raises the warp's reference max (no weight exceeds 2^20).
constexpr float kRaiseMass = 0x1p20f;
// Sampler walk: fp32 exponents are clamped here (a reference below the max gives t <= 20).
constexpr float kWalkClamp = 64.0f;

enum Status : int32_t {
    kOk = 0,
    kEmpty = 1,
    kNaN = 2,
    kBadUniform = 3,
    kNoMass = 4,
    kPosInf = 5,
    kBadLength = 6,
    kTimeout = 7,
    kBadMaskRow = 8,
};

enum Flags : uint32_t { kFlagNaN = 1u, kFlagAbort = 2u, kFlagBadMaskRow = 4u };

// Status of a merged argmax partial: a timed-out wait, then a bad mask-table index, then NaN
// anywhere in the row, then no valid token (csrc/argmax.cu:77-98 for the last two).
__host__ __device__ constexpr int32_t argmax_status(uint32_t flags, uint32_t total) {
    return (flags & kFlagAbort) ? kTimeout : (flags & kFlagBadMaskRow) ? kBadMaskRow : (flags & kFlagNaN) ? kNaN
                                                                       : (total == 0u) ? kEmpty : kOk;
}

// ----------------------------------------------------------------- dtypes
template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kBytes = 4;
    static constexpr int kVec = 4;  // tokens per 16-byte vector
    using NanAcc = float;
    __device__ static NanAcc nan_init() { return 0.0f; }
    __device__ static void decode(const uint4& r, float (&v)[kVec]) {
        v[0] = __uint_as_float(r.x);
        v[1] = __uint_as_float(r.y);
        v[2] = __uint_as_float(r.z);
        v[3] = __uint_as_float(r.w);
    }
    __device__ static void nan_update(NanAcc& a, const uint4& r) {
        a = ptx::max_nan(a, ptx::max_nan(ptx::max_nan(__uint_as_float(r.x), __uint_as_float(r.y)),
                                         ptx::max_nan(__uint_as_float(r.z), __uint_as_float(r.w))));
    }
    __device__ static bool has_nan(NanAcc a) { return a != a; }
    __device__ static float load(const void* p, int64_t i) { return static_cast<const float*>(p)[i]; }
    __device__ static uint32_t raw(const void* p, int64_t i) { return static_cast<const uint32_t*>(p)[i]; }
};

template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kBytes = 2;
    static constexpr int kVec = 8;
    using NanAcc = uint32_t;  // two packed bf16 maxima
    __device__ static NanAcc nan_init() { return 0u; }
    __device__ static void decode(const uint4& r, float (&v)[kVec]) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
    __device__ static void nan_update(NanAcc& a, const uint4& r) {
        a = ptx::max_nan_bf16x2(a, ptx::max_nan_bf16x2(ptx::max_nan_bf16x2(r.x, r.y), ptx::max_nan_bf16x2(r.z, r.w)));
    }
    __device__ static bool has_nan(NanAcc a) { return (a & 0x7FFFu) > 0x7F80u || ((a >> 16) & 0x7FFFu) > 0x7F80u; }
    __device__ static float load(const void* p, int64_t i) {
        return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p)[i]) << 16);
    }
    __device__ static uint32_t raw(const void* p, int64_t i) { return static_cast<const uint16_t*>(p)[i]; }
    static constexpr uint32_t kNegInf2 = 0xFF80FF80u;
    __device__ static uint32_t max2(uint32_t a, uint32_t b) { return ptx::max_bf16x2(a, b); }
    __device__ static float lo(uint32_t u) { return __uint_as_float(u << 16); }
    __device__ static float hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
};

template <>
struct Elem<__half> {
    static constexpr int kBytes = 2;
    static constexpr int kVec = 8;
    using NanAcc = uint32_t;  // two packed fp16 maxima
    __device__ static NanAcc nan_init() { return 0u; }
    __device__ static void decode(const uint4& r, float (&v)[kVec]) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h;
            memcpy(&h, &w[i], 4);
            const float2 f = __half22float2(h);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    __device__ static void nan_update(NanAcc& a, const uint4& r) {
        a = ptx::max_nan_f16x2(a, ptx::max_nan_f16x2(ptx::max_nan_f16x2(r.x, r.y), ptx::max_nan_f16x2(r.z, r.w)));
    }
    __device__ static bool has_nan(NanAcc a) { return (a & 0x7FFFu) > 0x7C00u || ((a >> 16) & 0x7FFFu) > 0x7C00u; }
    __device__ static float load(const void* p, int64_t i) {
        return __half2float(static_cast<const __half*>(p)[i]);
    }
    __device__ static uint32_t raw(const void* p, int64_t i) { return static_cast<const uint16_t*>(p)[i]; }
    static constexpr uint32_t kNegInf2 = 0xFC00FC00u;
    __device__ static uint32_t max2(uint32_t a, uint32_t b) { return ptx::max_f16x2(a, b); }
    __device__ static float lo(uint32_t u) { return __half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xFFFFu))); }
    __device__ static float hi(uint32_t u) { return __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16))); }
};

// Invalid tokens of a 16-bit vector set to -inf, valid ones kept: the 8 mask bits are spread
// to byte sign bits with one multiply, then sign-replicating byte permutes build the
// per-token 16-bit masks (token 2k in the low half of pair k).
template <typename E>
__device__ __forceinline__ void mask_pairs(const uint4& r, uint32_t bits8, uint32_t (&q)[4]) {
    const uint32_t slo = (bits8 & 0xFu) * 0x10204080u;  // byte k sign bit = mask bit k
    const uint32_t shi = (bits8 >> 4) * 0x10204080u;    // byte k sign bit = mask bit 4 + k
    q[0] = ptx::select_bits(r.x, ptx::prmt(slo, 0u, 0x9988u), E::kNegInf2);
    q[1] = ptx::select_bits(r.y, ptx::prmt(slo, 0u, 0xBBAAu), E::kNegInf2);
    q[2] = ptx::select_bits(r.z, ptx::prmt(shi, 0u, 0x9988u), E::kNegInf2);
    q[3] = ptx::select_bits(r.w, ptx::prmt(shi, 0u, 0xBBAAu), E::kNegInf2);
}

// Sum over a lane's 32 (16-bit) or 16 (fp32) masked tokens of 2^((x - m) log2(e) / T), one MUFU
// ex2 per token, pairwise sums per vector and across vectors.  Invalid tokens hold -inf (weight 0).
//  kMode 0: t = fma(x, s, c) with s = log2(e)/T and c = -(m s) rounded (the caller rescales the
//           sum by 2^(rounding error of c), which is common to every token);
//  kMode 1: t = (0.5x - 0.5m) * 2s -- cannot overflow for any finite logits;
//  kMode 2: as 1, clamped at 0 for an infinite scale (T below ~1e-38, where x == m gives 0 * inf).
template <typename E, int kMode>
__device__ __forceinline__ float lane_mass(const uint32_t (&q16)[kVecsPerLane][4],
                                           const float (&q32)[kVecsPerLane][E::kVec], float c, float scale) {
    constexpr int kVec = E::kVec;
    float part[kVecsPerLane];
#pragma unroll
    for (int j = 0; j < kVecsPerLane; ++j) {
        float w[kVec];
#pragma unroll
        for (int i = 0; i < kVec; ++i) {
            float x;
            if constexpr (E::kBytes == 2) x = (i & 1) ? E::hi(q16[j][i >> 1]) : E::lo(q16[j][i >> 1]);
            else x = q32[j][i];
            float t;
            if constexpr (kMode == 0) {
                t = fmaf(x, scale, c);
            } else {
                t = fmaf(x, 0.5f, c) * scale;
                if constexpr (kMode == 2) t = fminf(t, 0.0f);
            }
            w[i] = ptx::ex2(t);
        }
#pragma unroll
        for (int h = kVec / 2; h >= 1; h >>= 1)
#pragma unroll
            for (int i = 0; i < h; ++i) w[i] += w[i + h];
        part[j] = w[0];
    }
#pragma unroll
    for (int h = kVecsPerLane / 2; h >= 1; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; ++i) part[i] += part[i + h];
    return part[0];
}

// Mode 0 of lane_mass with paired fp32 arithmetic for 16-bit logits (fma.rn.f32x2 / add.rn.f32x2):
// the two tokens of a packed pair share one FFMA2 and their weights one FADD2.
template <typename E>
__device__ __forceinline__ float lane_mass_fast(const uint32_t (&q16)[kVecsPerLane][4],
                                                const float (&q32)[kVecsPerLane][E::kVec], float c, float scale) {
    if constexpr (E::kBytes == 4) {
        return lane_mass<E, 0>(q16, q32, c, scale);
    } else {
        const uint64_t s2 = ptx::pack2(scale, scale), c2 = ptx::pack2(c, c);
        uint64_t part[kVecsPerLane];
#pragma unroll
        for (int j = 0; j < kVecsPerLane; ++j) {
            uint64_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint64_t t = ptx::fma2(ptx::pack2(E::lo(q16[j][i]), E::hi(q16[j][i])), s2, c2);
                float t0, t1;
                ptx::unpack2(t, t0, t1);
                w[i] = ptx::pack2(ptx::ex2(t0), ptx::ex2(t1));
            }
            part[j] = ptx::add2(ptx::add2(w[0], w[1]), ptx::add2(w[2], w[3]));
        }
        static_assert(kVecsPerLane == 4, "pairwise tree over four vectors");
        const uint64_t acc = ptx::add2(ptx::add2(part[0], part[1]), ptx::add2(part[2], part[3]));
        float a, b;
        ptx::unpack2(acc, a, b);
        return a + b;
    }
}

// ----------------------------------------------------------------- params
// Per-row partial of one rank (cluster CTA or vocabulary shard), 32 bytes.  Argmax: a = ordered
// max bits, b = ~(global index of the first maximum), c = valid count, d = flags.  Sampler:
// a = max bits, b = valid count, c = flags, s = mass relative to the max.
struct alignas(16) GatherSlot {
    uint32_t a, b, c, d;
    double s;
    double pad;  // peer-memory exchange: the step's epoch (low word), read back by the merge
};
static_assert(sizeof(GatherSlot) == 32 && offsetof(GatherSlot, pad) == 24, "exchange merge reads the tag at byte 24");

struct SelectParams {
    const void* logits;      // [rows, logit_stride] elements
    const int32_t* masks;    // [rows, mask_stride] words
    int64_t rows;
    int64_t vocab;           // tokens per row
    int64_t logit_stride;    // elements between rows
    int64_t mask_stride;     // words between rows
    int64_t segment;         // tokens per cluster rank, multiple of 32
    int64_t token_offset;    // added to reported token ids (vocabulary shards)
    int64_t* tokens;         // [rows] selected token, -1 on error
    int64_t* counts;         // [rows] valid-token count (nullable)
    int32_t* status;         // [rows]
    // sampler
    const double* uniforms;  // [rows]
    double temperature;
    double inv_temperature;  // 1 / T where finite, else 0 (exponents then divide by T)
    float scale2;            // 2 * log2(e) / T as float, clamped to >= the smallest denormal
    float scale;             // log2(e) / T as float (inf for tiny T)
    // vocabulary shards
    int64_t mask_word_offset;  // added to every mask word index (the shard's first word in the full row)
    GatherSlot* partials;      // non-null: write one partial record per row instead of the outputs
    uint8_t* granule_out;      // sampler partials: per-row granule record (SamplerRecord layout)
    int64_t granule_stride;    // bytes between granule records
    // dynamic schedule (one-CTA clusters; ws == nullptr: each cluster owns a fixed block of rows)
    uint8_t* ws;               // workspace (layout above)
    int64_t ws_rows;           // its split-row capacity
    int64_t whole_rows;        // tickets [0, whole_rows) are rows 0.. handed out whole
    int64_t tickets;           // then blocks of chunks over the split rows' chunks (row-major):
    int64_t tier_tickets[2];   //   tier_tickets[i] blocks of tier_block[i] chunks (i = 0, 1), then
    int32_t tier_block[2];     //   blocks of `block` chunks
    int32_t block;
    uint32_t epoch;            // this launch's tag, never 0
    int32_t dynamic_always;    // host only: take the dynamic schedule for any batch size
    int32_t flat;              // sampler: consumers store granule records to the workspace (flat schedule)
    int32_t ws_flat;           // host only: the workspace has the flat-record area
    // mask table (nullable): row r's mask is row mask_rows[r] of `masks` ([mask_table_rows, W]);
    // an index outside [0, mask_table_rows) fails the row with status 8
    const int32_t* mask_rows;
    int64_t mask_table_rows;
    // peer-memory shard exchange (xranks > 0, argmax partials): every row's partial also goes to
    // xpeer[q] + row, this rank's slot in rank q's exchange area (ExchangeHeader below)
    GatherSlot* xpeer[kMaxExchangeRanks];
    uint8_t* xarea[kMaxExchangeRanks];  // every rank's exchange area (xarea[xrank] is this rank's)
    int32_t xranks;
    int32_t xrank;
    uint32_t xepoch;                    // this exchange step, >= 1, one more per step
};

// ----------------------------------------------------------------- peer-memory shard exchange
// Each rank of a vocabulary-sharded group owns one exchange area in its device memory, mapped
// by every peer (CUDA IPC): a header of epoch flags, then partial slots [2][ranks][rows_cap],
// double-buffered by epoch parity.  Step e: rank q's selection launch waits until every rank
// has merged step e - 2 (consumed[r] in q's own area, so slot e & 1 is free everywhere), stores
// each row's partial into slot e & 1 of every area at [q][row] while it streams, and its last
// CTA publishes ready[q] = e in every area (release, system scope).  Rank r's merge launch waits
// for ready[q] >= e of every rank q in its own area, merges, and its last CTA publishes
// consumed[r] = e in every area.  Every wait is bounded; a selection launch that gave up stores
// and publishes nothing, so the peers' merges report status 7.
struct alignas(128) ExchangeHeader {
    uint32_t ready[kMaxExchangeRanks];     // rank q's partials of step ready[q] are in this area
    uint32_t consumed[kMaxExchangeRanks];  // rank r merged step consumed[r]
    uint32_t select_done;                  // CTAs of this rank's running selection launch (+ 2^16 per timeout)
    uint32_t merge_done;                   // CTAs of this rank's running merge launch
};

__host__ __device__ constexpr int64_t exchange_slots_offset() { return 256; }
static_assert(sizeof(ExchangeHeader) <= exchange_slots_offset(), "exchange header fits before the slots");
__host__ __device__ constexpr int64_t exchange_bytes(int64_t ranks, int64_t rows_cap) {
    return exchange_slots_offset() + 2 * ranks * rows_cap * static_cast<int64_t>(sizeof(GatherSlot));
}
// Rank q's slot of step `epoch` in an area.
__host__ __device__ inline GatherSlot* exchange_slot(uint8_t* area, int64_t ranks, int64_t rows_cap, uint32_t epoch,
                                                     int64_t q) {
    return reinterpret_cast<GatherSlot*>(area + exchange_slots_offset()) + ((epoch & 1u) * ranks + q) * rows_cap;
}

// Bounded wait (one second of %globaltimer) until flags[i] - target >= 0 (as signed) for every
// i < n; false on time-out.  Polls back off (__nanosleep) so that many waiting CTAs do not crowd
// the flag's memory while a peer's store to it is on its way.
__device__ inline bool wait_flags_at_least(const uint32_t* flags, int n, uint32_t target) {
    const uint64_t t0 = ptx::globaltimer();
    for (int i = 0; i < n; ++i) {
        while (static_cast<int32_t>(ptx::ld_acquire_sys(flags + i) - target) < 0) {
            if (ptx::globaltimer() - t0 > kTimeoutNs) return false;
            __nanosleep(128);
        }
    }
    return true;
}

// Order-preserving map of a non-NaN float to uint32 (-0.0 folded onto +0.0).
__device__ __forceinline__ uint32_t ordered_bits(float v) {
    v = v + 0.0f;  // -0.0 + 0.0 == +0.0
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float ordered_to_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// ----------------------------------------------------------------- shared memory
template <typename T>
struct Layout {
    static constexpr int kTokensPerChunk = kChunkBytes / Elem<T>::kBytes;
    static constexpr int kTokensPerWarp = kTokensPerChunk / kConsumerWarps;
    static constexpr int kMaskWords = kTokensPerChunk / 32 + 4;  // + misalignment slack
    static constexpr int kMaskBytes = ((kMaskWords * 4) + 15) / 16 * 16;
    static constexpr int kStageBytes = kChunkBytes + kMaskBytes;
};

// One consumer warp's contribution to one row.
struct alignas(16) WarpPartial {
    uint32_t key;    // argmax: ordered masked max (0 = no valid token) | sampler: ordered running max
    uint32_t chunk;  // argmax: first chunk in which a lane of this warp reached `key`
    uint32_t count;  // valid tokens
    uint32_t flags;  // kFlagNaN
    double mass;     // sampler: the warp's mass relative to its running max (fp64)
    double pad;
};

constexpr int kStagesMax = 8;

// A unit of work: chunks [c0, c1) of one row's segment.  A whole unit is finished in this CTA
// (or cluster); a split unit is one piece of a row whose pieces are merged through the
// workspace by the CTA that completes the row; the end unit stops the CTA.
enum UnitKind : int32_t { kUnitWhole = 0, kUnitSplit = 1, kUnitEnd = 2 };

struct alignas(16) Unit {
    int64_t row;
    int32_t c0, c1;
    int32_t kind;
    int32_t mask_bad;  // the row's mask-table index was out of range (table row 0 is read instead)
    int64_t mask_row;  // row of `masks` holding this row's mask words
};

constexpr int kUnitSlots = 4;  // producer -> consumers descriptor ring

struct alignas(16) Shared {
    uint64_t full[kStagesMax];
    uint64_t empty[kStagesMax];
    uint64_t part_full[2];   // consumers -> finalizer, one arrive per consumer warp
    uint64_t part_empty[2];  // finalizer -> consumers, slot (and granule table) reusable
    uint64_t gather[2];      // cluster all-gather, one arrive per rank
    uint64_t unit_full[kUnitSlots];   // producer -> consumers, descriptor written
    uint64_t unit_empty[kUnitSlots];  // consumers -> producer, one arrive per consumer warp
    Unit units[kUnitSlots];
    Unit part_unit[2];                // the unit of each partial slot (consumers -> finalizer)
    double part_uniform[2];           // sampler: the unit row's uniform, fetched while it streams
    GatherSlot slots[2][kMaxCluster];
    WarpPartial part[2][kConsumerWarps];
    int32_t piece_c0[32];             // finalizer: first chunks of a split row's pieces, in order
    GatherSlot piece_part[32];        // finalizer: their partials
    // Flat schedule: each consumer warp's last granule record and its destination (nullptr: none),
    // stored one chunk later, after the next stage's release, so that no release waits for it.
    uint4 flat_rec[kConsumerWarps];
    uint4* flat_dst[kConsumerWarps];
    volatile int32_t abort;
};

// ----------------------------------------------------------------- dynamic-schedule workspace
// Sampler pieces publish their granules already scaled to the piece's max, so that the merge
// needs only the pieces' partials and the row's granules.  Caller-owned device memory, zeroed
// once.  Every launch returns its ticket, done and row
// counters to zero (after a timed-out wait, its last CTA clears every row counter) and tags its
// pieces with its epoch (never 0), so that consecutive launches and graph replays need no
// clearing and pieces of an earlier launch are never merged.  Layout: WsHeader | row counters [rows_cap] | pieces [rows_cap][kWsChunks] |
// granules [rows_cap][kConsumerWarps][kWsChunks] doubles (warp-major, as in shared memory).
constexpr int kWsChunks = 64;  // chunks per split row (longer rows are not split)

struct alignas(64) WsHeader {
    unsigned long long tickets;  // next ticket
    unsigned long long done;     // CTAs finished (low word) and timed out (high word): after a
                                 // timeout the last CTA clears every row counter
    unsigned long long pad[6];
};

struct alignas(16) WsPiece {     // one per (split row, first chunk of a piece)
    uint32_t epoch;              // launch that wrote it
    int32_t c1;                  // end chunk of the piece
    uint32_t pad[2];
    GatherSlot part;             // the piece's partial (argmax or sampler form)
};

__host__ __device__ constexpr int64_t ws_counters_offset() { return sizeof(WsHeader); }
__host__ __device__ constexpr int64_t ws_pieces_offset(int64_t rows_cap) {
    return (ws_counters_offset() + 8 * rows_cap + 255) / 256 * 256;
}
__host__ __device__ constexpr int64_t ws_granules_offset(int64_t rows_cap) {
    return ws_pieces_offset(rows_cap) + static_cast<int64_t>(sizeof(WsPiece)) * kWsChunks * rows_cap;
}
// Flat schedule: one 16-byte record per (row, chunk, warp) granule, [rows_cap][kWsChunks][warp]:
// (reference max, mass relative to it as fp32 bits, valid tokens, flags), stored by the consumer
// warp that streamed the granule.  A separate area, so that no record can pass for a piece.
__host__ __device__ constexpr int64_t ws_flat_offset(int64_t rows_cap) {
    return (ws_granules_offset(rows_cap) + 8ll * kConsumerWarps * kWsChunks * rows_cap + 255) / 256 * 256;
}
// Workspace without the flat-record area (argmax-only callers).
__host__ __device__ constexpr int64_t ws_split_bytes(int64_t rows_cap) { return ws_flat_offset(rows_cap); }
__host__ __device__ constexpr int64_t ws_bytes(int64_t rows_cap) {
    return ws_flat_offset(rows_cap) + 16ll * kConsumerWarps * kWsChunks * rows_cap;
}

// Sampler-only shared memory after the control block.
struct SamplerShared {
    // Per row slot, one entry per (chunk, warp) granule at [warp * kMaxChunksSampler + chunk]
    // (warp-major: a warp's lanes walking consecutive chunks hit distinct banks): while streaming
    // a float2 (running max, mass relative to it); after the row, the granule's mass relative to
    // its warp's max (double).
    double granules[2][kMaxChunksSampler * kConsumerWarps];
    float walk[32][33];                                       // finalizer: the walked granule, one row per lane
    double fac[kConsumerWarps];                               // finalizer: warp max -> row max factors
};

// Bounded mbarrier wait.  Returns false (and latches `abort`) after kTimeoutNs.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int32_t* abort,
                                             bool cluster_scope = false) {
    if (cluster_scope ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer();
    for (;;) {
        if (*abort) return false;
        if (cluster_scope ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity)) return true;
        if (ptx::globaltimer() - t0 > kTimeoutNs) {
            *abort = 1;
            return false;
        }
    }
}

// Bounded wait that ignores the abort latch: used only to let issued copies land.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = ptx::globaltimer();
    while (!ptx::mbar_try_wait(bar, parity)) {
        if (ptx::globaltimer() - t0 > kTimeoutNs) return;
    }
}

// ----------------------------------------------------------------- warp helpers (finalizer)
__device__ __forceinline__ double warp_inclusive_scan(double v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Sum of lanes 0..7 (every other lane holds 0), complete on lanes 0..7.
__device__ __forceinline__ double warp_sum8(double v) {
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// exp((x - M) / T) for a valid, finite-or(-inf) logit; the reference's weight.
// exp(d / T) (d below about 14 T: references trail maxima by at most 2^20 in weight), multiplying by 1 / T where that is finite (inv > 0) and dividing
// otherwise (denormal temperatures).
__device__ __forceinline__ double scaled_exp(double d, double temp, double inv) {
    return inv > 0.0 ? exp(d * inv) : exp(d / temp);
}

__device__ __forceinline__ double exact_weight(float x, double M, double T, double inv) {
    return x > -__int_as_float(0x7F800000) ? scaled_exp(static_cast<double>(x) - M, T, inv) : 0.0;
}


// A finalizer lane's slice of n consecutive tokens: 16-bit logits kept packed two per word.
template <typename E, int n>
struct Slice {
    static constexpr int kWords = E::kBytes == 2 ? n / 2 : n;
    uint32_t w[kWords];
    uint32_t bits;  // mask bits of the slice (bit i = token t0 + i), 0 past the end
    __device__ __forceinline__ float value(int i) const {
        if constexpr (E::kBytes == 2) return (i & 1) ? E::hi(w[i >> 1]) : E::lo(w[i >> 1]);
        else return __uint_as_float(w[i]);
    }
};

// Loads [t0, t0 + n) of a row with independent loads (tokens at or past `end` read as 0 with
// their mask bits cleared).  t0 is a multiple of 32, so the slice lies in one mask word.
template <typename E, int n>
__device__ __forceinline__ void load_slice(const uint8_t* lrow, const int32_t* mrow, int64_t t0, int64_t end,
                                           Slice<E, n>& sl) {
    static_assert(n <= 32 && n % 2 == 0, "slice must fit one mask word");
    uint32_t word = t0 < end ? static_cast<uint32_t>(mrow[t0 >> 5]) >> (t0 & 31) : 0u;
#pragma unroll
    for (int i = 0; i < Slice<E, n>::kWords; ++i) {
        if constexpr (E::kBytes == 2) {
            const uint32_t a = (t0 + 2 * i < end) ? E::raw(lrow, t0 + 2 * i) : 0u;
            const uint32_t b = (t0 + 2 * i + 1 < end) ? E::raw(lrow, t0 + 2 * i + 1) : 0u;
            sl.w[i] = a | (b << 16);
        } else {
            sl.w[i] = (t0 + i < end) ? E::raw(lrow, t0 + i) : 0u;
        }
    }
    const int64_t avail = end - t0;
    if (avail < n) word &= avail <= 0 ? 0u : ((1u << avail) - 1u);
    if constexpr (n < 32) word &= (1u << n) - 1u;
    sl.bits = word;
}

// All-gather of one 32-byte slot per rank across the cluster (finalizer lane 0 issues it;
// the caller syncs the warp before reading).  Rank q's data lands in slots[slot][q] of every CTA.
__device__ __forceinline__ void cluster_allgather(Shared& sh, uint32_t slot, uint32_t crank, uint32_t csize,
                                                  const GatherSlot& mine, uint32_t parity) {
    const uint32_t local = ptx::smem_addr(&sh.slots[slot][crank]);
    const uint32_t bar = ptx::smem_addr(&sh.gather[slot]);
    uint32_t sbits[2];
    memcpy(sbits, &mine.s, 8);
    for (uint32_t q = 0; q < csize; ++q) {
        const uint32_t dst = ptx::mapa(local, q);
        ptx::st_cluster_v4(dst, mine.a, mine.b, mine.c, mine.d);
        ptx::st_cluster_v4(dst + 16, sbits[0], sbits[1], 0u, 0u);
        ptx::mbar_arrive_remote(ptx::mapa(bar, q));
    }
    wait_bounded(ptx::smem_addr(&sh.gather[slot]), parity, &sh.abort, true);
}

// ----------------------------------------------------------------- sampler merge and walk
// One row's per-rank sampler partials merged in rank order -- the same arithmetic whether the
// ranks are CTAs of a cluster or vocabulary shards on different GPUs.
struct SampleMerge {
    int32_t code;
    uint32_t total;
    int owner;      // rank holding the first crossing of u * total (or the last positive rank)
    bool fallback;  // rounding left u * total past the last positive mass
    double M, cutoff, prefix;
    double rank_fac;  // the owner's mass factor exp((owner max - M) / T)
};

// Warp-cooperative (all 32 lanes call it, at most 32 ranks): lane q holds rank q (`in`).  Rank masses are
// rescaled to the row max in parallel (a rank already at the max keeps its mass exactly), then
// located by a warp scan in rank order.
__device__ __forceinline__ SampleMerge merge_sampler_lanes(const GatherSlot& e, bool in, double u, double temp,
                                                           double inv, uint32_t extra_flags, int lane) {
    const float kInf = __int_as_float(0x7F800000);
    SampleMerge r;
    const float a = in ? __uint_as_float(e.a) : -kInf;
    const float rm = ordered_to_float(__reduce_max_sync(0xFFFFFFFFu, ordered_bits(a)));
    const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, in ? e.b : 0u);
    const uint32_t fl = __reduce_or_sync(0xFFFFFFFFu, in ? e.c : 0u) | extra_flags;
    r.total = total;
    r.code = (fl & kFlagAbort) ? kTimeout
             : (fl & kFlagBadMaskRow) ? kBadMaskRow
             : (fl & kFlagNaN) ? kNaN
             : (rm == kInf) ? kPosInf
             : (total == 0u) ? kEmpty
             : (rm == -kInf) ? kNoMass
             : !(u >= 0.0 && u < 1.0) ? kBadUniform
                                      : kOk;
    r.M = rm;
    r.owner = -1;
    r.fallback = false;
    r.cutoff = 0.0;
    r.prefix = 0.0;
    r.rank_fac = 1.0;
    if (r.code != kOk) return r;
    const bool pos_in = in && e.s > 0.0;
    const double f = pos_in ? (a == rm ? 1.0 : scaled_exp(static_cast<double>(a) - static_cast<double>(rm), temp, inv))
                            : 0.0;
    const double m = pos_in ? e.s * f : 0.0;
    const double incl = warp_inclusive_scan(m, lane);
    const double up = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    const double before = lane > 0 ? up : 0.0;
    r.cutoff = u * __shfl_sync(0xFFFFFFFFu, incl, 31);
    const uint32_t positive = __ballot_sync(0xFFFFFFFFu, m > 0.0);
    const uint32_t hits = __ballot_sync(0xFFFFFFFFu, m > 0.0 && r.cutoff < incl);
    int owner;
    if (hits) {
        owner = __ffs(hits) - 1;
    } else {
        r.fallback = true;
        owner = positive ? 31 - __clz(positive) : -1;
    }
    r.owner = owner;
    const double pre = __shfl_sync(0xFFFFFFFFu, before, owner < 0 ? 0 : owner);
    const double rf = __shfl_sync(0xFFFFFFFFu, f, owner < 0 ? 0 : owner);
    if (owner >= 0) {
        r.prefix = pre;
        r.rank_fac = rf;
    }
    return r;
}

__device__ __forceinline__ SampleMerge merge_sampler_ranks(const GatherSlot* g, int64_t stride, uint32_t n, double u,
                                                           double temp, double inv, uint32_t extra_flags, int lane) {
    if (n == 1) {
        // One rank: its max is the row max and its mass the total (the scan of merge_sampler_lanes
        // over one lane, without the warp round trips).
        const float kInf = __int_as_float(0x7F800000);
        const GatherSlot e = g[0];
        const float rm = __uint_as_float(e.a);
        const uint32_t fl = e.c | extra_flags;
        SampleMerge r;
        r.total = e.b;
        r.code = (fl & kFlagAbort) ? kTimeout
                 : (fl & kFlagBadMaskRow) ? kBadMaskRow
                 : (fl & kFlagNaN) ? kNaN
                 : (rm == kInf) ? kPosInf
                 : (e.b == 0u) ? kEmpty
                 : (rm == -kInf) ? kNoMass
                 : !(u >= 0.0 && u < 1.0) ? kBadUniform
                                          : kOk;
        r.M = rm;
        r.owner = -1;
        r.fallback = false;
        r.cutoff = 0.0;
        r.prefix = 0.0;
        r.rank_fac = 1.0;
        if (r.code != kOk) return r;
        const double m = e.s > 0.0 ? e.s : 0.0;
        r.cutoff = u * m;
        if (m > 0.0) {
            r.owner = 0;
            r.fallback = !(r.cutoff < m);
        } else {
            r.fallback = true;
        }
        return r;
    }
    const bool in = static_cast<uint32_t>(lane) < n;
    GatherSlot e{0u, 0u, 0u, 0u, 0.0, 0.0};
    if (in) e = g[static_cast<int64_t>(lane) * stride];
    return merge_sampler_lanes(e, in, u, temp, inv, extra_flags, lane);
}

// Factor taking a warp's mass from its reference max to its rank's max (1 when equal).
__device__ __forceinline__ double warp_factor(float wmax, float seg_m, double temp, double inv) {
    return wmax == seg_m ? 1.0 : scaled_exp(static_cast<double>(wmax) - static_cast<double>(seg_m), temp, inv);
}

template <typename T>
__device__ int64_t walk_granule(int gsel, double gprefix, bool walk_fallback, double M, double cutoff, double temp,
                                double inv, float scale2, int64_t seg_begin, int64_t seg_end, const uint8_t* lrow,
                                const int32_t* mrow, float (*walk)[33], int lane);

// The owning rank's walk (one warp): find the granule holding the crossing from the granule
// masses (each relative to its warp's reference max; `fac` = warp factor x rank factor rescales
// them to the row max), then the lane of that granule with fp32 weights, then the token with the
// reference's exact fp64 weights.  Granule g (chunk g / 8, warp g % 8, in token order) is read at
// granules[(g / 8) * cstride + (g % 8) * wstride]: the shared-memory table is warp-major (cstride
// 1, wstride kMaxChunksSampler), a vocabulary shard's record chunk-major (cstride 8, wstride 1).
// Lane w < 8 passes its warp's factor to the rank max (warp_factor) and mass.  Returns the token's
// index within the row (-1 if none).
template <typename T>
__device__ int64_t sampler_owner_walk(const double* granules, int cstride, int wstride, int ngran, double wfac,
                                      double wmass, bool has_warp,
                                      const SampleMerge& mg, double temp, double inv, float scale2, int64_t seg_begin,
                                      int64_t seg_end, const uint8_t* lrow, const int32_t* mrow, float (*walk)[33],
                                      double* fac, int lane) {
    const double M = mg.M, cutoff = mg.cutoff, prefix = mg.prefix;
    const bool fallback = mg.fallback;
    if (has_warp) fac[lane] = wmass > 0.0 ? wfac * mg.rank_fac : 0.0;
    __syncwarp();
    const int per = (ngran + 31) / 32;
    const int g0 = lane * per, g1 = min(g0 + per, ngran);
    double local = 0.0;
    auto mass_at = [&](int g) {
        const int w = g % kConsumerWarps;
        return granules[(g / kConsumerWarps) * cstride + w * wstride] * fac[w];
    };
    for (int g = g0; g < g1; ++g) local += mass_at(g);
    const double incl = warp_inclusive_scan(local, lane);
    double acc = prefix + incl - local;
    int cand = 0x7FFFFFFF, lastg = -1;
    double cand_prefix = 0.0;
    for (int g = g0; g < g1; ++g) {
        const double m = mass_at(g);
        if (!(m > 0.0)) continue;
        lastg = g;
        if (!fallback && cand == 0x7FFFFFFF && cutoff < acc + m) {
            cand = g;
            cand_prefix = acc;
        }
        acc += m;
    }
    int gsel = __reduce_min_sync(0xFFFFFFFFu, cand);
    const bool walk_fallback = gsel == 0x7FFFFFFF;
    double gprefix = 0.0;
    if (walk_fallback) {
        gsel = __reduce_max_sync(0xFFFFFFFFu, lastg);
    } else {
        const uint32_t owner_lane = __ffs(__ballot_sync(0xFFFFFFFFu, cand == gsel)) - 1;
        gprefix = __shfl_sync(0xFFFFFFFFu, cand_prefix, owner_lane);
    }
    if (gsel < 0) return -1;
    return walk_granule<T>(gsel, gprefix, walk_fallback, M, cutoff, temp, inv, scale2, seg_begin, seg_end, lrow, mrow,
                           walk, lane);
}

// The walk of one granule (one warp): granule `gsel` (chunk gsel / 8, warp gsel % 8 of the segment
// starting at token seg_begin) holds the crossing of `cutoff`, the masses before it summing to
// `gprefix` (relative to M); `fallback` asks for its last positive weight instead.  The lane of the
// crossing is found with fp32 weights (fp64 when every fp32 weight underflows), the token with the
// reference's exact fp64 weights.  Returns the token's index within the row (-1 if none).
template <typename T>
__device__ int64_t walk_granule(int gsel, double gprefix, bool walk_fallback, double M, double cutoff, double temp,
                                double inv, float scale2, int64_t seg_begin, int64_t seg_end, const uint8_t* lrow,
                                const int32_t* mrow, float (*walk)[33], int lane) {
    using E = Elem<T>;
    constexpr int kTPC = Layout<T>::kTokensPerChunk;
    constexpr int kTPW = Layout<T>::kTokensPerWarp;
    constexpr int kFinPer = kTPW / 32;
    const int gc = gsel / kConsumerWarps, gw = gsel % kConsumerWarps;
    const int64_t gt0 = seg_begin + static_cast<int64_t>(gc) * kTPC + gw * kTPW;
    const int64_t gt1 = min(gt0 + kTPW, seg_end);
    const int64_t my0 = gt0 + lane * kFinPer;
    uint32_t bits;
    {
        Slice<E, kFinPer> sl;
        load_slice<E, kFinPer>(lrow, mrow, my0, gt1, sl);
#pragma unroll
        for (int i = 0; i < kFinPer; ++i) walk[lane][i] = sl.value(i);
        bits = sl.bits;
    }
    __syncwarp();
    // (1) fp32 weights relative to M locate the lane whose tokens hold the crossing (its fp32
    // prefix is within ~1e-7 of the exact one).
    float lsum = 0.0f;
    {
        const float hm = -0.5f * static_cast<float>(M);
#pragma unroll
        for (int i = 0; i < kFinPer; ++i) {
            const float t = fminf(fmaf(walk[lane][i], 0.5f, hm) * scale2, kWalkClamp);
            const float w = ptx::ex2(t);
            lsum += ((bits >> i) & 1u) ? w : 0.0f;
        }
    }
    double lsum_d = lsum;
    // Every fp32 weight of the granule underflowed (tiny temperatures: its mass comes from weights
    // below 2^-149 relative to M): the lane is located with the exact fp64 weights instead.
    if (__ballot_sync(0xFFFFFFFFu, lsum > 0.0f) == 0u) {
        lsum_d = 0.0;
#pragma unroll 1
        for (int i = 0; i < kFinPer; ++i)
            if ((bits >> i) & 1u) lsum_d += exact_weight(walk[lane][i], M, temp, inv);
    }
    const double lincl = warp_inclusive_scan(lsum_d, lane);
    const bool positive = lsum_d > 0.0;
    const uint32_t pos_mask = __ballot_sync(0xFFFFFFFFu, positive);
    const uint32_t cross_mask = __ballot_sync(0xFFFFFFFFu, !walk_fallback && positive && cutoff < gprefix + lincl);
    const bool lane_fallback = cross_mask == 0u;
    const int L = lane_fallback ? (pos_mask ? 31 - __clz(pos_mask) : -1) : __ffs(cross_mask) - 1;
    if (L < 0) return -1;
    // (2) exact fp64 weights of lane L's tokens, one per lane, scanned in token order.
    const uint32_t bitsL = __shfl_sync(0xFFFFFFFFu, bits, L);
    const double prefixL = gprefix + __shfl_sync(0xFFFFFFFFu, lincl - lsum_d, L);
    const bool mine = lane < kFinPer && ((bitsL >> lane) & 1u);
    const double w = mine ? exact_weight(walk[L][lane < kFinPer ? lane : 0], M, temp, inv) : 0.0;
    const double winc = warp_inclusive_scan(w, lane);
    const uint32_t hits = __ballot_sync(0xFFFFFFFFu, !lane_fallback && w > 0.0 && cutoff < prefixL + winc);
    const uint32_t pos = __ballot_sync(0xFFFFFFFFu, w > 0.0);
    const int64_t base = gt0 + static_cast<int64_t>(L) * kFinPer;
    if (hits) return base + (__ffs(hits) - 1);
    if (pos) return base + (31 - __clz(pos));  // rounding: the last positive weight
    return -1;
}

// Byte layout of a sampler partial's granule record (vocabulary shards).
struct SamplerRecord {
    static constexpr int64_t kWarpMaxOffset = 0;                           // float[8]
    static constexpr int64_t kWarpMassOffset = 32;                         // double[8]
    static constexpr int64_t kGranuleOffset = 96;                          // double[chunks * 8]
    static constexpr int64_t bytes(int chunks) { return kGranuleOffset + 8ll * chunks * kConsumerWarps; }
};

// ----------------------------------------------------------------- workspace access
__device__ __forceinline__ WsHeader* ws_header(const SelectParams& p) { return reinterpret_cast<WsHeader*>(p.ws); }
__device__ __forceinline__ unsigned long long* ws_row_counter(const SelectParams& p, int64_t t) {
    return reinterpret_cast<unsigned long long*>(p.ws + ws_counters_offset()) + t;
}
__device__ __forceinline__ WsPiece* ws_piece(const SelectParams& p, int64_t t, int c) {
    return reinterpret_cast<WsPiece*>(p.ws + ws_pieces_offset(p.ws_rows)) + (t * kWsChunks + c);
}
// Split row t's granule block, [warp][chunk] with kWsChunks chunks per warp.
__device__ __forceinline__ double* ws_granules(const SelectParams& p, int64_t t) {
    return reinterpret_cast<double*>(p.ws + ws_granules_offset(p.ws_rows)) + t * kWsChunks * kConsumerWarps;
}
// Flat schedule: row t's granule records, [chunk][warp].
__device__ __forceinline__ uint4* ws_flat_records(const SelectParams& p, int64_t t) {
    return reinterpret_cast<uint4*>(p.ws + ws_flat_offset(p.ws_rows)) + t * kWsChunks * kConsumerWarps;
}

// ----------------------------------------------------------------- the kernel
// Merge of one split row (one warp): the row's pieces of this launch (epoch), read from the
// workspace and merged in chunk order -- the same merge as cluster ranks and vocabulary shards --
// then the row's outputs: the argmax index is recovered from the winning region only, the sampler
// walks the owning piece.  `granules` is a shared-memory table [warp][kMaxChunksSampler] that the
// row's granules are copied into (sampler); `piece_c0` / `piece_part` hold up to 32 pieces.  A
// row without pieces of this launch (handed out whole) is left alone.  `reset` returns the row's
// chunk counter to zero for the next launch (in-kernel merges only).
template <typename T, bool kSample>
__device__ void merge_split_row(const SelectParams& p, int64_t row, int64_t t, int row_chunks, double* granules,
                                double uniform, uint32_t abort_flag, int32_t* piece_c0, GatherSlot* piece_part,
                                float (*walk)[33], double* fac, const uint8_t* lrow, const int32_t* mrow, int lane,
                                bool reset) {
    using E = Elem<T>;
    constexpr int kTPC = Layout<T>::kTokensPerChunk;
    constexpr int kTPW = Layout<T>::kTokensPerWarp;
    constexpr int kFinPer = kTPW / 32;
    __syncwarp();  // every lane is done with the scratch of the warp's previous row
    // One round trip: the sampler's row granules stream into shared memory (no registers) while
    // the piece records at chunks c = lane and lane + 32 load; records of this launch (epoch) are
    // compacted in chunk order (at most 32 pieces: rows of <= 64 chunks in blocks of >= 4 chunks,
    // split at most once more at a row boundary).
    if constexpr (kSample) {
        // Both tables are [warp][64 chunks]: each warp's row_chunks doubles in 16-byte copies (an
        // odd count copies one unused double past them).
        static_assert(kWsChunks == kMaxChunksSampler, "workspace and shared granule rows match");
        const uint8_t* src = reinterpret_cast<const uint8_t*>(ws_granules(p, t));
        const uint32_t dst = ptx::smem_addr(granules);
        const int pairs = (row_chunks + 1) / 2;
        for (int i = lane; i < pairs * kConsumerWarps; i += 32) {
            const int w = i / pairs, k = i - w * pairs;
            const int off = (w * kMaxChunksSampler + 2 * k) * 8;
            ptx::cp_async_16(dst + off, src + off);
        }
    }
    auto head = [&](int c, uint32_t& epoch, GatherSlot& g) {
        const uint4* src = reinterpret_cast<const uint4*>(ws_piece(p, t, c));
        const uint4 h = __ldcg(src), x = __ldcg(src + 1), y = __ldcg(src + 2);
        epoch = h.x;
        memcpy(&g, &x, 16);
        memcpy(reinterpret_cast<uint8_t*>(&g) + 16, &y, 16);
    };
    uint32_t ea = 0, eb = 0;
    GatherSlot ga{0u, 0u, 0u, 0u, 0.0, 0.0}, gb{0u, 0u, 0u, 0u, 0.0, 0.0};
    if (lane < row_chunks) head(lane, ea, ga);
    if (lane + 32 < row_chunks) head(lane + 32, eb, gb);
    const bool va = lane < row_chunks && ea == p.epoch;
    const bool vb = lane + 32 < row_chunks && eb == p.epoch;
    const uint32_t ba = __ballot_sync(0xFFFFFFFFu, va), bb = __ballot_sync(0xFFFFFFFFu, vb);
    const uint32_t below = (1u << lane) - 1u;
    const int na = __popc(ba);
    if (va) {
        piece_c0[__popc(ba & below)] = lane;
        piece_part[__popc(ba & below)] = ga;
    }
    if (vb && na + __popc(bb & below) < 32) {
        piece_c0[na + __popc(bb & below)] = lane + 32;
        piece_part[na + __popc(bb & below)] = gb;
    }
    const int npieces = min(na + __popc(bb), 32);
    if constexpr (kSample) ptx::cp_async_wait_all();
    if (npieces == 0) return;  // handed out whole: the selection launch wrote the row
    __syncwarp();
    const bool in = lane < npieces;
    const GatherSlot e = in ? piece_part[lane] : GatherSlot{0u, 0u, 0u, 0u, 0.0, 0.0};
    if constexpr (!kSample) {
        const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, e.a);
        const uint32_t region = __reduce_min_sync(0xFFFFFFFFu, (in && hi != 0u && e.a == hi) ? e.b : 0xFFFFFFFFu);
        const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, in ? e.c : 0u);
        const uint32_t fl = __reduce_or_sync(0xFFFFFFFFu, in ? e.d : 0u) | abort_flag;
        // The first (chunk, warp) region holding the row maximum; its lowest valid token equal to
        // the maximum is the row's argmax.
        uint32_t found = 0xFFFFFFFFu;
        if (region != 0xFFFFFFFFu) {
            const float target = ordered_to_float(hi);
            const int64_t r0 = static_cast<int64_t>(region / kConsumerWarps) * kTPC +
                               static_cast<int64_t>(region % kConsumerWarps) * kTPW;
            const int64_t my0 = r0 + lane * kFinPer;
            Slice<E, kFinPer> sl;
            load_slice<E, kFinPer>(lrow, mrow, my0, p.vocab, sl);
#pragma unroll
            for (int i = kFinPer - 1; i >= 0; --i)
                if (((sl.bits >> i) & 1u) && sl.value(i) == target) found = static_cast<uint32_t>(my0 + i);
        }
        found = __reduce_min_sync(0xFFFFFFFFu, found);
        if (lane == 0) {
            const int32_t code = argmax_status(fl, total);
            p.status[row] = code;
            p.tokens[row] = (code == kOk && found != 0xFFFFFFFFu) ? p.token_offset + static_cast<int64_t>(found) : -1;
            if (p.counts) p.counts[row] = total;
        }
    } else {
        const SampleMerge mg = merge_sampler_lanes(e, in, uniform, p.temperature, p.inv_temperature, abort_flag, lane);
        int64_t chosen = -1;
        if (mg.code == kOk) {
            const int q = mg.owner;
            const int oc0 = piece_c0[q];
            const int oc1 = q + 1 < npieces ? piece_c0[q + 1] : row_chunks;
            // The owner's granules are already relative to its max: every warp factor is the
            // owner's rank factor.
            const int64_t b0 = static_cast<int64_t>(oc0) * kTPC;
            const int64_t b1 = static_cast<int64_t>(oc1) * kTPC < p.vocab ? static_cast<int64_t>(oc1) * kTPC : p.vocab;
            chosen = sampler_owner_walk<T>(granules + oc0, 1, kMaxChunksSampler, (oc1 - oc0) * kConsumerWarps, 1.0, 1.0,
                                           lane < kConsumerWarps, mg, p.temperature, p.inv_temperature, p.scale2, b0, b1,
                                           lrow, mrow, walk, fac, lane);
        }
        if (lane == 0) {
            p.status[row] = mg.code != kOk ? mg.code : chosen >= 0 ? kOk : kNoMass;
            p.tokens[row] = mg.code == kOk && chosen >= 0 ? p.token_offset + chosen : -1;
            if (p.counts) p.counts[row] = mg.total;
        }
    }
    // The next launch (or graph replay) counts this row from zero.
    if (reset && lane == 0) atomicExch(ws_row_counter(p, t), 0ull);
}

// Finalizer (one warp) of a split unit: the piece's partial (argmax: key, first region holding
// it, count, flags; sampler: max, count, flags, mass) and, for the sampler, its granules scaled
// to the piece's max go to the workspace; the CTA whose piece completes the row's chunk count
// merges the row (merge_split_row).  Sampler: `granules` (shared memory) holds the piece's granules, lanes
// w < 8 pass warp w's factor to the piece max; the buffer is then reused for the row's granules;
// `uniform` is the row's uniform.
template <typename T, bool kSample>
__device__ void finish_split_piece(const SelectParams& p, const Unit& d, int row_chunks, const GatherSlot& part, double wf,
                                   double* granules, double uniform, Shared& sh, SamplerShared& ss, const uint8_t* lrow,
                                   const int32_t* mrow, int lane) {
    const int64_t t = d.row - p.whole_rows;
    const int nch = d.c1 - d.c0;
    WsPiece* pc = ws_piece(p, t, d.c0);
    if (lane == 0) {
        pc->epoch = p.epoch;
        pc->c1 = d.c1;
        pc->part = part;
    }
    if constexpr (kSample) {
        if (lane < kConsumerWarps) ss.fac[lane] = wf;
        __syncwarp();
        double* g = ws_granules(p, t) + d.c0;
        for (int i = lane; i < nch * kConsumerWarps; i += 32) {
            const int w = i / nch, c = i - w * nch;
            g[w * kWsChunks + c] = granules[w * kMaxChunksSampler + c] * ss.fac[w];
        }
    }
    // Publish the piece and count its chunks in with one acquire-release add: the add that
    // reaches the row's total identifies the merging CTA, which then sees every piece.
    __syncwarp();
    unsigned long long before = 0;
    if (lane == 0) before = ptx::atom_add_acq_rel_gpu(ws_row_counter(p, t), static_cast<uint64_t>(nch));
    before = __shfl_sync(0xFFFFFFFFu, before, 0);
    if (before + static_cast<unsigned long long>(nch) != static_cast<unsigned long long>(row_chunks)) return;
    __syncwarp();

    merge_split_row<T, kSample>(p, d.row, t, row_chunks, granules, uniform, sh.abort ? kFlagAbort : 0u, sh.piece_c0,
                                sh.piece_part, ss.walk, ss.fac, lrow, mrow, lane, true);
}

// Programmatic dependent launch: a dependent grid (the next selection launch, the verification
// epilogue) may be scheduled once every thread of every CTA executed this or exited.  The
// finalizer warp executes it on entry and the producer and consumer warps when they have
// streamed their last chunk, so the dependent's launch overlaps the row-end work of the last
// rows; the dependent still waits for this grid's completion before touching memory.
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename T, bool kSample, bool kBulk, int kStages, bool kFlat = false>
__global__ void __launch_bounds__(kThreads, 3) select_rows_kernel(const SelectParams p) {
    static_assert(!kFlat || (kSample && kBulk), "the flat schedule is a sampler schedule of bulk-copied rows");
    using E = Elem<T>;
    using L = Layout<T>;
    constexpr int kVec = E::kVec;
    constexpr int kTPC = L::kTokensPerChunk;
    constexpr int kTPW = L::kTokensPerWarp;
    constexpr uint32_t kVecMask = (1u << kVec) - 1u;
    constexpr int kFinPer = kTPW / 32;
    const float kInf = __int_as_float(0x7F800000);

    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* stages = smem_raw;
    Shared& sh = *reinterpret_cast<Shared*>(smem_raw + kStages * L::kStageBytes);
    SamplerShared& ss = *reinterpret_cast<SamplerShared*>(reinterpret_cast<uint8_t*>(&sh) + sizeof(Shared));

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t crank = ptx::cluster_ctarank();
    const uint32_t csize = ptx::cluster_nctarank();
    const uint32_t cid = ptx::cluster_id_x();
    const uint32_t nclusters = ptx::ncluster_x();
    const bool dynamic = p.ws != nullptr;  // tickets from the workspace (one-CTA clusters only)
    constexpr bool flat = kFlat;  // granule records to the workspace (dynamic schedule, sampler)

    // Fixed schedule: a contiguous, remainder-balanced block of rows per cluster (neighbouring
    // rows, often of different mask densities, hence cost, land on the same cluster).
    const int64_t rows_q = p.rows / nclusters, rows_r = p.rows % nclusters;
    const int64_t row_begin = static_cast<int64_t>(cid) * rows_q + (cid < rows_r ? cid : rows_r);
    const int64_t row_end = row_begin + rows_q + (cid < rows_r ? 1 : 0);
    const int64_t seg_begin_raw = static_cast<int64_t>(crank) * p.segment;
    const int64_t seg_begin = seg_begin_raw < p.vocab ? seg_begin_raw : p.vocab;
    const int64_t seg_end = (seg_begin_raw + p.segment) < p.vocab ? (seg_begin_raw + p.segment) : p.vocab;
    const int nchunks = static_cast<int>((seg_end - seg_begin + kTPC - 1) / kTPC);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            ptx::mbar_init(ptx::smem_addr(&sh.full[s]), 1);
            ptx::mbar_init(ptx::smem_addr(&sh.empty[s]), kConsumerWarps);
        }
        for (int s = 0; s < 2; ++s) {
            ptx::mbar_init(ptx::smem_addr(&sh.part_full[s]), kConsumerWarps);
            ptx::mbar_init(ptx::smem_addr(&sh.part_empty[s]), 1);
            ptx::mbar_init(ptx::smem_addr(&sh.gather[s]), csize);
        }
        for (int s = 0; s < kUnitSlots; ++s) {
            ptx::mbar_init(ptx::smem_addr(&sh.unit_full[s]), 1);
            ptx::mbar_init(ptx::smem_addr(&sh.unit_empty[s]), kConsumerWarps);
        }
        for (int w = 0; w < kConsumerWarps; ++w) sh.flat_dst[w] = nullptr;
        sh.abort = 0;
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    // Launched as a programmatic dependent, this grid may have started while the previous grid in
    // the stream was still running: no global memory is touched before that grid completed.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Peer-memory exchange: slot xepoch & 1 is free in every area once every rank merged step
    // xepoch - 2.  A CTA that gives up stores nothing to its peers (its rows report status 7).
    if (p.xranks > 0) {
        if (tid == 0) {
            const ExchangeHeader* own = reinterpret_cast<const ExchangeHeader*>(p.xarea[p.xrank]);
            if (!wait_flags_at_least(own->consumed, p.xranks, p.xepoch - 2u)) sh.abort = 1;
        }
        __syncthreads();
    }
    // Every CTA of the cluster has initialised its barriers before any remote arrive.
    if (csize > 1) {
        ptx::cluster_arrive();
        ptx::cluster_wait();
    }

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer warp
        // Lane 0 publishes each unit's descriptor, then (bulk path) streams its chunks.
        if (lane == 0) {
            uint32_t it = 0;  // chunks issued (stage ring position)
            uint32_t u = 0;   // units published (descriptor ring position)
            bool stop = false;
            auto push = [&](const Unit& d) -> bool {
                const uint32_t s = u % kUnitSlots, use = u / kUnitSlots;
                if (use > 0 && !wait_bounded(ptx::smem_addr(&sh.unit_empty[s]), (use - 1u) & 1u, &sh.abort)) return false;
                sh.units[s] = d;
                ptx::mbar_arrive(ptx::smem_addr(&sh.unit_full[s]));
                ++u;
                return true;
            };
            auto issue = [&](const Unit& d) -> bool {
                if constexpr (kBulk) {
                    const uint8_t* lrow = static_cast<const uint8_t*>(p.logits) +
                                          static_cast<size_t>(d.row) * static_cast<size_t>(p.logit_stride) * E::kBytes;
                    const int32_t* mbase = p.masks + static_cast<size_t>(d.mask_row) * static_cast<size_t>(p.mask_stride);
                    for (int c = d.c0; c < d.c1; ++c, ++it) {
                        const int stage = static_cast<int>(it % kStages);
                        const uint32_t use = it / kStages;
                        // Consumers stopped releasing stages: issue no more copies.
                        if (use > 0 && !wait_bounded(ptx::smem_addr(&sh.empty[stage]), (use - 1) & 1u, &sh.abort))
                            return false;
                        const int64_t t0 = seg_begin + static_cast<int64_t>(c) * kTPC;
                        const int64_t t1 = (t0 + kTPC) < seg_end ? (t0 + kTPC) : seg_end;
                        const uint32_t lbytes = static_cast<uint32_t>((t1 - t0) * E::kBytes);
                        const int64_t w0 = p.mask_word_offset + (t0 >> 5), w1 = p.mask_word_offset + ((t1 + 31) >> 5);
                        const int64_t a0 = w0 & ~int64_t(3), a1 = (w1 + 3) & ~int64_t(3);
                        const uint32_t mbytes = static_cast<uint32_t>((a1 - a0) * 4);
                        uint8_t* st = stages + stage * L::kStageBytes;
                        const uint32_t full = ptx::smem_addr(&sh.full[stage]);
                        ptx::mbar_arrive_expect_tx(full, lbytes + mbytes);
                        ptx::bulk_load(ptx::smem_addr(st), lrow + t0 * E::kBytes, lbytes, full);
                        ptx::bulk_load(ptx::smem_addr(st + kChunkBytes), mbase + a0, mbytes, full);
                    }
                }
                return true;
            };
            auto run = [&](int64_t row, int c0, int c1, int32_t kind) {
                if (stop) return;
                int64_t mr = row;
                int32_t bad = 0;
                if (p.mask_rows != nullptr) {
                    mr = p.mask_rows[row];
                    bad = (mr < 0 || mr >= p.mask_table_rows) ? 1 : 0;
                    if (bad) mr = 0;
                }
                const Unit d{row, c0, c1, kind, bad, mr};
                stop = !push(d) || !issue(d);
            };
            if (!dynamic) {
                for (int64_t row = row_begin; row < row_end && !stop; ++row) run(row, 0, nchunks, kUnitWhole);
            } else {
                // Tickets: rows [0, whole_rows) whole, then blocks over the remaining (split)
                // rows' chunks in row-major order, shrinking by tier (tier_tickets / tier_block,
                // then `block`).
                const int64_t split_chunks = (p.rows - p.whole_rows) * nchunks;
                unsigned long long* tickets = &ws_header(p)->tickets;
                for (bool first = true; !stop; first = false) {
                    // CTA b's first ticket is b; later ones come from the counter (one atomic per
                    // ticket, the counter starting every launch at 0).
                    // The flat schedule takes every ticket from the counter, so that a CTA starting
                    // late holds no block of its own.
                    const int64_t tk = flat    ? static_cast<int64_t>(atomicAdd(tickets, 1ull))
                                       : first ? static_cast<int64_t>(blockIdx.x)
                                               : static_cast<int64_t>(gridDim.x) + static_cast<int64_t>(atomicAdd(tickets, 1ull));
                    if (tk >= p.tickets) break;
                    if (tk < p.whole_rows) {
                        run(tk, 0, nchunks, kUnitWhole);
                        continue;
                    }
                    const int64_t sk = tk - p.whole_rows;
                    const int64_t n0 = p.tier_tickets[0], n1 = p.tier_tickets[1];
                    const int64_t b0 = p.tier_block[0], b1 = p.tier_block[1];
                    const int64_t g0 = sk < n0        ? sk * b0
                                       : sk < n0 + n1 ? n0 * b0 + (sk - n0) * b1
                                                      : n0 * b0 + n1 * b1 + (sk - n0 - n1) * p.block;
                    const int64_t len = sk < n0 ? b0 : sk < n0 + n1 ? b1 : p.block;
                    const int64_t g1 = (g0 + len) < split_chunks ? (g0 + len) : split_chunks;
                    for (int64_t r = g0 / nchunks; r <= (g1 - 1) / nchunks; ++r) {
                        const int c0 = static_cast<int>(g0 > r * nchunks ? g0 - r * nchunks : 0);
                        const int c1 = static_cast<int>(g1 < (r + 1) * nchunks ? g1 - r * nchunks : nchunks);
                        run(p.whole_rows + r, c0, c1, (c0 == 0 && c1 == nchunks) ? kUnitWhole : kUnitSplit);
                    }
                }
            }
            // The end marker (if its slot never frees, the consumers' bounded waits end them).
            push(Unit{0, 0, 0, kUnitEnd, 0, 0});
            // Every issued copy must have landed before this CTA's shared memory can go away.
            if constexpr (kBulk) {
                for (int s = 0; s < kStages; ++s) {
                    if (it > static_cast<uint32_t>(s)) {
                        const uint32_t last = (it - 1u - static_cast<uint32_t>(s)) / kStages;
                        drain_wait(ptx::smem_addr(&sh.full[s]), last & 1u);
                    }
                }
            }
        }
        __syncwarp();
        launch_dependents();
    } else if (warp == kFinalizerWarp) {
        // ------------------------------------------------------------ finalizer warp
        launch_dependents();
        if constexpr (kFlat) {
            // Flat schedule: the rows are merged by the merge launch that follows this one.
        } else {
            for (uint32_t k = 0;; ++k) {
                const uint32_t slot = k & 1u;
                if (!wait_bounded(ptx::smem_addr(&sh.part_full[slot]), (k >> 1) & 1u, &sh.abort)) break;
                const Unit d = sh.part_unit[slot];
                if (d.kind == kUnitEnd) break;
                const int64_t row = d.row;
                const uint8_t* lrow = static_cast<const uint8_t*>(p.logits) +
                                      static_cast<size_t>(row) * static_cast<size_t>(p.logit_stride) * E::kBytes;
                const int32_t* mrow =
                    p.masks + static_cast<size_t>(d.mask_row) * static_cast<size_t>(p.mask_stride) + p.mask_word_offset;
                const int nch = d.c1 - d.c0;
                const bool in = lane < kConsumerWarps;
                const WarpPartial wp = in ? sh.part[slot][lane] : WarpPartial{0u, 0xFFFFFFFFu, 0u, 0u, 0.0, 0.0};
                const uint32_t cnt = __reduce_add_sync(0xFFFFFFFFu, wp.count);
                const uint32_t flags = __reduce_or_sync(0xFFFFFFFFu, wp.flags) | (sh.abort ? kFlagAbort : 0u) |
                                       (d.mask_bad ? kFlagBadMaskRow : 0u);
                const uint32_t ckey = __reduce_max_sync(0xFFFFFFFFu, wp.key);

                if constexpr (!kSample) {
                    // First (chunk, warp) region holding the segment maximum; its lowest valid token
                    // equal to the maximum is the segment's argmax.
                    const uint32_t region = (in && ckey != 0u && wp.key == ckey) ? (wp.chunk * kConsumerWarps + lane)
                                                                                  : 0xFFFFFFFFu;
                    const uint32_t rmin = __reduce_min_sync(0xFFFFFFFFu, region);
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(ptx::smem_addr(&sh.part_empty[slot]));
                    if (d.kind == kUnitSplit && p.partials == nullptr) {
                        // The index is recovered by the row's merge, from the winning piece only.
                        finish_split_piece<T, false>(p, d, nchunks, GatherSlot{ckey, rmin, cnt, flags, 0.0, 0.0}, 0.0,
                                                     nullptr, 0.0, sh, ss, lrow, mrow, lane);
                        continue;
                    }
                    uint32_t found = 0xFFFFFFFFu;
                    if (rmin != 0xFFFFFFFFu) {
                        const float target = ordered_to_float(ckey);
                        const int64_t r0 = seg_begin + static_cast<int64_t>(rmin / kConsumerWarps) * kTPC +
                                           static_cast<int64_t>(rmin % kConsumerWarps) * kTPW;
                        const int64_t my0 = r0 + lane * kFinPer;
                        Slice<E, kFinPer> sl;
                        load_slice<E, kFinPer>(lrow, mrow, my0, seg_end, sl);
    #pragma unroll
                        for (int i = kFinPer - 1; i >= 0; --i)
                            if (((sl.bits >> i) & 1u) && sl.value(i) == target) found = static_cast<uint32_t>(my0 + i);
                    }
                    uint32_t hi = ckey;
                    uint32_t lo = __reduce_min_sync(0xFFFFFFFFu, found);
                    lo = lo == 0xFFFFFFFFu ? 0u : 0xFFFFFFFFu - static_cast<uint32_t>(p.token_offset + lo);
                    uint32_t total = cnt, fl = flags;
                    if (p.partials != nullptr) {  // vocabulary shard: the row's partial is the output
                        GatherSlot rec{hi, lo, total, fl, 0.0, 0.0};
                        // An exchange step tags each partial with its epoch, so that a merge finding
                        // another tag in a rank's slot (that rank's step had fewer rows) fails the row
                        // instead of merging a partial left there by an earlier step.
                        if (p.xranks > 0) rec.pad = __longlong_as_double(static_cast<long long>(p.xepoch));
                        if (lane == 0) p.partials[row] = rec;
                        // Peer-memory exchange: the same record in every other rank's area (NVLink
                        // stores overlapping the streaming of the next rows).
                        if (lane < p.xranks && lane != p.xrank && !sh.abort) p.xpeer[lane][row] = rec;
                        continue;
                    }
                    if (csize > 1) {
                        if (lane == 0)
                            cluster_allgather(sh, slot, crank, csize, GatherSlot{hi, lo, total, fl, 0.0, 0.0}, (k >> 1) & 1u);
                        __syncwarp();
                        const bool inr = lane < static_cast<int>(csize);
                        const GatherSlot g = inr ? sh.slots[slot][lane] : GatherSlot{0u, 0u, 0u, 0u, 0.0, 0.0};
                        hi = __reduce_max_sync(0xFFFFFFFFu, g.a);
                        lo = __reduce_max_sync(0xFFFFFFFFu, (inr && g.a == hi) ? g.b : 0u);
                        total = __reduce_add_sync(0xFFFFFFFFu, g.c);
                        fl = __reduce_or_sync(0xFFFFFFFFu, g.d) | (sh.abort ? kFlagAbort : 0u);
                    }
                    if (crank == 0 && lane == 0) {
                        const int32_t code = argmax_status(fl, total);
                        p.status[row] = code;
                        p.tokens[row] = code == kOk ? static_cast<int64_t>(0xFFFFFFFFu - lo) : -1;
                        if (p.counts) p.counts[row] = total;
                    }
                } else {
                    // Segment maximum and mass relative to it: the consumer warps already folded their
                    // granules to their own maxima; combine the 8 warp masses in warp order.
                    double* granules = ss.granules[slot];
                    const int ngran = nch * kConsumerWarps;
                    const float seg_m = ckey ? ordered_to_float(ckey) : -kInf;
                    const bool seg_finite = seg_m > -kInf && seg_m < kInf;
                    const float wmax = in ? ordered_to_float(wp.key) : -kInf;
                    const double wf = (seg_finite && in && wp.mass > 0.0)
                                          ? warp_factor(wmax, seg_m, p.temperature, p.inv_temperature)
                                          : 0.0;
                    const double term = wp.mass * wf;
                    const double seg_s = warp_sum8(term);  // read on lane 0
                    if (p.partials != nullptr) {
                        // Vocabulary shard: the row's partial and granule record are the output.
                        if (lane == 0) p.partials[row] = GatherSlot{__float_as_uint(seg_m), cnt, flags, 0u, seg_s, 0.0};
                        uint8_t* rec = p.granule_out + row * p.granule_stride;
                        if (in) {
                            reinterpret_cast<float*>(rec + SamplerRecord::kWarpMaxOffset)[lane] = wmax;
                            reinterpret_cast<double*>(rec + SamplerRecord::kWarpMassOffset)[lane] = wp.mass;
                        }
                        double* rg = reinterpret_cast<double*>(rec + SamplerRecord::kGranuleOffset);
                        // The record is chunk-major ([chunk][warp]); the table warp-major.
                        for (int i = lane; i < ngran; i += 32) {
                            const int w = i / nch, c = i - w * nch;
                            rg[c * kConsumerWarps + w] = granules[w * kMaxChunksSampler + c];
                        }
                    } else if (d.kind == kUnitSplit) {
                        finish_split_piece<T, true>(p, d, nchunks, GatherSlot{__float_as_uint(seg_m), cnt, flags, 0u, seg_s, 0.0},
                                                    wf, granules, sh.part_uniform[slot], sh, ss, lrow, mrow, lane);
                    } else {
                        // Rank partials, all-gathered in rank order, merged identically on every rank.
                        if (lane == 0) {
                            const GatherSlot mine{__float_as_uint(seg_m), cnt, flags, 0u, seg_s, 0.0};
                            if (csize > 1) cluster_allgather(sh, slot, crank, csize, mine, (k >> 1) & 1u);
                            else sh.slots[slot][0] = mine;
                        }
                        __syncwarp();
                        const SampleMerge mg = merge_sampler_ranks(sh.slots[slot], 1, csize, sh.part_uniform[slot], p.temperature,
                                                                   p.inv_temperature, sh.abort ? kFlagAbort : 0u, lane);
                        if (mg.code != kOk) {
                            if (crank == 0 && lane == 0) {
                                p.status[row] = mg.code;
                                p.tokens[row] = -1;
                                if (p.counts) p.counts[row] = mg.total;
                            }
                        } else if (mg.owner == static_cast<int>(crank)) {
                            const int64_t chosen =
                                sampler_owner_walk<T>(granules, 1, kMaxChunksSampler, ngran, wf, wp.mass, in, mg, p.temperature,
                                                      p.inv_temperature, p.scale2, seg_begin, seg_end, lrow, mrow, ss.walk,
                                                      ss.fac, lane);
                            if (lane == 0) {
                                p.status[row] = chosen >= 0 ? kOk : kNoMass;
                                p.tokens[row] = chosen >= 0 ? p.token_offset + chosen : -1;
                                if (p.counts) p.counts[row] = mg.total;
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(ptx::smem_addr(&sh.part_empty[slot]));
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumer warps
        uint32_t stage = 0, phase = 0;  // ring position of the next chunk (matches the producer)
        // Chunks holding kTPC tokens (every chunk but a ragged last one) take the unpredicated path.
        const int nfull = static_cast<int>((seg_end - seg_begin) / kTPC);
        // A stage's mask words start at the 16-byte boundary at or below the chunk's first word;
        // chunks start on multiples of 128 words, so the word offset is the same for every chunk.
        const int moff = static_cast<int>((p.mask_word_offset + (seg_begin >> 5)) & 3);
        for (uint32_t u = 0, k = 0;; ++u, ++k) {  // u: units read, k: partial slots used
            const uint32_t us = u % kUnitSlots;
            const bool got = wait_bounded(ptx::smem_addr(&sh.unit_full[us]), (u / kUnitSlots) & 1u, &sh.abort);
            const Unit d = got ? sh.units[us] : Unit{0, 0, 0, kUnitEnd, 0, 0};
            __syncwarp();
            if (got && lane == 0) ptx::mbar_arrive(ptx::smem_addr(&sh.unit_empty[us]));
            const uint32_t slot = k & 1u;
            if (flat) {
                if (d.kind == kUnitEnd) {
                    // The warp's last record (its stores complete before the grid does).
                    if (lane == 0 && sh.flat_dst[warp] != nullptr) *sh.flat_dst[warp] = sh.flat_rec[warp];
                    launch_dependents();
                    break;
                }
            } else {
                // The finalizer has released this partial slot (and granule table).
                if (k >= 2) wait_bounded(ptx::smem_addr(&sh.part_empty[slot]), ((k >> 1) - 1u) & 1u, &sh.abort);
                if (d.kind == kUnitEnd) {
                    if (lane == 0) {
                        if (warp == 0) sh.part_unit[slot] = d;
                        ptx::mbar_arrive(ptx::smem_addr(&sh.part_full[slot]));
                    }
                    launch_dependents();
                    break;
                }
            }
            // Sampler: the row's uniform is copied to the partial slot while the row streams (the
            // finalizer needs it right after the last chunk).
            const bool fetch_uniform =
                kSample && !flat && warp == 0 && lane == 0 && p.uniforms != nullptr && p.partials == nullptr;
            if (fetch_uniform) ptx::cp_async_8(ptx::smem_addr(&sh.part_uniform[slot]), p.uniforms + d.row);
            const int64_t row = d.row;
            const uint8_t* lrow = static_cast<const uint8_t*>(p.logits) +
                                  static_cast<size_t>(row) * static_cast<size_t>(p.logit_stride) * E::kBytes;
            const int32_t* mrow =
                p.masks + static_cast<size_t>(d.mask_row) * static_cast<size_t>(p.mask_stride) + p.mask_word_offset;
            const int nch = d.c1 - d.c0;
            double* granules = ss.granules[slot & 1u];
            float2* granules_f = reinterpret_cast<float2*>(granules);
            // Flat schedule: this warp's granule records of the unit's row, and the flags they carry.
            uint4* frec = flat ? ws_flat_records(p, row) + warp : nullptr;
            const uint32_t unit_flags = d.mask_bad ? kFlagBadMaskRow : 0u;
            typename E::NanAcc nan_acc = E::nan_init();
            uint32_t count = 0;
            // argmax: lane's running masked max and the chunk it came from
            float best = -kInf;
            int best_idx = -1;
            int first_valid_chunk = -1;
            // sampler: a warp-uniform reference max `ref` of the valid logits seen so far
            float ref = -kInf;
            bool fast = false;  // weights as one FFMA from `ref` (see lane_mass, mode 0)
            float chi = 0.0f, corr = 1.0f;
            const float sc = p.scale;

            auto chunk = [&](auto full_tag, int c) {
                constexpr bool kFull = decltype(full_tag)::value;
                [[maybe_unused]] const uint32_t count_in = count;  // flat schedule: the chunk's own count
                uint8_t* st = stages + (kBulk ? stage : 0u) * L::kStageBytes;
                const uint32_t* smask;
                int ntok = kTPC;
                if constexpr (!kFull) {
                    const int64_t t0 = seg_begin + static_cast<int64_t>(c) * kTPC;
                    ntok = static_cast<int>(((t0 + kTPC) < seg_end ? (t0 + kTPC) : seg_end) - t0);
                }
                if constexpr (kBulk) {
                    wait_bounded(ptx::smem_addr(&sh.full[stage]), phase, &sh.abort);
                    smask = reinterpret_cast<const uint32_t*>(st + kChunkBytes) + moff;
                } else {
                    // Cooperative plain loads for rows the bulk engine cannot address.
                    const int64_t t0 = seg_begin + static_cast<int64_t>(c) * kTPC;
                    const int nvec_pad = (ntok + kVec - 1) / kVec * kVec;
                    for (int i = tid; i < nvec_pad; i += kConsumerThreads) {
                        uint32_t v = 0u;
                        if (i < ntok) v = E::raw(lrow, t0 + i);
                        if constexpr (E::kBytes == 4) reinterpret_cast<uint32_t*>(st)[i] = v;
                        else reinterpret_cast<uint16_t*>(st)[i] = static_cast<uint16_t>(v);
                    }
                    const int nwords = (ntok + 31) >> 5;
                    for (int i = tid; i < nwords; i += kConsumerThreads) {
                        uint32_t wv = static_cast<uint32_t>(mrow[(t0 >> 5) + i]);
                        const int64_t first_tok = t0 + 32 * static_cast<int64_t>(i);
                        if (first_tok + 31 >= p.vocab) {
                            const int keep = static_cast<int>(p.vocab - first_tok);
                            wv &= keep >= 32 ? 0xFFFFFFFFu : ((1u << keep) - 1u);
                        }
                        reinterpret_cast<uint32_t*>(st + kChunkBytes)[i] = wv;
                    }
                    ptx::named_sync(1, kConsumerThreads);
                    smask = reinterpret_cast<const uint32_t*>(st + kChunkBytes);
                }

                const int nvec = (ntok + kVec - 1) / kVec;
                const uint8_t* wl = st + warp * kWarpBytes;
                uint4 raw[kVecsPerLane];
                uint32_t bits[kVecsPerLane];
#pragma unroll
                for (int j = 0; j < kVecsPerLane; ++j) {
                    const int vec = j * 32 + lane;
                    const bool in = kFull || warp * (kTPW / kVec) + vec < nvec;
                    raw[j] = in ? *reinterpret_cast<const uint4*>(wl + vec * 16) : make_uint4(0, 0, 0, 0);
                    if constexpr (kVec == 8) {
                        // 8 tokens per vector: vector v's bits are byte v of the little-endian words.
                        const uint8_t* wb = reinterpret_cast<const uint8_t*>(smask) + warp * (kTPW / 8);
                        bits[j] = in ? wb[vec] : 0u;
                    } else {
                        const uint32_t* wm = smask + warp * (kTPW / 32);
                        const uint32_t word = in ? wm[(vec * kVec) >> 5] : 0u;
                        bits[j] = (word >> ((vec * kVec) & 31)) & kVecMask;
                    }
                }
                // A full chunk's valid tokens are counted on whole mask words (one word per lane),
                // a ragged last chunk's per vector.
                uint32_t cword = 0u;
                if constexpr (kFull) {
                    constexpr int kWords = kTPW / 32;
                    if (kWords >= 32 || lane < kWords) cword = smask[warp * kWords + lane];
                }
                // Stage contents are in registers: release it to the producer.
                if constexpr (kBulk) {
                    __syncwarp();
                    if (lane == 0) {
                        ptx::mbar_arrive(ptx::smem_addr(&sh.empty[stage]));
                        // Flat schedule: the previous chunk's record, stored after the release.
                        if (flat && sh.flat_dst[warp] != nullptr) {
                            *sh.flat_dst[warp] = sh.flat_rec[warp];
                            sh.flat_dst[warp] = nullptr;
                        }
                    }
                } else {
                    ptx::named_sync(1, kConsumerThreads);  // stage 0 reusable
                }
                if constexpr (kFull) count += __popc(cword);

                if constexpr (!kSample) {
                    // Masked max of the lane's tokens in this chunk (invalid tokens = -inf).  Only
                    // the chunk where the lane's max first reached its value is remembered; the
                    // finalizer recovers the token index from that chunk.
                    float vmax;
                    uint32_t anyb = 0u;
                    if constexpr (E::kBytes == 2) {
                        uint32_t t = E::kNegInf2;
#pragma unroll
                        for (int j = 0; j < kVecsPerLane; ++j) {
                            E::nan_update(nan_acc, raw[j]);
                            if constexpr (!kFull) count += __popc(bits[j]);
                            anyb |= bits[j];
                            uint32_t q[4];
                            mask_pairs<E>(raw[j], bits[j], q);
                            t = E::max2(t, E::max2(E::max2(q[0], q[1]), E::max2(q[2], q[3])));
                        }
                        vmax = fmaxf(E::lo(t), E::hi(t));
                    } else {
                        vmax = -kInf;
#pragma unroll
                        for (int j = 0; j < kVecsPerLane; ++j) {
                            E::nan_update(nan_acc, raw[j]);
                            if constexpr (!kFull) count += __popc(bits[j]);
                            anyb |= bits[j];
                            float v[kVec];
                            E::decode(raw[j], v);
#pragma unroll
                            for (int i = 0; i < kVec; ++i) vmax = fmaxf(vmax, ((bits[j] >> i) & 1u) ? v[i] : -kInf);
                        }
                    }
                    if (vmax > best) {
                        best = vmax;
                        best_idx = c;
                    }
                    if (first_valid_chunk < 0 && anyb != 0u) first_valid_chunk = c;
                } else {
                    // Pass 1 over registers: NaN, count, masked values (-inf where invalid).  A
                    // warp without valid tokens in the chunk records mass 0 and computes no weights.
                    uint32_t anyb = 0u;
#pragma unroll
                    for (int j = 0; j < kVecsPerLane; ++j) {
                        E::nan_update(nan_acc, raw[j]);
                        if constexpr (!kFull) count += __popc(bits[j]);
                        anyb |= bits[j];
                    }
                    const bool warp_any = __any_sync(0xFFFFFFFFu, anyb != 0u);
                    uint32_t q16[kVecsPerLane][4];
                    float q32[kVecsPerLane][kVec];
#pragma unroll
                    for (int j = 0; j < kVecsPerLane && warp_any; ++j) {
                        if constexpr (E::kBytes == 2) {
                            mask_pairs<E>(raw[j], bits[j], q16[j]);
                        } else {
                            float v[kVec];
                            E::decode(raw[j], v);
#pragma unroll
                            for (int i = 0; i < kVec; ++i) q32[j][i] = ((bits[j] >> i) & 1u) ? v[i] : -kInf;
                        }
                    }
                    // Raise the warp's reference to the chunk's max of valid logits (NaN ignored:
                    // it fails the row through the NaN flag) and re-derive the exponent form.
                    auto raise = [&]() {
                        float lmax;
                        if constexpr (E::kBytes == 2) {
                            uint32_t t = E::max2(E::max2(E::max2(q16[0][0], q16[0][1]), E::max2(q16[0][2], q16[0][3])),
                                                 E::max2(E::max2(q16[1][0], q16[1][1]), E::max2(q16[1][2], q16[1][3])));
                            t = E::max2(t, E::max2(E::max2(E::max2(q16[2][0], q16[2][1]), E::max2(q16[2][2], q16[2][3])),
                                                   E::max2(E::max2(q16[3][0], q16[3][1]), E::max2(q16[3][2], q16[3][3]))));
                            lmax = fmaxf(E::lo(t), E::hi(t));
                        } else {
                            lmax = -kInf;
#pragma unroll
                            for (int j = 0; j < kVecsPerLane; ++j)
#pragma unroll
                                for (int i = 0; i < kVec; ++i) lmax = fmaxf(lmax, q32[j][i]);
                        }
                        const uint32_t lkey = (lmax == lmax) ? ordered_bits(lmax) : 0u;
                        const uint32_t wkey = __reduce_max_sync(0xFFFFFFFFu, lkey);
                        if (wkey != 0u) ref = fmaxf(ref, ordered_to_float(wkey));
                        const float msc = ref * sc;
                        // One FFMA per token, t = x s - (ref s) rounded: the rounding error `clo` of
                        // ref s is the same for every token and is folded back once per granule as
                        // 2^clo ~ 1 + clo ln 2, exact to ~1e-9 for |ref s| < 2^11 (|clo| <= 2^-14).
                        fast = ref > -kInf && ref < kInf && sc >= 1e-30f && fabsf(msc) < 0x1p11f;
                        chi = -msc;
                        const float clo = fmaf(-ref, sc, -chi);
                        corr = fmaf(clo, 0.6931471805599453f, 1.0f);
                    };
                    // Pass 2: fp32 weights 2^((x - ref) * log2(e) / T), invalid tokens entering as
                    // -inf (weight 0).  In the one-FFMA form the reference may trail the running
                    // max: it is raised only when a lane's mass exceeds kRaiseMass = 2^20 (or is
                    // +inf), so no weight exceeds 2^20.  Otherwise (no valid logit yet, a
                    // tiny temperature or huge logits) it is raised to every chunk's max.
                    float mass = 0.0f;
                    bool done = false, any_mass = false;
                    if (!warp_any) {
                        done = true;
                    } else if (fast) {
                        mass = lane_mass_fast<E>(q16, q32, chi, sc);
                        any_mass = true;
                        if (__any_sync(0xFFFFFFFFu, mass > kRaiseMass)) raise();
                        else done = true;
                    } else {
                        raise();
                        any_mass = true;
                    }
                    if (!done && any_mass) {
                        if (fast) {
                            mass = lane_mass_fast<E>(q16, q32, chi, sc);
                        } else if (ref > -kInf && ref < kInf) {
                            // ref is this chunk's max or above: x - ref <= 0, formed as
                            // 0.5x - 0.5ref so that it cannot overflow, times scale2 = 2 log2(e) / T.
                            const float nhm = -0.5f * ref;
                            const float sc2 = p.scale2;
                            if (sc2 < kInf) mass = lane_mass<E, 1>(q16, q32, nhm, sc2);
                            else mass = lane_mass<E, 2>(q16, q32, nhm, sc2);
                        } else {
                            mass = 0.0f;
                        }
                    }
                    if (any_mass) {
#pragma unroll
                        for (int o = 16; o >= 1; o >>= 1) mass += __shfl_xor_sync(0xFFFFFFFFu, mass, o);
                        if (fast) mass *= corr;
                    }
                    if (flat) {
                        // The granule's record for the workspace: (reference, mass, valid tokens,
                        // flags); NaN is flagged from the first chunk of the unit that met it on.
                        const uint32_t ccount = __reduce_add_sync(0xFFFFFFFFu, count - count_in);
                        const uint32_t cflags = (__any_sync(0xFFFFFFFFu, E::has_nan(nan_acc)) ? kFlagNaN : 0u) | unit_flags |
                                                (sh.abort ? kFlagAbort : 0u);
                        if (lane == 0) {
                            sh.flat_rec[warp] = make_uint4(__float_as_uint(ref), __float_as_uint(mass), ccount, cflags);
                            sh.flat_dst[warp] = frec + c * kConsumerWarps;
                        }
                    } else if (lane == 0) {
                        granules_f[warp * kMaxChunksSampler + (c - d.c0)] = make_float2(ref, mass);
                    }
                }
                if constexpr (kBulk) {
                    if (++stage == static_cast<uint32_t>(kStages)) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            };
            const int cfull = d.c1 < nfull ? d.c1 : nfull;
            for (int c = d.c0; c < cfull; ++c) chunk(std::true_type{}, c);
            for (int c = d.c0 > nfull ? d.c0 : nfull; c < d.c1; ++c) chunk(std::false_type{}, c);

            if (flat) continue;  // nothing to hand over: the records carry the unit
            // ---------------------------------------------------- warp partial -> finalizer
            const bool nan_local = E::has_nan(nan_acc);
            const uint32_t wcount = __reduce_add_sync(0xFFFFFFFFu, count);
            const uint32_t wflags = __any_sync(0xFFFFFFFFu, nan_local) ? kFlagNaN : 0u;
            uint32_t wkey, wchunk = 0xFFFFFFFFu;
            double wmass = 0.0;
            if constexpr (kSample) {
                // Fold the warp's granules to its final reference (one fp64 exp per lane per chunk)
                // so that the finalizer combines 8 warp masses, not every granule.
                wkey = ordered_bits(ref);
                const double wm = static_cast<double>(ref);
                __syncwarp();
                double local = 0.0;
                for (int c = lane; c < nch; c += 32) {
                    const float2 e = granules_f[warp * kMaxChunksSampler + c];
                    const double gm = !(e.y > 0.0f) ? 0.0
                                      : e.x == ref  ? static_cast<double>(e.y)
                                                    : static_cast<double>(e.y) *
                                                          scaled_exp(static_cast<double>(e.x) - wm, p.temperature, p.inv_temperature);
                    granules[warp * kMaxChunksSampler + c] = gm;
                    local += gm;
                }
                wmass = warp_sum(local);
            } else {
                const bool has = best_idx >= 0 || first_valid_chunk >= 0;
                const uint32_t key = has ? ordered_bits(best) : 0u;
                wkey = __reduce_max_sync(0xFFFFFFFFu, key);
                const uint32_t chunk_id = static_cast<uint32_t>(best_idx >= 0 ? best_idx : first_valid_chunk);
                wchunk = __reduce_min_sync(0xFFFFFFFFu, (has && key == wkey) ? chunk_id : 0xFFFFFFFFu);
            }
            if (fetch_uniform) ptx::cp_async_wait_all();
            if (lane == 0) {
                if (warp == 0) sh.part_unit[slot] = d;
                sh.part[slot][warp] = WarpPartial{wkey, wchunk, wcount, wflags, wmass, 0.0};
                ptx::mbar_arrive(ptx::smem_addr(&sh.part_full[slot]));
            }
        }
    }

    // No CTA may exit while a peer can still write into its shared memory.
    if (csize > 1 || dynamic || p.xranks > 0) __syncthreads();
    // Peer-memory exchange: the last CTA to finish publishes this step in every area, unless a
    // CTA gave up waiting (its rows' partials never reached the peers).  The finalizer's peer
    // stores precede the barrier above, which orders them before thread 0's release pattern
    // (fence + counter); the release is cumulative, so a peer that acquires the flag sees them.
    if (p.xranks > 0 && tid == 0) {
        ExchangeHeader* own = reinterpret_cast<ExchangeHeader*>(p.xarea[p.xrank]);
        ptx::fence_acq_rel_sys();
        const uint32_t before = atomicAdd(&own->select_done, sh.abort ? 0x10001u : 1u);
        if ((before & 0xFFFFu) + 1u == gridDim.x) {
            atomicExch(&own->select_done, 0u);
            ptx::fence_acq_rel_sys();
            if ((before >> 16) == 0u && !sh.abort)
                for (int q = 0; q < p.xranks; ++q)
                    ptx::st_release_sys(&reinterpret_cast<ExchangeHeader*>(p.xarea[q])->ready[p.xrank], p.xepoch);
        }
    }
    if (csize > 1) {
        ptx::cluster_arrive();
        ptx::cluster_wait();
    }
    // The last CTA of a dynamic launch to finish returns the ticket and done counters to zero
    // (every CTA took its last ticket before counting itself done; every CTA gets here, bounded
    // waits included, so the counters start each launch at zero).
    if (dynamic && tid == 0) {
        WsHeader* hd = ws_header(p);
        __threadfence();
        // Low word: CTAs done; high word: CTAs that timed out.
        const unsigned long long before = atomicAdd(&hd->done, sh.abort ? (1ull << 32) + 1ull : 1ull);
        if ((before & 0xFFFFFFFFull) + 1ull == gridDim.x) {
            if ((before >> 32) != 0 || sh.abort)
                for (int64_t r = 0; r < p.ws_rows; ++r) atomicExch(ws_row_counter(p, r), 0ull);
            atomicExch(&hd->tickets, 0ull);
            atomicExch(&hd->done, 0ull);
        }
    }
}

constexpr int kFlatMergeWarps = 4;

// Shared memory of one flat_merge_kernel CTA.
struct FlatMergeShared {
    uint4 table[kMaxChunksSampler * kConsumerWarps];  // the row's granule records
    float walk[32][33];
    uint32_t red[kFlatMergeWarps][3];                 // per-warp max key, count, flags
    double wsum[kFlatMergeWarps];                     // per-warp mass sums (block scan)
    double wprefix[kFlatMergeWarps];                  // per-warp first crossing: masses before it
    int32_t wcand[kFlatMergeWarps];                   //   and its granule (0x7FFFFFFF: none)
    int32_t wlast[kFlatMergeWarps];                   // per-warp last positive granule
    double uniform;
};

// Second launch of the flat schedule: the selection launch left one record per (row, chunk, warp)
// granule in the workspace -- (reference max, mass relative to it as fp32 bits, valid tokens,
// flags), from whichever CTAs streamed the row.  One CTA per row (grid-stride) copies the records
// into shared memory and reduces them to the row's status, valid count and largest reference M;
// each thread rescales its granules to fp64 masses relative to M (one exp per granule whose
// reference is below M), a block scan in granule order locates the granule holding u * total, and
// warp 0 walks it (walk_granule).  Launched as a programmatic dependent of the selection launch;
// lets its own dependents start at once (they wait for its completion before touching memory).
template <typename T>
__global__ void __launch_bounds__(kFlatMergeWarps * 32) flat_merge_kernel(const SelectParams p) {
    __shared__ FlatMergeShared ms;
    launch_dependents();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    using E = Elem<T>;
    constexpr int kTPC = Layout<T>::kTokensPerChunk;
    constexpr int kN = kFlatMergeWarps * 32;
    const float kInf = __int_as_float(0x7F800000);
    const int tid = threadIdx.x, lane = tid & 31, wib = tid >> 5;
    const int row_chunks = static_cast<int>((p.vocab + kTPC - 1) / kTPC);
    const int ngran = row_chunks * kConsumerWarps;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        __syncthreads();  // the previous row's tables are no longer read
        const uint4* src = ws_flat_records(p, row);
        const uint32_t dst = ptx::smem_addr(ms.table);
        for (int g = tid; g < ngran; g += kN) ptx::cp_async_16(dst + 16u * static_cast<uint32_t>(g), src + g);
        if (tid == 0) ms.uniform = p.uniforms != nullptr ? p.uniforms[row] : 0.0;
        ptx::cp_async_wait_all();
        __syncthreads();
        uint32_t mkey = 0u, cnt = 0u, fl = 0u;
        for (int g = tid; g < ngran; g += kN) {
            const uint4 r = ms.table[g];
            mkey = max(mkey, ordered_bits(__uint_as_float(r.x)));
            cnt += r.z;
            fl |= r.w;
        }
        mkey = __reduce_max_sync(0xFFFFFFFFu, mkey);
        cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
        fl = __reduce_or_sync(0xFFFFFFFFu, fl);
        if (lane == 0) {
            ms.red[wib][0] = mkey;
            ms.red[wib][1] = cnt;
            ms.red[wib][2] = fl;
        }
        __syncthreads();
        mkey = 0u;
        cnt = 0u;
        fl = 0u;
#pragma unroll
        for (int w = 0; w < kFlatMergeWarps; ++w) {
            mkey = max(mkey, ms.red[w][0]);
            cnt += ms.red[w][1];
            fl |= ms.red[w][2];
        }
        const float M = ordered_to_float(mkey);
        const double u = ms.uniform;
        const int32_t code = (fl & kFlagAbort) ? kTimeout
                             : (fl & kFlagBadMaskRow) ? kBadMaskRow
                             : (fl & kFlagNaN) ? kNaN
                             : (M == kInf) ? kPosInf
                             : (cnt == 0u) ? kEmpty
                             : (M == -kInf) ? kNoMass
                             : !(u >= 0.0 && u < 1.0) ? kBadUniform
                                                      : kOk;
        // Thread t owns granules [t * per, (t + 1) * per): their fp64 masses relative to M (one exp
        // per granule whose reference is below M), a block scan of the owners' sums in granule
        // order, and the first granule whose running mass passes u * total (or, after rounding,
        // the last positive one) with the masses before it.
        const int per = (ngran + kN - 1) / kN;  // <= 4
        const int g0 = tid * per;
        double m[4] = {0.0, 0.0, 0.0, 0.0};
        double local = 0.0;
        if (code == kOk) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int g = g0 + i;
                if (i >= per || g >= ngran) break;
                const uint4 r = ms.table[g];
                const float ref = __uint_as_float(r.x), mass = __uint_as_float(r.y);
                m[i] = !(mass > 0.0f) ? 0.0
                       : ref == M     ? static_cast<double>(mass)
                                      : static_cast<double>(mass) *
                                            scaled_exp(static_cast<double>(ref) - static_cast<double>(M), p.temperature,
                                                       p.inv_temperature);
                local += m[i];
            }
        }
        const double incl = warp_inclusive_scan(local, lane);
        if (lane == 31) ms.wsum[wib] = incl;
        __syncthreads();
        double before = incl - local, total = 0.0;
#pragma unroll
        for (int w = 0; w < kFlatMergeWarps; ++w) {
            if (w < wib) before += ms.wsum[w];
            total += ms.wsum[w];
        }
        const double cutoff = u * total;
        const bool fallback = !(cutoff < total);
        int cand = 0x7FFFFFFF, lastg = -1;
        double cand_prefix = 0.0, acc = before;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (!(m[i] > 0.0)) continue;
            lastg = g0 + i;
            if (!fallback && cand == 0x7FFFFFFF && cutoff < acc + m[i]) {
                cand = g0 + i;
                cand_prefix = acc;
            }
            acc += m[i];
        }
        const int wc = __reduce_min_sync(0xFFFFFFFFu, cand);
        const int wl = __reduce_max_sync(0xFFFFFFFFu, lastg);
        if (cand == wc && wc != 0x7FFFFFFF) ms.wprefix[wib] = cand_prefix;  // one owner per warp
        if (lane == 0) {
            ms.wcand[wib] = wc;
            ms.wlast[wib] = wl;
        }
        __syncthreads();
        if (wib != 0) continue;
        int64_t chosen = -1;
        if (code == kOk && total > 0.0) {
            int gsel = 0x7FFFFFFF, glast = -1;
            double gprefix = 0.0;
#pragma unroll
            for (int w = 0; w < kFlatMergeWarps; ++w) {
                if (ms.wcand[w] < gsel) {
                    gsel = ms.wcand[w];
                    gprefix = ms.wprefix[w];
                }
                glast = max(glast, ms.wlast[w]);
            }
            const bool walk_fallback = gsel == 0x7FFFFFFF;
            if (walk_fallback) {
                gsel = glast;
                gprefix = 0.0;
            }
            if (gsel >= 0) {
                int64_t mr = row;
                if (p.mask_rows != nullptr) {  // a bad index is flagged in the row's records
                    mr = p.mask_rows[row];
                    if (mr < 0 || mr >= p.mask_table_rows) mr = 0;
                }
                const uint8_t* lrow = static_cast<const uint8_t*>(p.logits) +
                                      static_cast<size_t>(row) * static_cast<size_t>(p.logit_stride) * E::kBytes;
                const int32_t* mrow = p.masks + static_cast<size_t>(mr) * static_cast<size_t>(p.mask_stride) + p.mask_word_offset;
                chosen = walk_granule<T>(gsel, gprefix, walk_fallback, static_cast<double>(M), cutoff, p.temperature,
                                         p.inv_temperature, p.scale2, 0, p.vocab, lrow, mrow, ms.walk, lane);
            }
        }
        if (lane == 0) {
            p.status[row] = code != kOk ? code : chosen >= 0 ? kOk : kNoMass;
            p.tokens[row] = code == kOk && chosen >= 0 ? p.token_offset + chosen : -1;
            if (p.counts) p.counts[row] = cnt;
        }
    }
}

// Shared-memory bytes the kernel needs (stages + control block + sampler tables).
template <typename T, bool kSample>
constexpr size_t select_smem_bytes(int stages) {
    return static_cast<size_t>(stages) * Layout<T>::kStageBytes + sizeof(Shared) + (kSample ? sizeof(SamplerShared) : 0);
}

}  // namespace bms
