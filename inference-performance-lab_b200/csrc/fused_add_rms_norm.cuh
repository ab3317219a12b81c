// Fused residual add + RMSNorm for sm_100a: kernels and the host-side dispatch.
//
// Semantics (reference: csrc/fused_add_rms_norm_kernel.cu:38-88 and :153-272 of the reference,
// oracle src/inference_performance_lab/kernels/reference.py:7-23), per row of H elements:
//
//   v[c]        = fp32(x[c]) + fp32(residual[c])     fp32 add, round to nearest
//   residual[c] = bf16(v[c])                          bit-exact with bf16(x.float() + r.float())
//   inv         = 1 / sqrt(sum(v^2) / H + eps)        fp32 sum of fp32 squares
//   x[c]        = bf16((v[c] * inv) * fp32(weight[c]))
//
// Kernels:
//
// * rmsnorm_staged_kernel - rows off 16 bytes (x and residual alike) that the shifted kernel does
//   not take and widths that are not a multiple of 8, bf16 outputs. Persistent: one CTA per SM, each CTA owns a
//   contiguous block of rows. One producer thread streams whole rows of x and residual into a
//   ring of shared-memory stages with bulk async copies (cp.async.bulk, completion on an
//   mbarrier); consumer warps take a row at a time (a "group" of 1, 2, 4 or 8 warps per row,
//   chosen from the row count) and make two passes over the staged row: pass 1 computes v,
//   writes residual and accumulates sum(v^2); pass 2 recomputes v from the staged bytes and
//   writes x. The row therefore crosses HBM exactly once in each direction, the register cost
//   does not grow with H, and the gamma vector is staged in shared memory once per CTA (once
//   per SM). Misaligned rows are handled by copying the 16-byte-aligned span that covers the
//   row and masking the elements outside it; gamma is staged with the same shift so that every
//   shared-memory access is a 16-byte vector. Requires x and residual to share their offset
//   modulo 16 bytes (they are then aligned alike in every row).
//
// * rmsnorm_warp_kernel - many short rows (H <= 1024, H % 8 == 0, 16-byte aligned) that move
//   under 7 KiB each: a warp per row, eight rows a CTA, values in registers; see below.
//
// * rmsnorm_cta_kernel - 16-byte aligned rows of H <= 16384, up to 256 of them (decode batches)
//   or, with one chunk a thread, as many as have their CTAs resident at once: a CTA per row, the
//   row in registers, one memory round trip.
//
// * rmsnorm_stash_kernel - the main path of every op: more 16-byte aligned rows, up to
//   H = 32768. A small CTA for every row, each thread's raw chunks held in registers across the
//   reduction. The planner (ipl_b200.cu) gives the measured crossovers.
//
// * rmsnorm_shifted_kernel<P> - the stash kernel's scheme for many rows off 16 bytes (P elements,
//   x and residual alike), bf16 outputs, on the aligned chunks that cover each row.
//
// * rmsnorm_rowwise_kernel - the general fallback for any alignment (e.g. only one of x and
//   residual misaligned, as in the reference's misaligned tests) and for rows too long to
//   stage: one CTA per row, coalesced 2-byte accesses, values cached in registers when
//   H <= 4096, otherwise a second read of the row (which hits L2).
#pragma once

#include "ipl_common.cuh"

namespace ipl {

// What a row kernel computes.
//   kModeFused:    residual = bf16(x + residual); x = bf16(norm)           (the reference op)
//   kModePlain:    out = bf16(norm(x))                                     (RMSNorm, no residual)
//   kModeFusedFp8: residual = bf16(x + residual); out8 = e4m3(norm / scale) (x read only)
// norm = (v * rsqrt(mean(v^2) + eps)) * gamma with v = fp32 sum (or fp32 x).
constexpr int kModeFused = 0;
constexpr int kModePlain = 1;
constexpr int kModeFusedFp8 = 2;

constexpr int kStagedConsumerWarps = 16;
constexpr int kStagedThreads = (kStagedConsumerWarps + 1) * kWarpSize;  // + 1 producer warp
constexpr int kStagedMaxStages = 32;
constexpr int kStagedUnroll = 2;  // chunks per thread in flight between shared-memory loads and use
constexpr int kRowwiseThreads = 256;
constexpr int kRowwiseCachedPerThread = 16;  // rows up to 4096 elements keep v in registers

struct StagedParams {
    uint16_t* x;          // input rows (and the normalised output of the fused op)
    uint16_t* residual;   // fused op: residual rows, updated in place; plain RMSNorm: unused
    uint16_t* out;        // normalised output rows (== x for the fused op)
    uint8_t* out8;        // fp8 (e4m3) output rows of kModeFusedFp8
    const float* scale;   // kModeFusedFp8: device scalar, output = norm / *scale
    const uint16_t* weight;
    int64_t rows;
    int hidden;
    int chunks_max;     // 16-byte chunks in one staged row (covers any phase)
    int stage_bytes;    // bytes of one stage: x span, then (fused op) residual span
    int stages;         // ring depth S (any value >= 1; see the consumer's wait)
    int row_phase;      // element offset of row 0 of x (and residual) inside its 16-byte chunk
    float epsilon;
};

// Shared memory map (dynamic):
//   [stages * stage_bytes]      staged rows (x span, then residual span)
//   [chunks_max * 16]           gamma as copied (bf16, 16-byte aligned span around the weight)
//   [chunks_max * 32]           gamma widened to fp32 and aligned to the rows' phase, in two
//                               planes of chunks_max * 16 bytes: elements 0-3 of chunk k at
//                               plane 0 + 16k, elements 4-7 at plane 1 + 16k (a warp's 16-byte
//                               loads of consecutive chunks then hit consecutive banks)
//   [2 * stages + 1] mbarriers  S full, S empty, 1 gamma
//   [2 * 16 floats]             cross-warp partial sums (two parities)
//   [kStagedMaxStages ints]     per-stage count of warp releases (W per consumed row)
//   [16 bytes]                  abort flag
struct StagedLayout {
    uint32_t weight_raw_offset;
    uint32_t weight_f32_offset;
    uint32_t barrier_offset;
    uint32_t reduce_offset;
    uint32_t released_offset;
    uint32_t abort_offset;
    uint32_t total;
};

__host__ __device__ inline StagedLayout staged_layout(int stages, int stage_bytes, int chunks_max) {
    StagedLayout l;
    const uint32_t span = static_cast<uint32_t>(chunks_max) * 16u;
    l.weight_raw_offset = static_cast<uint32_t>(stages) * static_cast<uint32_t>(stage_bytes);
    l.weight_f32_offset = l.weight_raw_offset + span;
    l.barrier_offset = l.weight_f32_offset + 2u * span;
    l.reduce_offset = l.barrier_offset + 8u * (2u * static_cast<uint32_t>(stages) + 1u);
    l.released_offset = l.reduce_offset + 2u * kStagedConsumerWarps * 4u;
    l.abort_offset = l.released_offset + 4u * kStagedMaxStages;
    l.total = l.abort_offset + 16u;
    return l;
}

// The 8 values of a staged chunk as four fp32 pairs (element 2i in the low half of pair i).
struct Pairs4 {
    F32x2 v[4];
};

__device__ __forceinline__ Pairs4 chunk_sum(const U32x4& xs, const U32x4& rs) {
    Pairs4 v;
#pragma unroll
    for (int i = 0; i < 4; ++i) v.v[i] = f32x2_add(bf16x2_widen(xs.v[i]), bf16x2_widen(rs.v[i]));
    return v;
}

__device__ __forceinline__ Pairs4 chunk_widen(const U32x4& xs) {
    Pairs4 v;
#pragma unroll
    for (int i = 0; i < 4; ++i) v.v[i] = bf16x2_widen(xs.v[i]);
    return v;
}

// Zeroes the elements of a partial chunk that lie outside the row ([0, hidden)).
__device__ __forceinline__ void mask_outside(Pairs4& v, int first, int hidden) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float lo, hi;
        f32x2_split(v.v[i], lo, hi);
        const int c = first + 2 * i;
        lo = (c >= 0 && c < hidden) ? lo : 0.0f;
        hi = (c + 1 >= 0 && c + 1 < hidden) ? hi : 0.0f;
        v.v[i] = f32x2_make(lo, hi);
    }
}

__device__ __forceinline__ U32x4 chunk_to_bf16(const Pairs4& v) {
    U32x4 out;
#pragma unroll
    for (int i = 0; i < 4; ++i) out.v[i] = f32x2_to_bf16x2(v.v[i]);
    return out;
}

// Stores the valid elements of a chunk whose span is only partly inside the row.
__device__ __forceinline__ void store_partial_chunk(uint16_t* chunk_base, const U32x4& out, int first,
                                                    int hidden) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int column = first + e;
        if (column >= 0 && column < hidden) {
            const uint32_t word = out.v[e >> 1];
            chunk_base[e] = static_cast<uint16_t>((e & 1) ? (word >> 16) : (word & 0xffffu));
        }
    }
}

__device__ __forceinline__ void store_chunk(uint16_t* chunk_base, const U32x4& out, bool full, int first,
                                            int hidden) {
    if (full) {
        st_v4(chunk_base, out);
    } else {
        store_partial_chunk(chunk_base, out, first, hidden);
    }
}

// Byte offset of fp32 gamma element i (element i % 8 of chunk i / 8) in the two-plane layout.
__device__ __forceinline__ uint32_t gamma_offset(int i, uint32_t plane_bytes) {
    return 16u * static_cast<uint32_t>(i >> 3) + ((i & 4) ? plane_bytes : 0u) + 4u * static_cast<uint32_t>(i & 3);
}

// 8 normalised values -> 8 e4m3 bytes (saturating, round to nearest even), stored at dst: one
// 8-byte store when the chunk is whole and dst is 8-byte aligned, element by element otherwise.
__device__ __forceinline__ void store_fp8_chunk(uint8_t* dst, const Pairs4& v, bool full, int first, int hidden) {
    const uint32_t w0 = f32x2_to_e4m3x2(v.v[0]) | (f32x2_to_e4m3x2(v.v[1]) << 16);
    const uint32_t w1 = f32x2_to_e4m3x2(v.v[2]) | (f32x2_to_e4m3x2(v.v[3]) << 16);
    if (full && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
        st_v2(dst, w0, w1);
        return;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int column = first + e;
        if (column >= 0 && column < hidden) dst[e] = static_cast<uint8_t>(((e < 4 ? w0 : w1) >> (8 * (e & 3))) & 0xffu);
    }
}

// fp32 gamma of chunk k as four pairs. With shift 0 two 16-byte loads (one per plane); otherwise
// (rows whose phase differs from row 0's, only when H % 8 != 0) gathered element by element,
// zero outside the staged span.
__device__ __forceinline__ Pairs4 weight_chunk(uint32_t wf_base, uint32_t plane_bytes, int k, int shift,
                                               int span) {
    Pairs4 w;
    if (shift == 0) {
        lds_pairs(wf_base + 16u * k, w.v[0], w.v[1]);
        lds_pairs(wf_base + plane_bytes + 16u * k, w.v[2], w.v[3]);
        return w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int i0 = 8 * k + 2 * i - shift;
        const float lo = (i0 >= 0 && i0 < span) ? lds_f32(wf_base + gamma_offset(i0, plane_bytes)) : 0.0f;
        const float hi =
            (i0 + 1 >= 0 && i0 + 1 < span) ? lds_f32(wf_base + gamma_offset(i0 + 1, plane_bytes)) : 0.0f;
        w.v[i] = f32x2_make(lo, hi);
    }
    return w;
}

// kMode: the bf16 modes (the fp8 output goes to the vector kernels or the row kernel). out must
// share x's offset modulo 16.
template <int kWarpsPerRow, int kMode>
__global__ void __launch_bounds__(kStagedThreads, 1) rmsnorm_staged_kernel(const StagedParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    static_assert(kMode != kModeFusedFp8, "the staged kernel writes bf16 outputs only");
    static_assert(kStagedConsumerWarps % kWarpsPerRow == 0, "groups must tile the consumer warps");
    constexpr int kGroups = kStagedConsumerWarps / kWarpsPerRow;
    constexpr int kGroupThreads = kWarpsPerRow * kWarpSize;
    constexpr int kConsumerThreads = kStagedConsumerWarps * kWarpSize;

    extern __shared__ __align__(128) unsigned char smem[];
    const StagedLayout layout = staged_layout(p.stages, p.stage_bytes, p.chunks_max);
    const uint32_t smem_base = smem_addr(smem);
    const uint32_t full_bar = smem_base + layout.barrier_offset;
    const uint32_t empty_bar = full_bar + 8u * static_cast<uint32_t>(p.stages);
    const uint32_t weight_bar = empty_bar + 8u * static_cast<uint32_t>(p.stages);
    float* partials = reinterpret_cast<float*>(smem + layout.reduce_offset);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + layout.abort_offset);
    int* released = reinterpret_cast<int*>(smem + layout.released_offset);
    const uint32_t half = static_cast<uint32_t>(p.chunks_max) * 16u;

    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;

    // Contiguous block of rows for this CTA.
    const int64_t row_begin = p.rows * blockIdx.x / gridDim.x;
    const int64_t row_end = p.rows * (blockIdx.x + 1) / gridDim.x;
    const int local_rows = static_cast<int>(row_end - row_begin);

    // The 16-byte aligned spans of x and residual that cover a row (what the producer copies).
    auto row_span = [&](int64_t row, uintptr_t& xbase, uintptr_t& rbase, uint32_t& bytes) {
        const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x + row * p.hidden);
        const uintptr_t ra = kResidual ? reinterpret_cast<uintptr_t>(p.residual + row * p.hidden) : 0;
        xbase = xa & ~static_cast<uintptr_t>(15);
        rbase = ra & ~static_cast<uintptr_t>(15);
        const uint32_t phase = static_cast<uint32_t>(xa - xbase) >> 1;
        bytes = ((phase + static_cast<uint32_t>(p.hidden) + 7u) >> 3) * 16u;
    };

    // While the previous kernel in the stream drains (this CTA may start before it completes),
    // ask L2 for the rows this CTA copies first, so HBM is busy through the dependency wait. A
    // prefetch only warms L2, the point where every SM's accesses meet, so it cannot return data
    // older than what the copies after the wait see.
    if (warp == kStagedConsumerWarps && lane == 0) {
        prefetch_span_l2(p.weight, 2u * static_cast<uint32_t>(p.hidden));  // gamma, copied first
        const int first_round = local_rows < p.stages ? local_rows : p.stages;
        for (int j = 0; j < first_round; ++j) {
            uintptr_t xbase, rbase;
            uint32_t bytes;
            row_span(row_begin + j, xbase, rbase, bytes);
            bulk_prefetch_l2(reinterpret_cast<const void*>(xbase), bytes);
            if constexpr (kResidual) bulk_prefetch_l2(reinterpret_cast<const void*>(rbase), bytes);
        }
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full_bar + 8u * s, 1);
            mbar_init(empty_bar + 8u * s, kWarpsPerRow);
        }
        mbar_init(weight_bar, 1);
        for (int s = 0; s < p.stages; ++s) released[s] = 0;
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // Every input may have been written by the previous kernel in the stream.
    grid_dependency_wait();

    const uintptr_t wa = reinterpret_cast<uintptr_t>(p.weight);
    const int weight_phase = static_cast<int>((wa & 15u) >> 1);

    if (warp == kStagedConsumerWarps) {
        // ---------------- producer: one elected thread issues every bulk copy ----------------
        if (lane == 0) {
            // Gamma: the 16-byte aligned span around it, once per CTA.
            const uintptr_t wbase = wa & ~static_cast<uintptr_t>(15);
            const uint32_t wbytes =
                (static_cast<uint32_t>(wa - wbase) + 2u * static_cast<uint32_t>(p.hidden) + 15u) & ~15u;
            mbar_arrive_expect_tx(weight_bar, wbytes);
            bulk_load(smem_base + layout.weight_raw_offset, reinterpret_cast<const void*>(wbase), wbytes,
                      weight_bar, l2_policy_evict_last());

            // Round of the last copy issued into each stage (-1: none), for the drain below.
            int last_round[kStagedMaxStages];
            for (int s = 0; s < p.stages; ++s) last_round[s] = -1;
            const uint64_t policy = l2_policy_evict_first();  // normal and evict_last measured no faster
            for (int j = 0; j < local_rows; ++j) {
                const int s = j % p.stages;
                const int round = j / p.stages;
                // A wait that gives up (or sees a consumer's abort) ends the issuing: nothing
                // more is copied, and the drain below lets what was issued land.
                if (round > 0 &&
                    !mbar_wait_bounded(empty_bar + 8u * s, (round - 1) & 1, abort,
                                       kFaultEmptyBarrierTimeout)) {
                    break;
                }
#ifdef IPL_TEST_STAGED_SKIP_ROW
                // Test builds only: CTA 0 never issues this row's copy, so the consumers waiting
                // for it run out of time (nothing is left in flight for that stage).
                if (blockIdx.x == 0 && j == IPL_TEST_STAGED_SKIP_ROW) continue;
#endif
                uintptr_t xbase, rbase;
                uint32_t bytes;
                row_span(row_begin + j, xbase, rbase, bytes);
                const uint32_t stage = smem_base + static_cast<uint32_t>(s) * p.stage_bytes;
                const uint32_t bar = full_bar + 8u * static_cast<uint32_t>(s);
                mbar_arrive_expect_tx(bar, kResidual ? 2u * bytes : bytes);
                bulk_load(stage, reinterpret_cast<const void*>(xbase), bytes, bar, policy);
                if constexpr (kResidual) {
                    bulk_load(stage + half, reinterpret_cast<const void*>(rbase), bytes, bar, policy);
                }
                last_round[s] = round;
            }
            // Drain: the CTA must not end while a bulk copy still writes its shared memory. Each
            // stage's full barrier completes one phase per copy, and no copy follows the last one
            // issued into it, so the phase of that round completes exactly when it has landed
            // (at once if a consumer already saw it). Bounded by time alone: the abort flag does
            // not end these waits.
            for (int s = 0; s < p.stages; ++s) {
                if (last_round[s] >= 0) {
                    mbar_wait_timed(full_bar + 8u * static_cast<uint32_t>(s), last_round[s] & 1,
                                    kFaultCopyDrainTimeout);
                }
            }
            mbar_wait_timed(weight_bar, 0, kFaultCopyDrainTimeout);
        }
        return;
    }

    // ---------------- consumers ----------------
    // Agreed exit: a consumer warp whose bounded wait gives up (it then sets the CTA's abort flag)
    // or that finds the flag set never leaves early. It keeps its place in every named barrier
    // below - barrier 1 once, its group's barrier once per row, exactly as many times as its
    // group partners - and skips only the waits, loads, stores and releases it would have made,
    // so no warp of the CTA is left waiting at a barrier. `aborted` is made warp-uniform
    // (__any_sync) after every wait, so each barrier is reached by whole, converged warps.
    const int span = p.chunks_max * 8;
    bool aborted = __any_sync(0xffffffffu, !mbar_wait_bounded(weight_bar, 0, abort, kFaultFullBarrierTimeout));
    // Widen gamma to fp32 once per CTA, aligned to row 0's phase: column c of a row whose
    // phase is row_phase sits at index c + row_phase, so chunk k of such a row lines up with
    // bytes [32k, 32k + 32) of the fp32 copy. Entries outside [0, H) are zero.
    if (!aborted) {
        const uint16_t* raw = reinterpret_cast<const uint16_t*>(smem + layout.weight_raw_offset);
        unsigned char* wf = smem + layout.weight_f32_offset;
        for (int i = threadIdx.x; i < span; i += kConsumerThreads) {
            const int column = i - p.row_phase;
            *reinterpret_cast<float*>(wf + gamma_offset(i, half)) =
                (column >= 0 && column < p.hidden) ? bf16_bits_to_float(raw[column + weight_phase]) : 0.0f;
        }
    }
    named_barrier_sync(1, kConsumerThreads);
    grid_launch_dependents();
    const uint32_t wf_base = smem_base + layout.weight_f32_offset;

    const int group = warp / kWarpsPerRow;
    const int warp_in_group = warp % kWarpsPerRow;
    const int t = threadIdx.x % kGroupThreads;
    const float hidden_f = static_cast<float>(p.hidden);

    // When every row of this CTA has a stage of its own, no bulk copy ever refills a stage, so
    // pass 1 may overwrite the staged bytes with v (fp32) for pass 2 to read back. A refilled stage
    // would need a generic-to-async proxy fence before its release; streaming CTAs recompute v
    // from the staged x and residual instead.
    const bool stash = kResidual && local_rows <= p.stages;

    int parity_slot = 0;
    for (int j = group; j < local_rows; j += kGroups) {
        // Row j lives in stage s = j % S, round r = j / S. A phase-parity wait on the stage's
        // full barrier is exact only if the barrier is in phase r: round r - 1 (row j - S, held
        // by whichever group got it) must be complete, and round r + 1 cannot be, since row
        // j + S is loaded only after this group releases row j. Bulk copies may complete out of
        // issue order, so round r - 1's completion is established from its release count, not
        // from load order: once all W warps of its group released row j - S, it was loaded.
        const int s = j % p.stages;
        const int round = j / p.stages;
        if (!aborted && round > 0) {
            aborted = !spin_until_at_least(released + s, round * kWarpsPerRow, abort, kFaultFullBarrierTimeout);
        }
        aborted = __any_sync(0xffffffffu, aborted);
        const uint32_t bar = full_bar + 8u * static_cast<uint32_t>(s);
        if (!aborted) aborted = !mbar_wait_bounded(bar, round & 1, abort, kFaultFullBarrierTimeout);
        aborted = __any_sync(0xffffffffu, aborted);
        const int64_t row = row_begin + j;
        const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x + row * p.hidden);
        const uintptr_t ra = kResidual ? reinterpret_cast<uintptr_t>(p.residual + row * p.hidden) : 0;
        const uintptr_t oa = reinterpret_cast<uintptr_t>(p.out + row * p.hidden);
        uint16_t* obase = reinterpret_cast<uint16_t*>(oa & ~static_cast<uintptr_t>(15));
        uint16_t* rbase = reinterpret_cast<uint16_t*>(ra & ~static_cast<uintptr_t>(15));
        const int phase = static_cast<int>((xa & 15u) >> 1);
        const int chunks = aborted ? 0 : (phase + p.hidden + 7) >> 3;  // an aborted warp touches nothing
        const uint32_t stage = smem_base + static_cast<uint32_t>(s) * p.stage_bytes;
        const int weight_shift = phase - p.row_phase;

        // Pass 1: residual out + sum of squares (kStagedUnroll chunks loaded before use). With
        // `stash`, the fp32 sum v of chunk k replaces the chunk's staged bytes in place (elements
        // 0-3 over the x chunk, 4-7 over the residual chunk: 16 + 16 bytes either way), so pass 2
        // reads v back instead of widening and adding again; each thread rewrites only the
        // chunks it read.
        F32x2 acc = f32x2_make(0.0f, 0.0f);
        for (int k0 = t; k0 < chunks; k0 += kGroupThreads * kStagedUnroll) {
            U32x4 xs[kStagedUnroll], rs[kStagedUnroll];
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    xs[u] = lds_v4(stage + 16u * k);
                    if constexpr (kResidual) rs[u] = lds_v4(stage + half + 16u * k);
                }
            }
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    const int first = 8 * k - phase;
                    const bool full = first >= 0 && first + 8 <= p.hidden;
                    Pairs4 v;
                    if constexpr (kResidual) {
                        v = chunk_sum(xs[u], rs[u]);
                        const U32x4 out = chunk_to_bf16(v);
                        if (stash) {
                            sts_pairs(stage + 16u * k, v.v[0], v.v[1]);
                            sts_pairs(stage + half + 16u * k, v.v[2], v.v[3]);
                        }
                        store_chunk(rbase + 8 * k, out, full, first, p.hidden);
                    } else {
                        v = chunk_widen(xs[u]);
                    }
                    if (!full) mask_outside(v, first, p.hidden);
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc = f32x2_fma(v.v[i], v.v[i], acc);
                }
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        float sumsq = warp_sum(acc_lo + acc_hi);
        if constexpr (kWarpsPerRow > 1) {
            float* slot = partials + parity_slot * kStagedConsumerWarps + group * kWarpsPerRow;
            if (lane == 0) slot[warp_in_group] = sumsq;
            named_barrier_sync(2 + group, kGroupThreads);
            sumsq = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarpsPerRow; ++w) sumsq += slot[w];
            parity_slot ^= 1;
            // A partner that gave up before the barrier set the abort flag first, so after the
            // barrier every warp of the group sees it and drops the row (its partial sum is
            // missing): the group decides together.
            aborted = __any_sync(0xffffffffu, aborted || *abort != 0);
        }
        if (aborted) continue;  // no pass 2, no release; the next row's barrier is still reached
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);

        // Pass 2: normalised output (v * inv) * gamma; v read back (stash) or recomputed.
        for (int k0 = t; k0 < chunks; k0 += kGroupThreads * kStagedUnroll) {
            Pairs4 vs[kStagedUnroll], ws[kStagedUnroll];
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    if (stash) {
                        lds_pairs(stage + 16u * k, vs[u].v[0], vs[u].v[1]);
                        lds_pairs(stage + half + 16u * k, vs[u].v[2], vs[u].v[3]);
                    } else if constexpr (kResidual) {
                        vs[u] = chunk_sum(lds_v4(stage + 16u * k), lds_v4(stage + half + 16u * k));
                    } else {
                        vs[u] = chunk_widen(lds_v4(stage + 16u * k));
                    }
                    ws[u] = weight_chunk(wf_base, half, k, weight_shift, span);
                }
            }
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    const int first = 8 * k - phase;
                    const bool full = first >= 0 && first + 8 <= p.hidden;
                    Pairs4 v;
#pragma unroll
                    for (int i = 0; i < 4; ++i) v.v[i] = f32x2_mul(f32x2_mul(vs[u].v[i], inv2), ws[u].v[i]);
                    store_chunk(obase + 8 * k, chunk_to_bf16(v), full, first, p.hidden);
                }
            }
        }
        // Release the stage: every lane of this warp has finished reading it.
        __syncwarp();
        if (lane == 0) {
            atomicAdd(released + s, 1);
            mbar_arrive(empty_bar + 8u * s);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Short rows (H <= 1024, H % 8 == 0, 16-byte aligned rows): one warp per row, values in
// registers. A staged row of a few KB costs the producer a barrier round trip and two bulk copies
// for little data; here each lane loads its kChunks 16-byte chunks of x (and residual) with
// vector loads, many warps per SM keep the loads in flight, the reduction is five shuffles, and
// gamma is widened to fp32 in shared memory once per CTA. Measured on B200 against the staged
// kernel (131072 rows): 88 / 92 / 99 % of the copy peak at H = 256 / 512 / 1024 versus 18 / 35 /
// 66 %; from H = 1536 the staged kernel is ahead (its registers do not grow with H).

constexpr int kWarpRowThreads = 256;
constexpr int kWarpRowMaxHidden = 1024;

struct WarpRowParams {
    uint16_t* x;
    uint16_t* residual;
    uint16_t* out;
    uint8_t* out8;
    const float* scale;
    const uint16_t* weight;
    int64_t rows;
    int hidden;
    float epsilon;
    // Stash and shifted kernels: the CTAs the GPU holds at once for this launch (one resident
    // wave) when the launch has rows beyond it, else 0; and how many CTAs, from the first, ask L2
    // for the row one wave ahead of theirs. See prefetch_next_wave_row.
    int64_t lookahead;
    int64_t lookahead_ctas;
    // Cluster kernel: 16-byte chunks of a row that each CTA of a cluster owns (the last CTA
    // may own fewer).
    int cluster_slice;
};

template <int kChunks, int kMode>
__global__ void __launch_bounds__(kWarpRowThreads) rmsnorm_warp_kernel(const WarpRowParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    extern __shared__ __align__(128) unsigned char smem[];  // fp32 gamma, two planes
    const int chunks = p.hidden >> 3;
    const uint32_t plane = static_cast<uint32_t>(chunks) * 16u;
    const uint32_t gamma_base = smem_addr(smem);
    grid_dependency_wait();
    for (int i = threadIdx.x; i < p.hidden; i += kWarpRowThreads) {
        *reinterpret_cast<float*>(smem + gamma_offset(i, plane)) = bf16_bits_to_float(p.weight[i]);
    }
    __syncthreads();
    grid_launch_dependents();
    const float scale_inv = kFp8 ? 1.0f / *p.scale : 1.0f;
    const F32x2 scale_inv2 = f32x2_make(scale_inv, scale_inv);

    const int lane = threadIdx.x % kWarpSize;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kWarpRowThreads / kWarpSize);
    const float hidden_f = static_cast<float>(p.hidden);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * (kWarpRowThreads / kWarpSize) + threadIdx.x / kWarpSize;
         row < p.rows; row += warps) {
        const uint16_t* xr = p.x + row * p.hidden;
        uint16_t* rr = kResidual ? p.residual + row * p.hidden : nullptr;
        uint16_t* orow = p.out + row * p.hidden;
        U32x4 xs[kChunks], rs[kChunks];
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + kWarpSize * i;
            if (c < chunks) {
                xs[i] = ld_v4(xr + 8 * c);
                if constexpr (kResidual) rs[i] = ld_v4(rr + 8 * c);
            }
        }
        Pairs4 v[kChunks];
        F32x2 acc = f32x2_make(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + kWarpSize * i;
            if (c < chunks) {
                if constexpr (kResidual) {
                    v[i] = chunk_sum(xs[i], rs[i]);
                    st_v4(rr + 8 * c, chunk_to_bf16(v[i]));
                } else {
                    v[i] = chunk_widen(xs[i]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) acc = f32x2_fma(v[i].v[e], v[i].v[e], acc);
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float sumsq = warp_sum(acc_lo + acc_hi);
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + kWarpSize * i;
            if (c < chunks) {
                Pairs4 w;
                lds_pairs(gamma_base + 16u * c, w.v[0], w.v[1]);
                lds_pairs(gamma_base + plane + 16u * c, w.v[2], w.v[3]);
#pragma unroll
                for (int e = 0; e < 4; ++e) v[i].v[e] = f32x2_mul(f32x2_mul(v[i].v[e], inv2), w.v[e]);
                if constexpr (kFp8) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[i].v[e] = f32x2_mul(v[i].v[e], scale_inv2);
                    store_fp8_chunk(p.out8 + row * p.hidden + 8 * c, v[i], true, 8 * c, p.hidden);
                } else {
                    st_v4(orow + 8 * c, chunk_to_bf16(v[i]));
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Few rows of any width up to 16384 (decode-sized batches; H % 8 == 0, 16-byte aligned rows): one
// CTA per row, every value in registers. Each thread owns kChunks 16-byte chunks of the row and
// issues the loads of its gamma, x and residual chunks back to back, so a row costs one memory
// round trip, one warp-shuffle reduction and one __syncthreads. The staged kernel's bulk copies,
// mbarrier hand-off and shared-memory gamma pay off when a CTA streams many rows; for a handful of
// rows they are latency on the critical path.

constexpr int kCtaRowMaxThreads = 512;

// Gamma chunk c (8 bf16) as four packed pairs: one 16-byte load (kept in L1, since every CTA on
// the SM reads the same gamma) when gamma is 16-byte aligned, eight 2-byte loads otherwise.
__device__ __forceinline__ U32x4 load_weight_chunk(const uint16_t* weight, int c, bool aligned) {
    if (aligned) return ld_shared_ro_v4(weight + 8 * c);
    U32x4 w;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        w.v[e] = static_cast<uint32_t>(weight[8 * c + 2 * e]) | (static_cast<uint32_t>(weight[8 * c + 2 * e + 1]) << 16);
    }
    return w;
}
constexpr int kCtaRowMaxHidden = 4 * 8 * kCtaRowMaxThreads;  // 16384: four chunks per thread
constexpr int64_t kCtaRowMaxRows = 256;
// Registers of the one-chunk instances (H <= 4096), held there by their launch bound, so the
// planner can tell how many of their CTAs an SM holds at once: the bf16 ops 40, the fp8 op 64.
constexpr int kRegistersPerSm = 65536;
constexpr int kThreadsPerSm = 2048;
constexpr int kCtaRowRegs = 40;
constexpr int kCtaRowRegsFp8 = 64;
constexpr int kCtaRowMaxResident = 8;  // CTAs an SM is counted on for one wave (at 10, 1480 x 1032 lost 13 %)

constexpr unsigned kGammaPrefetchCtas = 148;

// Before the dependency wait of a CTA-per-row kernel: ask L2 for the CTA's first row (16-byte
// aligned rows, H % 8 == 0), so its loads after the wait find it there. Safe for the same reason
// as the staged kernel's prefetch: L2 is where every SM's accesses meet.
template <bool kResidual>
__device__ __forceinline__ void prefetch_first_row(const WarpRowParams& p) {
    if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) < p.rows) {
        const int64_t row = blockIdx.x;
        const uint32_t bytes = 2u * static_cast<uint32_t>(p.hidden);
        bulk_prefetch_l2(p.x + row * p.hidden, bytes);
        if constexpr (kResidual) bulk_prefetch_l2(p.residual + row * p.hidden, bytes);
        // Gamma too (each layer of a model has its own, cold in L2 by the time it runs again);
        // every row's pass 2 waits on it. The first CTAs are enough: later ones find it in L2.
        if (blockIdx.x < kGammaPrefetchCtas) prefetch_span_l2(p.weight, bytes);
    }
}

// After its dependency wait, CTA b (b < lookahead_ctas) asks L2 for row b + lookahead, one wave
// ahead: a row that a CTA of the following wave will load. A launch of a few waves otherwise runs
// out of DRAM requests once its first wave's loads have returned: the first wave's rows were
// prefetched before the wait and arrive from L2, while the next wave's CTAs issue their loads
// only as the first wave's CTAs retire. With the look-ahead the next wave's rows stream from HBM
// while the current wave computes. Issued after the wait, it cannot race the previous kernel's
// writes, and it competes with no earlier launch's traffic. The planner lets every CTA ask in a
// launch of up to four waves and only the first wave beyond that, where the extra requests only
// compete with the demand loads. Measured on B200 (cold, CUDA graph, fused op, against no
// look-ahead): 2048 x 3584 9.31 against 10.29 us, 1536 x 3584 8.14 against 8.68, every CTA at
// 4096 x 3584 17.66 against 18.96 and at 2048 x 8192 20.28 against 21.93; at 8192 x 4096 every
// CTA asking was 2 % slower and the first wave alone 3 % faster, at 32768 and 262144 x 8192 every
// CTA 2 % slower and the first wave alone level; a distance of two waves thrashed L2 at
// 262144 x 8192 (3056 against 2468 us), hence one.
template <bool kResidual>
__device__ __forceinline__ void prefetch_next_wave_row(const WarpRowParams& p) {
    if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) < p.lookahead_ctas &&
        static_cast<int64_t>(blockIdx.x) + p.lookahead < p.rows) {
        const int64_t row = static_cast<int64_t>(blockIdx.x) + p.lookahead;
        const uint32_t bytes = 2u * static_cast<uint32_t>(p.hidden);
        prefetch_span_l2(p.x + row * p.hidden, bytes);
        if constexpr (kResidual) prefetch_span_l2(p.residual + row * p.hidden, bytes);
    }
}

template <int kChunks, int kMode>
__global__ void __launch_bounds__(
    kCtaRowMaxThreads,
    kChunks == 1 ? kRegistersPerSm / (kCtaRowMaxThreads * (kMode == kModeFusedFp8 ? kCtaRowRegsFp8 : kCtaRowRegs))
                 : (kChunks == 2 ? 2 : 1)) rmsnorm_cta_kernel(const WarpRowParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    __shared__ float partials[2][kCtaRowMaxThreads / kWarpSize];
    const int chunks = p.hidden >> 3;
    const int warps = static_cast<int>(blockDim.x) / kWarpSize;
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const float hidden_f = static_cast<float>(p.hidden);

    prefetch_first_row<kResidual>(p);
    // Every input (gamma and the scale included) may have been written by the previous kernel.
    grid_dependency_wait();
    grid_launch_dependents();
    U32x4 wraw[kChunks];
    const bool weight_aligned = (reinterpret_cast<uintptr_t>(p.weight) & 15u) == 0;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const int c = threadIdx.x + static_cast<int>(blockDim.x) * i;
        if (c < chunks) wraw[i] = load_weight_chunk(p.weight, c, weight_aligned);
    }
    const float scale_inv = kFp8 ? 1.0f / *p.scale : 1.0f;
    const F32x2 scale_inv2 = f32x2_make(scale_inv, scale_inv);

    int parity = 0;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint16_t* xr = p.x + row * p.hidden;
        uint16_t* rr = kResidual ? p.residual + row * p.hidden : nullptr;
        U32x4 xs[kChunks], rs[kChunks];
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = threadIdx.x + static_cast<int>(blockDim.x) * i;
            if (c < chunks) {
                xs[i] = ld_v4(xr + 8 * c);
                if constexpr (kResidual) rs[i] = ld_v4(rr + 8 * c);
            }
        }
        Pairs4 v[kChunks];
        F32x2 acc = f32x2_make(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = threadIdx.x + static_cast<int>(blockDim.x) * i;
            if (c < chunks) {
                if constexpr (kResidual) {
                    v[i] = chunk_sum(xs[i], rs[i]);
                    st_v4(rr + 8 * c, chunk_to_bf16(v[i]));
                } else {
                    v[i] = chunk_widen(xs[i]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) acc = f32x2_fma(v[i].v[e], v[i].v[e], acc);
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float warp_total = warp_sum(acc_lo + acc_hi);
        // Two parities of partials: row k + 1 writes the other set, and row k + 2 can only write
        // this one after every thread has passed row k + 1's barrier, i.e. finished reading it.
        if (lane == 0) partials[parity][warp] = warp_total;
        __syncthreads();
        float sumsq = 0.0f;
        for (int w = 0; w < warps; ++w) sumsq += partials[parity][w];
        parity ^= 1;
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = threadIdx.x + static_cast<int>(blockDim.x) * i;
            if (c < chunks) {
                const Pairs4 w = chunk_widen(wraw[i]);
#pragma unroll
                for (int e = 0; e < 4; ++e) v[i].v[e] = f32x2_mul(f32x2_mul(v[i].v[e], inv2), w.v[e]);
                if constexpr (kFp8) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[i].v[e] = f32x2_mul(v[i].v[e], scale_inv2);
                    store_fp8_chunk(p.out8 + row * p.hidden + 8 * c, v[i], true, 8 * c, p.hidden);
                } else {
                    st_v4(p.out + row * p.hidden + 8 * c, chunk_to_bf16(v[i]));
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Many rows of moderate width (H % 8 == 0, 16-byte aligned rows, 1024 < H <= 16384): a small CTA
// for every row - ceil(H / (8 * U)) threads rounded up to a warp (64..512), each owning up to U
// 16-byte chunks whose loads it issues back to back - so a row costs one memory round trip and the
// hardware keeps many rows per SM in flight, starting the next as soon as one retires. Each thread
// keeps its raw x (and residual) words in registers across the row's reduction: pass 1 computes
// v, writes residual and sums v^2; pass 2 recomputes v from the same words (the same fp32 adds, so
// bit for bit) and writes the output. No shared memory holds the row, and HBM sees each byte once.
// The launch bound holds every instance to 64 registers (fused 62, plain 56, fp8 62, plain with
// U = 8 56; no spills): the fp8 and U = 8 instances exceed that unbounded (100 and 112) for no
// gain in rows per SM, and 64 is what the fused op's 60 registers are allocated as anyway.

constexpr int kStashChunks = 4;       // 16-byte chunks per thread: all of a thread's loads in flight at once
constexpr int kStashWideChunks = 8;   // plain RMSNorm of long rows: twice the bytes in flight per thread
constexpr int kStashMinThreads = 64;
constexpr int kStashMaxThreads = 512;
constexpr int kStashMaxHidden = 16384;      // 512 threads of four chunks
constexpr int kStashMaxLongHidden = 32768;  // 512 threads of eight chunks
// Add+RMSNorm and the fp8 op on rows of 16384 < H <= 20480 (up to 320 threads of eight chunks),
// more than 256 of them: the capped instance, held to 96 registers (4-8 bytes of spills) so that
// two CTAs share an SM - 16-25 % faster from 1024 rows than one CTA an SM at 128 registers, which
// stays the choice from H = 24576 (two no longer fit) and for fewer rows.
constexpr int kStashCappedThreads = 320;
constexpr int kStashCappedMaxHidden = 8 * kStashWideChunks * kStashCappedThreads;  // 20480
// A row the stash kernel takes beyond one wave moves at least this many bytes through HBM: below
// it one CTA a row is held to the rate at which the GPU starts CTAs (about one a nanosecond).
constexpr int64_t kStashMinRowBytes = 7168;

template <int kUnroll, int kMode, bool kCapped = false>
__global__ void __launch_bounds__(kCapped ? kStashCappedThreads : kStashMaxThreads,
                                  kCapped || !(kUnroll > kStashChunks && kMode != kModePlain) ? 2 : 1)
    rmsnorm_stash_kernel(const WarpRowParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    __shared__ float partials[2][kStashMaxThreads / kWarpSize];
    const int threads = static_cast<int>(blockDim.x);
    const int warps = threads / kWarpSize;
    const int chunks = p.hidden >> 3;
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const float hidden_f = static_cast<float>(p.hidden);
    const bool weight_aligned = (reinterpret_cast<uintptr_t>(p.weight) & 15u) == 0;
    // Gamma staged in shared memory (four chunks a thread, 16-byte aligned weight; the launch
    // gives H * 2 bytes of dynamic shared memory): each thread copies the gamma chunks it will use
    // in pass 2 with cp.async right after the dependency wait, so the copies land while the row's
    // own loads are in flight and pass 2 reads shared memory instead of making an L1/L2 round trip
    // after the reduction barrier. Each thread reads only the chunks it copied, so waiting for
    // its own copies is enough. Measured on B200 (cold, CUDA graph, fused op, against gamma loaded
    // in pass 2): 2048 x 3584 9.15 against 9.34 us, 1536 x 3584 7.47 against 7.94, 8192 x 3584
    // -1.7 %, 2048 x 8192 -1.3 %, 262144 x 8192 -0.2 %.
    extern __shared__ __align__(16) unsigned char gamma_smem[];
    const uint32_t gamma_base = smem_addr(gamma_smem);
    const bool gamma_staged = kUnroll == kStashChunks && weight_aligned;

    prefetch_first_row<kResidual>(p);
    grid_dependency_wait();
    grid_launch_dependents();
    prefetch_next_wave_row<kResidual>(p);
    if (gamma_staged) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) cp_async_16(gamma_base + 16u * c, p.weight + 8 * c);
        }
    }
    const float scale_inv = kFp8 ? 1.0f / *p.scale : 1.0f;
    const F32x2 scale_inv2 = f32x2_make(scale_inv, scale_inv);

    int parity = 0;
    // threads * kUnroll >= chunks, as planned: every chunk of the row belongs to one thread.
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint16_t* xr = p.x + row * p.hidden;
        uint16_t* rr = kResidual ? p.residual + row * p.hidden : nullptr;
        F32x2 acc = f32x2_make(0.0f, 0.0f);
        U32x4 xs[kUnroll], rs[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                xs[u] = ld_v4(xr + 8 * c);
                if constexpr (kResidual) rs[u] = ld_v4(rr + 8 * c);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                Pairs4 v;
                if constexpr (kResidual) {
                    v = chunk_sum(xs[u], rs[u]);
                    st_v4(rr + 8 * c, chunk_to_bf16(v));
                } else {
                    v = chunk_widen(xs[u]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) acc = f32x2_fma(v.v[e], v.v[e], acc);
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float warp_total = warp_sum(acc_lo + acc_hi);
        if (lane == 0) partials[parity][warp] = warp_total;  // two parities: see rmsnorm_cta_kernel
        if (gamma_staged) cp_async_wait_all();
        __syncthreads();
        float sumsq = 0.0f;
        for (int w = 0; w < warps; ++w) sumsq += partials[parity][w];
        parity ^= 1;
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                Pairs4 v = kResidual ? chunk_sum(xs[u], rs[u]) : chunk_widen(xs[u]);
                const Pairs4 w = chunk_widen(gamma_staged ? lds_v4(gamma_base + 16u * c)
                                                          : load_weight_chunk(p.weight, c, weight_aligned));
#pragma unroll
                for (int e = 0; e < 4; ++e) v.v[e] = f32x2_mul(f32x2_mul(v.v[e], inv2), w.v[e]);
                if constexpr (kFp8) {
                    // The planner gives this kernel 8-byte aligned fp8 rows (H % 8 == 0).
#pragma unroll
                    for (int e = 0; e < 4; ++e) v.v[e] = f32x2_mul(v.v[e], scale_inv2);
                    const uint32_t w0 = f32x2_to_e4m3x2(v.v[0]) | (f32x2_to_e4m3x2(v.v[1]) << 16);
                    const uint32_t w1 = f32x2_to_e4m3x2(v.v[2]) | (f32x2_to_e4m3x2(v.v[3]) << 16);
                    st_v2(p.out8 + row * p.hidden + 8 * c, w0, w1);
                } else {
                    st_v4(p.out + row * p.hidden + 8 * c, chunk_to_bf16(v));
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// The stash kernel's scheme with 256-bit accesses, for add+RMSNorm and its fp8 output: a CTA for
// every row of H / 16 threads (rounded up to a warp), each owning one pair of adjacent 16-byte
// chunks - a 32-byte load of x and of residual, 32-byte stores of residual and x (16 bytes of e4m3
// for the fp8 op) - and staging its 32 bytes of gamma in shared memory by cp.async (the planner
// gives it a 16-byte aligned weight only: a fallback for another weight cost the kernel 3-4 %
// through its registers and schedule). Half the load and store instructions of four 16-byte
// chunks a thread, and smaller CTAs (half the bytes in flight each), so a CTA retires sooner. For
// 1536 <= H <= 5120, H % 16 == 0, 32-byte aligned rows and 257-4096 rows, measured on B200 (cold
// L2, CUDA graph, every CTA looking one wave ahead) against the four-chunk instance: 1.02-1.21x
// (2048 x 3584 8.96 against 9.34 us, 2048 x 2048 5.39 against 6.51), and 1.02-1.12x against the
// CTA-per-row kernel on the one-wave launches it had taken. At H = 6144 and beyond, or past 4096
// rows with only the first wave looking ahead, it fell behind; plain RMSNorm did too.
constexpr int kStashV8MinHidden = 1536;
constexpr int kStashV8MaxHidden = 5120;  // 320 threads
constexpr int64_t kStashV8MaxRows = 4096;

template <int kMode>
__global__ void __launch_bounds__(kStashMaxThreads, 2) rmsnorm_stash_v8_kernel(const WarpRowParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    __shared__ float partials[2][kStashMaxThreads / kWarpSize];
    extern __shared__ __align__(16) unsigned char gamma_smem[];  // H * 2 bytes: gamma, as in the weight
    const int warps = static_cast<int>(blockDim.x) / kWarpSize;
    const int q = threadIdx.x;  // this thread's pair: chunks 2q and 2q + 1
    const bool active = q < (p.hidden >> 4);
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const float hidden_f = static_cast<float>(p.hidden);
    const uint32_t gamma_base = smem_addr(gamma_smem) + 32u * static_cast<uint32_t>(q);

    prefetch_first_row<kResidual>(p);
    grid_dependency_wait();
    grid_launch_dependents();
    prefetch_next_wave_row<kResidual>(p);
    if (active) {
        cp_async_16(gamma_base, p.weight + 16 * q);
        cp_async_16(gamma_base + 16u, p.weight + 16 * q + 8);
    }

    int parity = 0;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint16_t* xr = p.x + row * p.hidden + 16 * q;
        uint16_t* rr = kResidual ? p.residual + row * p.hidden + 16 * q : nullptr;
        U32x8 xs, rs;
        F32x2 acc = f32x2_make(0.0f, 0.0f);
        if (active) {
            xs = ld_v8(xr);
            if constexpr (kResidual) rs = ld_v8(rr);
            const U32x4 x0 = {{xs.v[0], xs.v[1], xs.v[2], xs.v[3]}}, x1 = {{xs.v[4], xs.v[5], xs.v[6], xs.v[7]}};
            Pairs4 a, b;
            if constexpr (kResidual) {
                a = chunk_sum(x0, {{rs.v[0], rs.v[1], rs.v[2], rs.v[3]}});
                b = chunk_sum(x1, {{rs.v[4], rs.v[5], rs.v[6], rs.v[7]}});
                const U32x4 ra = chunk_to_bf16(a), rb = chunk_to_bf16(b);
                st_v8(rr, {{ra.v[0], ra.v[1], ra.v[2], ra.v[3], rb.v[0], rb.v[1], rb.v[2], rb.v[3]}});
            } else {
                a = chunk_widen(x0);
                b = chunk_widen(x1);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = f32x2_fma(a.v[e], a.v[e], acc);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = f32x2_fma(b.v[e], b.v[e], acc);
        }
        // The fp8 op's scale, read behind the row's loads and inverted after the barrier: read
        // ahead of them, its round trip held up every CTA's loads (fp8 output at [2048, 3584] on
        // B200: 9.33 against 9.07 us a launch over 3000 steps, the same bits).
        float scale = 1.0f;
        if constexpr (kFp8) scale = ld_nc_f32(p.scale);
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float warp_total = warp_sum(acc_lo + acc_hi);
        if (lane == 0) partials[parity][warp] = warp_total;  // two parities: see rmsnorm_cta_kernel
        cp_async_wait_all();
        __syncthreads();
        float sumsq = 0.0f;
        for (int w = 0; w < warps; ++w) sumsq += partials[parity][w];
        parity ^= 1;
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
        const float scale_inv = kFp8 ? 1.0f / scale : 1.0f;
        const F32x2 scale_inv2 = f32x2_make(scale_inv, scale_inv);
        if (active) {
            const U32x4 x0 = {{xs.v[0], xs.v[1], xs.v[2], xs.v[3]}}, x1 = {{xs.v[4], xs.v[5], xs.v[6], xs.v[7]}};
            Pairs4 a, b;
            if constexpr (kResidual) {
                a = chunk_sum(x0, {{rs.v[0], rs.v[1], rs.v[2], rs.v[3]}});
                b = chunk_sum(x1, {{rs.v[4], rs.v[5], rs.v[6], rs.v[7]}});
            } else {
                a = chunk_widen(x0);
                b = chunk_widen(x1);
            }
            const Pairs4 wa = chunk_widen(lds_v4(gamma_base));
            const Pairs4 wb = chunk_widen(lds_v4(gamma_base + 16u));
#pragma unroll
            for (int e = 0; e < 4; ++e) a.v[e] = f32x2_mul(f32x2_mul(a.v[e], inv2), wa.v[e]);
#pragma unroll
            for (int e = 0; e < 4; ++e) b.v[e] = f32x2_mul(f32x2_mul(b.v[e], inv2), wb.v[e]);
            if constexpr (kFp8) {
                // 16 e4m3 bytes; the planner gives this kernel a 16-byte aligned fp8 output.
#pragma unroll
                for (int e = 0; e < 4; ++e) a.v[e] = f32x2_mul(a.v[e], scale_inv2);
#pragma unroll
                for (int e = 0; e < 4; ++e) b.v[e] = f32x2_mul(b.v[e], scale_inv2);
                const U32x4 o = {{f32x2_to_e4m3x2(a.v[0]) | (f32x2_to_e4m3x2(a.v[1]) << 16),
                                  f32x2_to_e4m3x2(a.v[2]) | (f32x2_to_e4m3x2(a.v[3]) << 16),
                                  f32x2_to_e4m3x2(b.v[0]) | (f32x2_to_e4m3x2(b.v[1]) << 16),
                                  f32x2_to_e4m3x2(b.v[2]) | (f32x2_to_e4m3x2(b.v[3]) << 16)}};
                st_v4(p.out8 + row * p.hidden + 16 * q, o);
            } else {
                const U32x4 oa = chunk_to_bf16(a), ob = chunk_to_bf16(b);
                st_v8(p.out + row * p.hidden + 16 * q,
                      {{oa.v[0], oa.v[1], oa.v[2], oa.v[3], ob.v[0], ob.v[1], ob.v[2], ob.v[3]}});
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// A row split over a thread-block cluster (H % 8 == 0, 16-byte aligned rows): the C CTAs of a
// cluster (2..8, along x; grid = rows * C) share one row, CTA k owning its 16-byte chunks
// [k * S, min((k + 1) * S, H / 8)), S = p.cluster_slice, in registers as in the stash kernel
// (kUnroll chunks a thread, gamma staged in shared memory by cp.async). Each CTA reduces its Σv²
// over its warps through shared memory, then writes it into slot k of every CTA's `row_sums`
// through distributed shared memory; after one cluster barrier every CTA adds the C slots in the
// same order, so all of them normalise with the same inverse RMS. Two places where one CTA a
// row leaves the GPU short of work: rows longer than one CTA holds in registers (H > 32768, where
// the only other aligned kernel is the rowwise one with 2-byte accesses), and launches of a few
// long rows, where C CTAs a row put C times the SMs on the row's loads.
//
// Barrier protocol, per cluster: every thread arrives (relaxed) at the start and waits before its
// CTA's remote stores, so every CTA of the cluster is running before any writes into its shared
// memory; the stores are followed by a release arrive and an acquire wait, after which each CTA
// reads only its own shared memory, so a CTA that finishes early leaves while no peer can still
// access its shared memory. Both are hardware cluster barriers (no spin of ours), reached
// unconditionally by every thread.
constexpr int kClusterMaxCtas = 8;  // the portable cluster size: no opt-in attribute

template <int kUnroll, int kMode>
__global__ void __launch_bounds__(kStashMaxThreads, 2) rmsnorm_cluster_kernel(const WarpRowParams p) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    __shared__ float partials[kStashMaxThreads / kWarpSize];
    __shared__ float row_sums[kClusterMaxCtas];
    extern __shared__ __align__(16) unsigned char gamma_smem[];  // this CTA's slice of gamma
    const int threads = static_cast<int>(blockDim.x);
    const int warps = threads / kWarpSize;
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const uint32_t rank = cluster_ctarank();
    const uint32_t ctas = cluster_nctarank();
    const int64_t row = static_cast<int64_t>(blockIdx.x) / ctas;
    const int chunks = p.hidden >> 3;
    const int first = static_cast<int>(rank) * p.cluster_slice;
    const int end = first + p.cluster_slice < chunks ? first + p.cluster_slice : chunks;
    const float hidden_f = static_cast<float>(p.hidden);
    const bool weight_aligned = (reinterpret_cast<uintptr_t>(p.weight) & 15u) == 0;
    const uint32_t gamma_base = smem_addr(gamma_smem);
    const uint16_t* xr = p.x + row * p.hidden;
    uint16_t* rr = kResidual ? p.residual + row * p.hidden : nullptr;

    cluster_arrive_relaxed();
    if (threadIdx.x == 0 && end > first) {  // this CTA's slice into L2 while the previous kernel drains
        const uint32_t bytes = 16u * static_cast<uint32_t>(end - first);
        bulk_prefetch_l2(xr + 8 * first, bytes);
        if constexpr (kResidual) bulk_prefetch_l2(rr + 8 * first, bytes);
        if (blockIdx.x < kGammaPrefetchCtas) prefetch_span_l2(p.weight + 8 * first, bytes);
    }
    grid_dependency_wait();
    grid_launch_dependents();
    if (weight_aligned) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = first + static_cast<int>(threadIdx.x) + u * threads;
            if (c < end) cp_async_16(gamma_base + 16u * (c - first), p.weight + 8 * c);
        }
    }
    const float scale_inv = kFp8 ? 1.0f / *p.scale : 1.0f;
    const F32x2 scale_inv2 = f32x2_make(scale_inv, scale_inv);

    U32x4 xs[kUnroll], rs[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int c = first + static_cast<int>(threadIdx.x) + u * threads;
        if (c < end) {
            xs[u] = ld_v4(xr + 8 * c);
            if constexpr (kResidual) rs[u] = ld_v4(rr + 8 * c);
        }
    }
    F32x2 acc = f32x2_make(0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int c = first + static_cast<int>(threadIdx.x) + u * threads;
        if (c < end) {
            Pairs4 v;
            if constexpr (kResidual) {
                v = chunk_sum(xs[u], rs[u]);
                st_v4(rr + 8 * c, chunk_to_bf16(v));
            } else {
                v = chunk_widen(xs[u]);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = f32x2_fma(v.v[e], v.v[e], acc);
        }
    }
    float acc_lo, acc_hi;
    f32x2_split(acc, acc_lo, acc_hi);
    const float warp_total = warp_sum(acc_lo + acc_hi);
    if (lane == 0) partials[warp] = warp_total;
    __syncthreads();
    float cta_total = 0.0f;
    for (int w = 0; w < warps; ++w) cta_total += partials[w];
    cluster_wait_acquire();  // every CTA of the cluster is running
    if (threadIdx.x < ctas) {
        st_shared_cluster_f32(map_shared_to_rank(smem_addr(&row_sums[rank]), threadIdx.x), cta_total);
    }
    if (weight_aligned) cp_async_wait_all();
    cluster_arrive_release();
    cluster_wait_acquire();  // every CTA's sum is in row_sums
    float sumsq = 0.0f;
    for (uint32_t k = 0; k < ctas; ++k) sumsq += row_sums[k];
    const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
    const F32x2 inv2 = f32x2_make(inv, inv);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int c = first + static_cast<int>(threadIdx.x) + u * threads;
        if (c < end) {
            Pairs4 v = kResidual ? chunk_sum(xs[u], rs[u]) : chunk_widen(xs[u]);
            const Pairs4 w = chunk_widen(weight_aligned ? lds_v4(gamma_base + 16u * (c - first))
                                                        : load_weight_chunk(p.weight, c, false));
#pragma unroll
            for (int e = 0; e < 4; ++e) v.v[e] = f32x2_mul(f32x2_mul(v.v[e], inv2), w.v[e]);
            if constexpr (kFp8) {
#pragma unroll
                for (int e = 0; e < 4; ++e) v.v[e] = f32x2_mul(v.v[e], scale_inv2);
                const uint32_t w0 = f32x2_to_e4m3x2(v.v[0]) | (f32x2_to_e4m3x2(v.v[1]) << 16);
                const uint32_t w1 = f32x2_to_e4m3x2(v.v[2]) | (f32x2_to_e4m3x2(v.v[3]) << 16);
                st_v2(p.out8 + row * p.hidden + 8 * c, w0, w1);
            } else {
                st_v4(p.out + row * p.hidden + 8 * c, chunk_to_bf16(v));
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Many rows that start `kPhase` elements (1..7) into a 16-byte block, x and residual (or x and
// out) alike; H % 8 == 0, so every row has that phase. The stash kernel's scheme on the H / 8 + 1
// aligned 16-byte chunks that cover each row: the elements of the first and last chunk that lie
// outside the row are masked out of the sum and not stored (those two chunks are stored in at most
// three aligned 8-, 4- or 2-byte pieces, which the phase fixes at compile time - 1.3-4.9 % faster
// for add+RMSNorm and 2-22 % for RMSNorm than eight checked 2-byte stores; the neighbouring rows'
// CTAs only read them and discard them), and gamma is shifted
// by the phase to match. The phase is a template parameter so that the shift is two aligned
// 16-byte loads and four funnel shifts of fixed registers (with a runtime shift the kernel was
// 2-5 % slower, with a runtime switch 5-10 %). Every loaded byte shares a 16-byte block with an
// element of its row, so it is mapped. Bf16 outputs only.
constexpr int kShiftedMaxHidden = 12288;       // add+RMSNorm
constexpr int kShiftedPlainMaxHidden = 4096;   // RMSNorm: the staged ring stays ahead beyond

// Gamma for aligned chunk a: weight[8a - P + k], k = 0..7, zero outside [0, hidden).
template <int P>
__device__ __forceinline__ U32x4 shifted_gamma_chunk(const uint16_t* weight, int a, int hidden, bool aligned) {
    static_assert(P >= 1 && P <= 7, "phase in elements");
    U32x4 g;
    if (aligned) {
        // The window of weight chunks a - 1 and a, each loaded only where it lies inside the weight.
        const U32x4 zero = {{0u, 0u, 0u, 0u}};
        const U32x4 lo = a > 0 ? ld_shared_ro_v4(weight + 8 * (a - 1)) : zero;
        const U32x4 hi = 8 * a < hidden ? ld_shared_ro_v4(weight + 8 * a) : zero;
        const uint32_t win[8] = {lo.v[0], lo.v[1], lo.v[2], lo.v[3], hi.v[0], hi.v[1], hi.v[2], hi.v[3]};
        constexpr int s = 8 - P;  // window element that is element 8a - P
        constexpr uint32_t bits = 16u * static_cast<uint32_t>(s & 1);
#pragma unroll
        for (int i = 0; i < 4; ++i) g.v[i] = __funnelshift_r(win[s / 2 + i], win[s / 2 + i + 1], bits);
        return g;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int j = 8 * a - P + 2 * i;
        const uint32_t lo = (j >= 0 && j < hidden) ? weight[j] : 0u;
        const uint32_t hi = (j + 1 >= 0 && j + 1 < hidden) ? weight[j + 1] : 0u;
        g.v[i] = lo | (hi << 16);
    }
    return g;
}

// Elements [kLo, kHi) of a 16-byte aligned chunk, stored with the widest aligned stores that fit
// (8, 4 or 2 bytes): at most three stores for any span of a chunk.
template <int kLo, int kHi>
__device__ __forceinline__ void store_span(uint16_t* chunk, const U32x4& w) {
    if constexpr (kLo < kHi) {
        if constexpr (kLo % 4 == 0 && kLo + 4 <= kHi) {
            st_v2(chunk + kLo, w.v[kLo / 2], w.v[kLo / 2 + 1]);
            store_span<kLo + 4, kHi>(chunk, w);
        } else if constexpr (kLo % 2 == 0 && kLo + 2 <= kHi) {
            asm volatile("st.global.b32 [%0], %1;" ::"l"(chunk + kLo), "r"(w.v[kLo / 2]) : "memory");
            store_span<kLo + 2, kHi>(chunk, w);
        } else {
            const uint16_t e = static_cast<uint16_t>((kLo & 1) ? (w.v[kLo / 2] >> 16) : (w.v[kLo / 2] & 0xffffu));
            asm volatile("st.global.b16 [%0], %1;" ::"l"(chunk + kLo), "h"(e) : "memory");
            store_span<kLo + 1, kHi>(chunk, w);
        }
    }
}

// Zeroes elements [kLo, kHi) of a chunk's values (those outside the row).
template <int kLo, int kHi>
__device__ __forceinline__ void zero_span(Pairs4& v) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool lo_out = 2 * i >= kLo && 2 * i < kHi;
        const bool hi_out = 2 * i + 1 >= kLo && 2 * i + 1 < kHi;
        if (lo_out || hi_out) {
            float lo, hi;
            f32x2_split(v.v[i], lo, hi);
            v.v[i] = f32x2_make(lo_out ? 0.0f : lo, hi_out ? 0.0f : hi);
        }
    }
}

template <int kMode, int kPhase>
__global__ void __launch_bounds__(kStashMaxThreads, 2) rmsnorm_shifted_kernel(const WarpRowParams p) {
    static_assert(kMode != kModeFusedFp8, "bf16 outputs only");
    constexpr bool kResidual = kMode != kModePlain;
    constexpr int kUnroll = kStashChunks;
    __shared__ float partials[2][kStashMaxThreads / kWarpSize];
    const int threads = static_cast<int>(blockDim.x);
    const int warps = threads / kWarpSize;
    const int chunks = (p.hidden >> 3) + 1;  // threads * kUnroll >= chunks, as planned
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const float hidden_f = static_cast<float>(p.hidden);
    const bool weight_aligned = (reinterpret_cast<uintptr_t>(p.weight) & 15u) == 0;

    if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) < p.rows) {
        const int64_t row = blockIdx.x;
        const uint32_t bytes = 2u * static_cast<uint32_t>(p.hidden);
        prefetch_span_l2(p.x + row * p.hidden, bytes);
        if constexpr (kResidual) prefetch_span_l2(p.residual + row * p.hidden, bytes);
        if (blockIdx.x < kGammaPrefetchCtas) prefetch_span_l2(p.weight, bytes);
    }
    grid_dependency_wait();
    grid_launch_dependents();
    prefetch_next_wave_row<kResidual>(p);

    int parity = 0;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        // Chunk c covers elements 8c - kPhase .. 8c - kPhase + 7 of the row.
        const uint16_t* xr = p.x + row * p.hidden - kPhase;
        uint16_t* rr = kResidual ? p.residual + row * p.hidden - kPhase : nullptr;
        uint16_t* orow = p.out + row * p.hidden - kPhase;
        F32x2 acc = f32x2_make(0.0f, 0.0f);
        U32x4 xs[kUnroll], rs[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                xs[u] = ld_v4(xr + 8 * c);
                if constexpr (kResidual) rs[u] = ld_v4(rr + 8 * c);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                // The first chunk (thread 0's first) holds elements [kPhase, 8) of the row, the
                // last elements [0, kPhase); both are stored piecewise.
                Pairs4 v = kResidual ? chunk_sum(xs[u], rs[u]) : chunk_widen(xs[u]);
                const bool head = u == 0 && threadIdx.x == 0;
                const bool tail = c == chunks - 1;
                if (head) zero_span<0, kPhase>(v);
                if (tail) zero_span<kPhase, 8>(v);
                if constexpr (kResidual) {
                    const U32x4 out = chunk_to_bf16(v);
                    if (head) {
                        store_span<kPhase, 8>(rr + 8 * c, out);
                    } else if (tail) {
                        store_span<0, kPhase>(rr + 8 * c, out);
                    } else {
                        st_v4(rr + 8 * c, out);
                    }
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) acc = f32x2_fma(v.v[e], v.v[e], acc);
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float warp_total = warp_sum(acc_lo + acc_hi);
        if (lane == 0) partials[parity][warp] = warp_total;  // two parities: see rmsnorm_cta_kernel
        __syncthreads();
        float sumsq = 0.0f;
        for (int w = 0; w < warps; ++w) sumsq += partials[parity][w];
        parity ^= 1;
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = threadIdx.x + u * threads;
            if (c < chunks) {
                Pairs4 v = kResidual ? chunk_sum(xs[u], rs[u]) : chunk_widen(xs[u]);
                const Pairs4 w = chunk_widen(shifted_gamma_chunk<kPhase>(p.weight, c, p.hidden, weight_aligned));
#pragma unroll
                for (int e = 0; e < 4; ++e) v.v[e] = f32x2_mul(f32x2_mul(v.v[e], inv2), w.v[e]);
                const U32x4 out = chunk_to_bf16(v);
                if (u == 0 && threadIdx.x == 0) {
                    store_span<kPhase, 8>(orow + 8 * c, out);
                } else if (c == chunks - 1) {
                    store_span<0, kPhase>(orow + 8 * c, out);
                } else {
                    st_v4(orow + 8 * c, out);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// The shifted kernel's scheme with 256-bit accesses (add+RMSNorm): rows that start kPhase
// elements into a 32-byte block (x and residual alike), so that the H / 8 + 1 aligned 16-byte
// chunks covering a row pair up into 32-byte blocks; H % 16 == 0, so the last pair holds only the
// row's tail chunk, which is loaded and stored with 16 bytes (the chunk after it can lie past the
// tensor's end). A thread owns one pair; its gamma is three aligned 16-byte loads (the chunk
// before the pair and the pair's two), shifted by the phase, where two chunks took four. The
// gamma loads are issued right behind the row's loads and shifted before the reduction, so that
// pass 2 starts from registers after the barrier: measured on B200 (chained launches at
// [2048, 3584], phase 1, the same bits) 10.16 against 10.62 us a launch with the loads after the
// barrier; gamma staged in shared memory by cp.async instead was level with the latter. The
// planner gives it a 16-byte aligned weight.
template <int P>
__device__ __forceinline__ U32x4 shift_window(const U32x4& lo, const U32x4& hi) {
    const uint32_t win[8] = {lo.v[0], lo.v[1], lo.v[2], lo.v[3], hi.v[0], hi.v[1], hi.v[2], hi.v[3]};
    constexpr int s = 8 - P;  // window element that is element 8a - P
    constexpr uint32_t bits = 16u * static_cast<uint32_t>(s & 1);
    U32x4 g;
#pragma unroll
    for (int i = 0; i < 4; ++i) g.v[i] = __funnelshift_r(win[s / 2 + i], win[s / 2 + i + 1], bits);
    return g;
}

constexpr int kShiftedV8MaxHidden = 4080;  // H / 16 + 1 pairs: at most 256 threads

template <int kPhase>
__global__ void __launch_bounds__(kStashMaxThreads, 2) rmsnorm_shifted_v8_kernel(const WarpRowParams p) {
    __shared__ float partials[2][kStashMaxThreads / kWarpSize];
    const int warps = static_cast<int>(blockDim.x) / kWarpSize;
    const int q = threadIdx.x;                   // pair q: aligned chunks 2q and 2q + 1
    const int last = p.hidden >> 4;              // the last pair: the tail chunk H / 8 alone
    const bool active = q <= last;
    const bool head = q == 0;
    const bool tail = q == last;
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const float hidden_f = static_cast<float>(p.hidden);
    const U32x4 zero = {{0u, 0u, 0u, 0u}};

    if (threadIdx.x == 0 && static_cast<int64_t>(blockIdx.x) < p.rows) {
        const int64_t row = blockIdx.x;
        const uint32_t bytes = 2u * static_cast<uint32_t>(p.hidden);
        prefetch_span_l2(p.x + row * p.hidden, bytes);
        prefetch_span_l2(p.residual + row * p.hidden, bytes);
        if (blockIdx.x < kGammaPrefetchCtas) prefetch_span_l2(p.weight, bytes);
    }
    grid_dependency_wait();
    grid_launch_dependents();
    prefetch_next_wave_row<true>(p);

    int parity = 0;
    for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        // Chunk c covers elements 8c - kPhase .. 8c - kPhase + 7 of the row; pair q starts at
        // element 16q - kPhase, a 32-byte boundary.
        uint16_t* xr = p.x + row * p.hidden - kPhase + 16 * q;
        uint16_t* rr = p.residual + row * p.hidden - kPhase + 16 * q;
        U32x4 x0 = zero, x1 = zero, r0 = zero, r1 = zero;
        if (active) {
            if (!tail) {
                const U32x8 xs = ld_v8(xr), rs = ld_v8(rr);
                x0 = {{xs.v[0], xs.v[1], xs.v[2], xs.v[3]}};
                x1 = {{xs.v[4], xs.v[5], xs.v[6], xs.v[7]}};
                r0 = {{rs.v[0], rs.v[1], rs.v[2], rs.v[3]}};
                r1 = {{rs.v[4], rs.v[5], rs.v[6], rs.v[7]}};
            } else {
                x0 = ld_v4(xr);
                r0 = ld_v4(rr);
            }
        }
        // Weight chunks 2q - 1, 2q and 2q + 1 (zero outside the weight); windows (2q - 1, 2q) and
        // (2q, 2q + 1) are the pair's gamma.
        U32x4 gamma_a = zero, gamma_b = zero;
        if (active) {
            const U32x4 wm = head ? zero : ld_shared_ro_v4(p.weight + 16 * q - 8);
            const U32x4 w0 = tail ? zero : ld_shared_ro_v4(p.weight + 16 * q);
            const U32x4 w1 = tail ? zero : ld_shared_ro_v4(p.weight + 16 * q + 8);
            gamma_a = shift_window<kPhase>(wm, w0);
            gamma_b = shift_window<kPhase>(w0, w1);
        }
        F32x2 acc = f32x2_make(0.0f, 0.0f);
        if (active) {
            Pairs4 a = chunk_sum(x0, r0);
            if (head) zero_span<0, kPhase>(a);
            if (tail) zero_span<kPhase, 8>(a);
            const U32x4 ra = chunk_to_bf16(a);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = f32x2_fma(a.v[e], a.v[e], acc);
            if (tail) {
                store_span<0, kPhase>(rr, ra);
            } else {
                const Pairs4 b = chunk_sum(x1, r1);
                const U32x4 rb = chunk_to_bf16(b);
#pragma unroll
                for (int e = 0; e < 4; ++e) acc = f32x2_fma(b.v[e], b.v[e], acc);
                if (head) {
                    store_span<kPhase, 8>(rr, ra);
                    st_v4(rr + 8, rb);
                } else {
                    st_v8(rr, {{ra.v[0], ra.v[1], ra.v[2], ra.v[3], rb.v[0], rb.v[1], rb.v[2], rb.v[3]}});
                }
            }
        }
        float acc_lo, acc_hi;
        f32x2_split(acc, acc_lo, acc_hi);
        const float warp_total = warp_sum(acc_lo + acc_hi);
        if (lane == 0) partials[parity][warp] = warp_total;  // two parities: see rmsnorm_cta_kernel
        __syncthreads();
        float sumsq = 0.0f;
        for (int w = 0; w < warps; ++w) sumsq += partials[parity][w];
        parity ^= 1;
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);
        const F32x2 inv2 = f32x2_make(inv, inv);
        if (active) {
            Pairs4 a = chunk_sum(x0, r0);
            const Pairs4 ga = chunk_widen(gamma_a);
#pragma unroll
            for (int e = 0; e < 4; ++e) a.v[e] = f32x2_mul(f32x2_mul(a.v[e], inv2), ga.v[e]);
            const U32x4 oa = chunk_to_bf16(a);
            uint16_t* orow = p.out + row * p.hidden - kPhase + 16 * q;
            if (tail) {
                store_span<0, kPhase>(orow, oa);
            } else {
                Pairs4 b = chunk_sum(x1, r1);
                const Pairs4 gb = chunk_widen(gamma_b);
#pragma unroll
                for (int e = 0; e < 4; ++e) b.v[e] = f32x2_mul(f32x2_mul(b.v[e], inv2), gb.v[e]);
                const U32x4 ob = chunk_to_bf16(b);
                if (head) {
                    store_span<kPhase, 8>(orow, oa);
                    st_v4(orow + 8, ob);
                } else {
                    st_v8(orow, {{oa.v[0], oa.v[1], oa.v[2], oa.v[3], ob.v[0], ob.v[1], ob.v[2], ob.v[3]}});
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ float block_sum_rowwise(float value, float* partials) {
    value = warp_sum(value);
    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    if (lane == 0) partials[warp] = value;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kRowwiseThreads / kWarpSize; ++w) total += partials[w];
    __syncthreads();  // partials are reused by the next row
    return total;
}

// kCached: v kept in registers (H <= kRowwiseThreads * kRowwiseCachedPerThread); otherwise the
// row is read twice. kMode as for the staged kernel; out may alias x.
template <bool kCached, int kMode>
__global__ void __launch_bounds__(kRowwiseThreads) rmsnorm_rowwise_kernel(
    const uint16_t* x, uint16_t* residual, uint16_t* out, uint8_t* out8, const float* scale,
    const uint16_t* __restrict__ weight, int64_t rows, int hidden, float epsilon) {
    constexpr bool kResidual = kMode != kModePlain;
    constexpr bool kFp8 = kMode == kModeFusedFp8;
    __shared__ float partials[kRowwiseThreads / kWarpSize];
    grid_dependency_wait();
    grid_launch_dependents();
    const float scale_inv = kFp8 ? 1.0f / *scale : 1.0f;
    const float den = static_cast<float>(hidden);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const uint16_t* xr = x + row * hidden;
        uint16_t* rr = kResidual ? residual + row * hidden : nullptr;
        uint16_t* orow = kFp8 ? nullptr : out + row * hidden;
        uint8_t* orow8 = kFp8 ? out8 + row * hidden : nullptr;
        auto emit = [&](int c, float normed) {
            if constexpr (kFp8) {
                orow8[c] = float_to_e4m3(__fmul_rn(normed, scale_inv));
            } else {
                orow[c] = float_to_bf16_bits(normed);
            }
        };
        auto load_v = [&](int c) {
            const float xv = bf16_bits_to_float(xr[c]);
            if constexpr (kResidual) {
                return __fadd_rn(xv, bf16_bits_to_float(rr[c]));
            } else {
                return xv;
            }
        };
        float sumsq = 0.0f;
        float cache[kCached ? kRowwiseCachedPerThread : 1];
        if constexpr (kCached) {
#pragma unroll
            for (int i = 0; i < kRowwiseCachedPerThread; ++i) {
                const int c = threadIdx.x + i * kRowwiseThreads;
                cache[i] = 0.0f;
                if (c < hidden) {
                    const float v = load_v(c);
                    cache[i] = v;
                    sumsq = fmaf(v, v, sumsq);
                    if constexpr (kResidual) rr[c] = float_to_bf16_bits(v);
                }
            }
        } else {
            for (int c = threadIdx.x; c < hidden; c += kRowwiseThreads) {
                const float v = load_v(c);
                sumsq = fmaf(v, v, sumsq);
            }
        }
        sumsq = block_sum_rowwise(sumsq, partials);
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, den) + epsilon);
        if constexpr (kCached) {
#pragma unroll
            for (int i = 0; i < kRowwiseCachedPerThread; ++i) {
                const int c = threadIdx.x + i * kRowwiseThreads;
                if (c < hidden) emit(c, __fmul_rn(__fmul_rn(cache[i], inv), bf16_bits_to_float(weight[c])));
            }
        } else {
            for (int c = threadIdx.x; c < hidden; c += kRowwiseThreads) {
                const float v = load_v(c);
                if constexpr (kResidual) rr[c] = float_to_bf16_bits(v);
                emit(c, __fmul_rn(__fmul_rn(v, inv), bf16_bits_to_float(weight[c])));
            }
        }
    }
}

}  // namespace ipl
