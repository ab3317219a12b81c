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
// * rmsnorm_staged_kernel - the main path. Persistent: one CTA per SM, each CTA owns a
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
// * rmsnorm_rowwise_kernel - the general fallback for any alignment (e.g. only one of x and
//   residual misaligned, as in the reference's misaligned tests) and for rows too long to
//   stage: one CTA per row, coalesced 2-byte accesses, values cached in registers when
//   H <= 4096, otherwise a second read of the row (which hits L2).
#pragma once

#include "ipl_common.cuh"

namespace ipl {

constexpr int kStagedConsumerWarps = 16;
constexpr int kStagedThreads = (kStagedConsumerWarps + 1) * kWarpSize;  // + 1 producer warp
constexpr int kStagedMaxStages = 32;
constexpr int kStagedUnroll = 2;  // chunks per thread in flight between shared-memory loads and use
constexpr int kRowwiseThreads = 256;
constexpr int kRowwiseCachedPerThread = 16;  // rows up to 4096 elements keep v in registers

struct StagedParams {
    uint16_t* x;
    uint16_t* residual;
    const uint16_t* weight;
    int64_t rows;
    int hidden;
    int chunks_max;     // 16-byte chunks in one staged row (covers any phase)
    int stage_bytes;    // bytes of one stage: x span then residual span
    int stages;         // ring depth S (any value >= 1; see the consumer's wait)
    int row_phase;      // element offset of row 0 of x (and residual) inside its 16-byte chunk
    int shift_weight;   // 1: gamma's own phase differs from row_phase, build a shifted copy
    float epsilon;
};

// Shared memory map (dynamic):
//   [stages * stage_bytes]      staged rows (x span, then residual span)
//   [chunks_max * 16]           gamma as copied (16-byte aligned span around the weight)
//   [chunks_max * 16]           gamma shifted to the rows' phase (only if shift_weight)
//   [2 * stages + 1] mbarriers  S full, S empty, 1 gamma
//   [2 * 16 floats]             cross-warp partial sums (two parities)
//   [kStagedMaxStages ints]     per-stage count of warp releases (W per consumed row)
//   [16 bytes]                  abort flag
struct StagedLayout {
    uint32_t weight_raw_offset;
    uint32_t weight_shifted_offset;
    uint32_t barrier_offset;
    uint32_t reduce_offset;
    uint32_t released_offset;
    uint32_t abort_offset;
    uint32_t total;
};

__host__ __device__ inline StagedLayout staged_layout(int stages, int stage_bytes, int chunks_max,
                                                      int shift_weight) {
    StagedLayout l;
    const uint32_t span = static_cast<uint32_t>(chunks_max) * 16u;
    l.weight_raw_offset = static_cast<uint32_t>(stages) * static_cast<uint32_t>(stage_bytes);
    l.weight_shifted_offset = l.weight_raw_offset + span;
    l.barrier_offset = l.weight_shifted_offset + (shift_weight ? span : 0u);
    l.reduce_offset = l.barrier_offset + 8u * (2u * static_cast<uint32_t>(stages) + 1u);
    l.released_offset = l.reduce_offset + 2u * kStagedConsumerWarps * 4u;
    l.abort_offset = l.released_offset + 4u * kStagedMaxStages;
    l.total = l.abort_offset + 16u;
    return l;
}

// Processes the 8 elements of one 16-byte chunk. `first` is the row column of element 0 of the
// chunk (negative, or running past H, for the partial first and last chunks).
template <bool kPass2>
__device__ __forceinline__ void staged_chunk(const U32x4& xs, const U32x4& rs, const U32x4& ws,
                                             int first, int hidden, float inv, float& sumsq,
                                             U32x4& out, bool& full) {
    full = first >= 0 && first + 8 <= hidden;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float v0 = __fadd_rn(bf16_lo(xs.v[i]), bf16_lo(rs.v[i]));
        const float v1 = __fadd_rn(bf16_hi(xs.v[i]), bf16_hi(rs.v[i]));
        if constexpr (!kPass2) {
            const bool ok0 = full || (first + 2 * i >= 0 && first + 2 * i < hidden);
            const bool ok1 = full || (first + 2 * i + 1 >= 0 && first + 2 * i + 1 < hidden);
            sumsq = fmaf(ok0 ? v0 : 0.0f, ok0 ? v0 : 0.0f, sumsq);
            sumsq = fmaf(ok1 ? v1 : 0.0f, ok1 ? v1 : 0.0f, sumsq);
            out.v[i] = pack_bf16x2(v0, v1);
        } else {
            const float o0 = __fmul_rn(__fmul_rn(v0, inv), bf16_lo(ws.v[i]));
            const float o1 = __fmul_rn(__fmul_rn(v1, inv), bf16_hi(ws.v[i]));
            out.v[i] = pack_bf16x2(o0, o1);
        }
    }
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

// Gamma for chunk k: 8 bf16 from shared memory. With shift 0 it is one aligned 16-byte load;
// otherwise (rows whose phase differs from the staged gamma's, only when H % 8 != 0) it is
// gathered element by element, zero outside the staged span.
__device__ __forceinline__ U32x4 weight_chunk(uint32_t weight_base, int k, int shift, int span) {
    if (shift == 0) return lds_v4(weight_base + 16u * k);
    U32x4 ws;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int i0 = 8 * k + 2 * i - shift;
        const uint32_t lo = (i0 >= 0 && i0 < span) ? lds_u16(weight_base + 2u * i0) : 0u;
        const uint32_t hi = (i0 + 1 >= 0 && i0 + 1 < span) ? lds_u16(weight_base + 2u * (i0 + 1)) : 0u;
        ws.v[i] = lo | (hi << 16);
    }
    return ws;
}

template <int kWarpsPerRow>
__global__ void __launch_bounds__(kStagedThreads, 1) rmsnorm_staged_kernel(const StagedParams p) {
    static_assert(kStagedConsumerWarps % kWarpsPerRow == 0, "groups must tile the consumer warps");
    constexpr int kGroups = kStagedConsumerWarps / kWarpsPerRow;
    constexpr int kGroupThreads = kWarpsPerRow * kWarpSize;
    constexpr int kConsumerThreads = kStagedConsumerWarps * kWarpSize;

    extern __shared__ __align__(128) unsigned char smem[];
    const StagedLayout layout = staged_layout(p.stages, p.stage_bytes, p.chunks_max, p.shift_weight);
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

            const uint64_t policy = l2_policy_evict_first();
            for (int j = 0; j < local_rows; ++j) {
                const int s = j % p.stages;
                const int round = j / p.stages;
                if (round > 0 &&
                    !mbar_wait_bounded(empty_bar + 8u * s, (round - 1) & 1, abort,
                                       kFaultEmptyBarrierTimeout)) {
                    break;
                }
                const int64_t row = row_begin + j;
                const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x + row * p.hidden);
                const uintptr_t ra = reinterpret_cast<uintptr_t>(p.residual + row * p.hidden);
                const uintptr_t xbase = xa & ~static_cast<uintptr_t>(15);
                const uintptr_t rbase = ra & ~static_cast<uintptr_t>(15);
                const uint32_t phase = static_cast<uint32_t>(xa - xbase) >> 1;
                const uint32_t chunks = (phase + static_cast<uint32_t>(p.hidden) + 7u) >> 3;
                const uint32_t bytes = chunks * 16u;
                const uint32_t stage = smem_base + static_cast<uint32_t>(s) * p.stage_bytes;
                const uint32_t bar = full_bar + 8u * static_cast<uint32_t>(s);
                mbar_arrive_expect_tx(bar, 2u * bytes);
                bulk_load(stage, reinterpret_cast<const void*>(xbase), bytes, bar, policy);
                bulk_load(stage + half, reinterpret_cast<const void*>(rbase), bytes, bar, policy);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int span = p.chunks_max * 8;
    if (!mbar_wait_bounded(weight_bar, 0, abort, kFaultFullBarrierTimeout)) return;
    // Gamma index of row column c is c + gamma_phase in the staged copy.
    int gamma_phase = weight_phase;
    uint32_t weight_base = smem_base + layout.weight_raw_offset;
    if (p.shift_weight) {
        // Re-stage gamma with the rows' phase so that chunk k of a row lines up with bytes
        // [16k, 16k + 16) of the copy.
        const uint16_t* raw = reinterpret_cast<const uint16_t*>(smem + layout.weight_raw_offset);
        uint16_t* shifted = reinterpret_cast<uint16_t*>(smem + layout.weight_shifted_offset);
        for (int i = threadIdx.x; i < span; i += kConsumerThreads) {
            const int src = i - p.row_phase + weight_phase;
            shifted[i] = (src >= 0 && src < span) ? raw[src] : static_cast<uint16_t>(0);
        }
        named_barrier_sync(1, kConsumerThreads);
        gamma_phase = p.row_phase;
        weight_base = smem_base + layout.weight_shifted_offset;
    }
    grid_launch_dependents();

    const int group = warp / kWarpsPerRow;
    const int warp_in_group = warp % kWarpsPerRow;
    const int t = threadIdx.x % kGroupThreads;
    const float hidden_f = static_cast<float>(p.hidden);

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
        if (round > 0 && !spin_until_at_least(released + s, round * kWarpsPerRow, abort,
                                              kFaultFullBarrierTimeout)) {
            break;
        }
        const uint32_t bar = full_bar + 8u * static_cast<uint32_t>(s);
        if (!mbar_wait_bounded(bar, round & 1, abort, kFaultFullBarrierTimeout)) break;
        const int64_t row = row_begin + j;
        const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x + row * p.hidden);
        const uintptr_t ra = reinterpret_cast<uintptr_t>(p.residual + row * p.hidden);
        uint16_t* xbase = reinterpret_cast<uint16_t*>(xa & ~static_cast<uintptr_t>(15));
        uint16_t* rbase = reinterpret_cast<uint16_t*>(ra & ~static_cast<uintptr_t>(15));
        const int phase = static_cast<int>((xa & 15u) >> 1);
        const int chunks = (phase + p.hidden + 7) >> 3;
        const uint32_t stage = smem_base + static_cast<uint32_t>(s) * p.stage_bytes;
        const int weight_shift = phase - gamma_phase;

        // Pass 1: residual out + sum of squares (kStagedUnroll chunks loaded before use).
        float sumsq = 0.0f;
        for (int k0 = t; k0 < chunks; k0 += kGroupThreads * kStagedUnroll) {
            U32x4 xs[kStagedUnroll], rs[kStagedUnroll];
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    xs[u] = lds_v4(stage + 16u * k);
                    rs[u] = lds_v4(stage + half + 16u * k);
                }
            }
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    U32x4 out;
                    bool full;
                    staged_chunk<false>(xs[u], rs[u], xs[u], 8 * k - phase, p.hidden, 0.0f, sumsq, out, full);
                    store_chunk(rbase + 8 * k, out, full, 8 * k - phase, p.hidden);
                }
            }
        }
        sumsq = warp_sum(sumsq);
        if constexpr (kWarpsPerRow > 1) {
            float* slot = partials + parity_slot * kStagedConsumerWarps + group * kWarpsPerRow;
            if (lane == 0) slot[warp_in_group] = sumsq;
            named_barrier_sync(2 + group, kGroupThreads);
            sumsq = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarpsPerRow; ++w) sumsq += slot[w];
            parity_slot ^= 1;
        }
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, hidden_f) + p.epsilon);

        // Pass 2: normalised output, v recomputed from the staged bytes.
        for (int k0 = t; k0 < chunks; k0 += kGroupThreads * kStagedUnroll) {
            U32x4 xs[kStagedUnroll], rs[kStagedUnroll], ws[kStagedUnroll];
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    xs[u] = lds_v4(stage + 16u * k);
                    rs[u] = lds_v4(stage + half + 16u * k);
                    ws[u] = weight_chunk(weight_base, k, weight_shift, span);
                }
            }
#pragma unroll
            for (int u = 0; u < kStagedUnroll; ++u) {
                const int k = k0 + u * kGroupThreads;
                if (k < chunks) {
                    U32x4 out;
                    bool full;
                    float unused = 0.0f;
                    staged_chunk<true>(xs[u], rs[u], ws[u], 8 * k - phase, p.hidden, inv, unused, out, full);
                    store_chunk(xbase + 8 * k, out, full, 8 * k - phase, p.hidden);
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
// row is read twice.
template <bool kCached>
__global__ void __launch_bounds__(kRowwiseThreads) rmsnorm_rowwise_kernel(
    uint16_t* __restrict__ x, uint16_t* __restrict__ residual, const uint16_t* __restrict__ weight,
    int64_t rows, int hidden, float epsilon) {
    __shared__ float partials[kRowwiseThreads / kWarpSize];
    grid_dependency_wait();
    grid_launch_dependents();
    const float den = static_cast<float>(hidden);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        uint16_t* xr = x + row * hidden;
        uint16_t* rr = residual + row * hidden;
        float sumsq = 0.0f;
        float cache[kCached ? kRowwiseCachedPerThread : 1];
        if constexpr (kCached) {
#pragma unroll
            for (int i = 0; i < kRowwiseCachedPerThread; ++i) {
                const int c = threadIdx.x + i * kRowwiseThreads;
                cache[i] = 0.0f;
                if (c < hidden) {
                    const float v = __fadd_rn(bf16_bits_to_float(xr[c]), bf16_bits_to_float(rr[c]));
                    cache[i] = v;
                    sumsq += __fmul_rn(v, v);
                    rr[c] = float_to_bf16_bits(v);
                }
            }
        } else {
            for (int c = threadIdx.x; c < hidden; c += kRowwiseThreads) {
                const float v = __fadd_rn(bf16_bits_to_float(xr[c]), bf16_bits_to_float(rr[c]));
                sumsq += __fmul_rn(v, v);
            }
        }
        sumsq = block_sum_rowwise(sumsq, partials);
        const float inv = 1.0f / sqrtf(__fdiv_rn(sumsq, den) + epsilon);
        if constexpr (kCached) {
#pragma unroll
            for (int i = 0; i < kRowwiseCachedPerThread; ++i) {
                const int c = threadIdx.x + i * kRowwiseThreads;
                if (c < hidden) {
                    xr[c] = float_to_bf16_bits(
                        __fmul_rn(__fmul_rn(cache[i], inv), bf16_bits_to_float(weight[c])));
                }
            }
        } else {
            for (int c = threadIdx.x; c < hidden; c += kRowwiseThreads) {
                const float v = __fadd_rn(bf16_bits_to_float(xr[c]), bf16_bits_to_float(rr[c]));
                rr[c] = float_to_bf16_bits(v);
                xr[c] = float_to_bf16_bits(__fmul_rn(__fmul_rn(v, inv), bf16_bits_to_float(weight[c])));
            }
        }
    }
}

}  // namespace ipl
