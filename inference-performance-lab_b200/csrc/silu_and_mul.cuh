// SiLU-and-multiply for sm_100a.
//
// out[r, c] = bf16(silu(g) * u), g = fp32(in[r, c]), u = fp32(in[r, I + c]), silu(g) = g / (1 + e^-g)
// (reference: csrc/silu_and_mul_kernel.cu:30-81; oracle
// src/inference_performance_lab/kernels/reference.py:26-35).
//
// * silu_vector_kernel<kBytes, kUnroll> - the aligned path. A 1-D grid over "packs" (kBytes of
//   output = kBytes/2 elements, with the matching gate and up packs of the input). kBytes is 32
//   (256-bit ld/st, sm_100) when the width and both pointers allow it, else 16. Each thread
//   issues kUnroll pack loads before consuming any, so a single wave of CTAs keeps the whole
//   working set in flight. Row/column of a pack come from a multiply-shift division by the
//   packs-per-row constant (Granlund & Montgomery, "Division by Invariant Integers using
//   Multiplication", PLDI 1994), computed once on the host.
// * silu_wave_kernel - 16-byte packs in one wave of 1024-thread CTAs, for launches of about one
//   wave (see its comment).
// * silu_scalar_kernel - any width, any alignment: one element per thread, coalesced 2-byte
//   accesses over the flattened output.
#pragma once

#include "ipl_common.cuh"

namespace ipl {

constexpr int kSiluThreads = 256;

// n / d for 32-bit n with a precomputed (multiplier, shift): q = (umulhi(n, m) + n) >> s.
struct FastDiv32 {
    uint32_t divisor;
    uint32_t multiplier;
    uint32_t shift;
};

inline FastDiv32 make_fast_div32(uint32_t d) {
    FastDiv32 f;
    f.divisor = d;
    uint32_t l = 0;
    while ((uint64_t{1} << l) < d) ++l;  // l = ceil(log2 d)
    f.shift = l;
    // m = floor(2^32 * (2^l - d) / d) + 1, fits in 32 bits for d >= 1.
    f.multiplier = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
    return f;
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv32& f) {
    const uint64_t t = static_cast<uint64_t>(__umulhi(n, f.multiplier)) + n;
    return static_cast<uint32_t>(t >> f.shift);
}

__device__ __forceinline__ float silu_mul(float gate, float up) {
    // gate / (1 + e^-gate) with the hardware exponential and fast division (a few ulp in fp32,
    // far below the bf16 rounding of the result). For gate < -87.3 the denominator exceeds
    // 2^126 and the quotient is 0 (the exact value is below 1e-36); gate = -inf gives NaN and
    // gate = +inf gives +inf, as in the reference.
    return __fmul_rn(__fdividef(gate, __fadd_rn(1.0f, __expf(-gate))), up);
}

template <int kWords>
__device__ __forceinline__ void silu_words(const uint32_t* g, const uint32_t* u, uint32_t* o) {
#pragma unroll
    for (int i = 0; i < kWords; ++i) {
        o[i] = pack_bf16x2(silu_mul(bf16_lo(g[i]), bf16_lo(u[i])), silu_mul(bf16_hi(g[i]), bf16_hi(u[i])));
    }
}

struct SiluVectorParams {
    uint16_t* out;
    const uint16_t* in;
    int64_t intermediate;   // I
    uint32_t total_packs;   // rows * packs_per_row
    FastDiv32 packs_per_row;
};

template <int kBytes, int kUnroll>
__global__ void __launch_bounds__(kSiluThreads) silu_vector_kernel(const SiluVectorParams p) {
    constexpr int kElems = kBytes / 2;
    constexpr int kWords = kBytes / 4;
    using Vec = typename std::conditional<kBytes == 32, U32x8, U32x4>::type;
    // Pack indices run in 64 bits: total_packs may be any 32-bit count, and base + stride * kUnroll
    // must not wrap past it. A pack below total_packs fits 32 bits for the division.
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    const uint64_t first = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    // While the previous kernel in the stream drains, ask L2 for this thread's first packs of
    // gate and up (a prefetch only warms L2, where every SM's accesses meet, so the loads after
    // the wait still see the previous kernel's writes).
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
        const uint64_t pack = first + k * stride;
        if (pack < p.total_packs) {
            const uint32_t row = fast_div(static_cast<uint32_t>(pack), p.packs_per_row);
            const uint32_t col = static_cast<uint32_t>(pack) - row * p.packs_per_row.divisor;
            const uint16_t* gate = p.in + static_cast<int64_t>(row) * 2 * p.intermediate + int64_t{col} * kElems;
            prefetch_l2(gate);
            prefetch_l2(gate + p.intermediate);
        }
    }
    grid_dependency_wait();
    grid_launch_dependents();

    for (uint64_t base = first; base < p.total_packs; base += stride * kUnroll) {
        Vec gate[kUnroll], up[kUnroll];
        int64_t out_off[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
            const uint64_t pack = base + k * stride;
            out_off[k] = -1;
            if (pack < p.total_packs) {
                const uint32_t row = fast_div(static_cast<uint32_t>(pack), p.packs_per_row);
                const uint32_t col = static_cast<uint32_t>(pack) - row * p.packs_per_row.divisor;
                const int64_t in_off = static_cast<int64_t>(row) * 2 * p.intermediate + int64_t{col} * kElems;
                out_off[k] = static_cast<int64_t>(row) * p.intermediate + int64_t{col} * kElems;
                if constexpr (kBytes == 32) {
                    gate[k] = ld_stream_v8(p.in + in_off);
                    up[k] = ld_stream_v8(p.in + in_off + p.intermediate);
                } else {
                    gate[k] = ld_stream_v4(p.in + in_off);
                    up[k] = ld_stream_v4(p.in + in_off + p.intermediate);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
            if (out_off[k] >= 0) {
                Vec o;
                silu_words<kWords>(gate[k].v, up[k].v, o.v);
                if constexpr (kBytes == 32) {
                    st_v8(p.out + out_off[k], o);
                } else {
                    st_v4(p.out + out_off[k], o);
                }
            }
        }
    }
}

// silu_wave_kernel - one 16-byte pack per thread, in a single wave of 1024-thread CTAs (two per
// SM), for launches whose 16-byte packs fill more than half of the SMs' thread slots and no more
// than all of them (e.g. [128, 37888]: 303,104 packs over 148 x 2048 threads). Against one 32-byte
// pack per thread in 256-thread CTAs, twice the loads in flight for the same bytes and a quarter
// of the CTAs to launch; while the previous kernel in the stream drains, each warp asks L2 for its
// 512 contiguous bytes of gate and of up with one bulk prefetch apiece (a line prefetch per thread
// where the warp's packs cross a row's end or the launch's end). Chained on B200, this shape runs
// 2.91 us a launch against 3.33 us for the 32-byte kernel.
constexpr int kSiluWaveThreads = 1024;

__global__ void __launch_bounds__(kSiluWaveThreads, 2) silu_wave_kernel(const SiluVectorParams p) {
    constexpr int kElems = 8;
    // grid * 1024 <= SMs * 2048 packs, far inside 32 bits.
    const uint32_t pack = blockIdx.x * kSiluWaveThreads + threadIdx.x;
    const bool active = pack < p.total_packs;
    int64_t in_off = 0, out_off = 0;
    if (active) {
        const uint32_t row = fast_div(pack, p.packs_per_row);
        const uint32_t col = pack - row * p.packs_per_row.divisor;
        in_off = static_cast<int64_t>(row) * 2 * p.intermediate + int64_t{col} * kElems;
        out_off = static_cast<int64_t>(row) * p.intermediate + int64_t{col} * kElems;
    }
    // Every thread of the warp reaches the shuffle and the vote (no thread has left).
    const uint32_t lane = threadIdx.x & 31u;
    const int64_t first = __shfl_sync(0xffffffffu, in_off, 0);
    const bool contiguous = __all_sync(0xffffffffu, active && in_off == first + int64_t{lane} * kElems);
    if (contiguous) {
        if (lane == 0) {
            bulk_prefetch_l2(p.in + first, 32 * 16);
            bulk_prefetch_l2(p.in + first + p.intermediate, 32 * 16);
        }
    } else if (active) {
        prefetch_l2(p.in + in_off);
        prefetch_l2(p.in + in_off + p.intermediate);
    }
    grid_dependency_wait();
    grid_launch_dependents();
    if (active) {
        const U32x4 gate = ld_stream_v4(p.in + in_off);
        const U32x4 up = ld_stream_v4(p.in + in_off + p.intermediate);
        U32x4 o;
        silu_words<4>(gate.v, up.v, o.v);
        st_v4(p.out + out_off, o);
    }
}

__global__ void __launch_bounds__(kSiluThreads) silu_scalar_kernel(uint16_t* __restrict__ out,
                                                                   const uint16_t* __restrict__ in,
                                                                   int64_t rows, int64_t intermediate) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int64_t total = rows * intermediate;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
        const int64_t row = e / intermediate;
        const int64_t col = e - row * intermediate;
        const uint16_t* g = in + row * 2 * intermediate + col;
        out[e] = float_to_bf16_bits(silu_mul(bf16_bits_to_float(g[0]), bf16_bits_to_float(g[intermediate])));
    }
}

}  // namespace ipl
