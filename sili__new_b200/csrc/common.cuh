// Device-side building blocks shared by every kernel of sili_b200.
//
// FP4 codec: restated from the reference's bit arithmetic
// (sili/lib/headers/fp4quant.hpp:68-121 decode/encode, :238-273 stochastic),
// not CUDA's e2m1 conversion: the reference's table puts NaN at code 8 and
// rounds midpoints up in magnitude, which the hardware conversion does not.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sili {

constexpr int kWarp = 32;

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

// fp4_decode_bits (fp4quant.hpp:68-84): equals FP4_TABLE, code 8 -> NaN.
__device__ __forceinline__ float fp4_decode(uint32_t code) {
    const uint32_t s = (code >> 3) & 1u, e = (code >> 1) & 3u, m = code & 1u;
    uint32_t bits;
    if (e == 0) bits = m ? (0x3F000000u | (s << 31)) : (s ? 0x7FC00000u : 0u);
    else bits = (s << 31) | ((e + 126u) << 23) | (m << 22);
    return u2f(bits);
}

// fp4_encode_bits (fp4quant.hpp:86-121): nearest, midpoints up in magnitude,
// saturating at 6, NaN -> 0, never code 8.
__device__ __forceinline__ uint32_t fp4_encode(float v) {
    const uint32_t bits = f2u(v), sign = bits >> 31, a = bits & 0x7FFFFFFFu;
    uint32_t mag;
    if (a > 0x7F800000u) return 0;
    if (a < 0x3E800000u) mag = 0;
    else if (a < 0x3F400000u) mag = 1;
    else if (a < 0x3F800000u) mag = 2;
    else {
        uint32_t r = a + (1u << 21);
        r = r > 0x40C00000u ? 0x40C00000u : r;
        mag = ((((r >> 23) & 0xFFu) - 126u) << 1) | ((r >> 22) & 1u);
    }
    return mag == 0 ? 0u : ((sign << 3) | mag);
}

// fp4_quantize_stochastic (fp4quant.hpp:238-273) with the 64-bit draw passed
// in: top 24 bits give the uniform for |v| < 1, low 22 bits the dither above.
// The uniform (24-bit integer) * 2^-24 is exact in float.
__device__ __forceinline__ uint32_t fp4_quantize_stochastic(float v, uint64_t r) {
    const uint32_t bits = f2u(v), sign = bits >> 31, a = bits & 0x7FFFFFFFu;
    uint32_t mag;
    if (a > 0x7F800000u) return 0;
    if (a >= 0x40C00000u) mag = 7;
    else if (a < 0x3F000000u) {
        const float p = u2f(a) * 2.0f;
        const float u = (float)(uint32_t)(r >> 40) * 0x1p-24f;
        mag = (u < p) ? 1u : 0u;
    } else if (a < 0x3F800000u) {
        const float p = __fsub_rn(u2f(a) * 2.0f, 1.0f);
        const float u = (float)(uint32_t)(r >> 40) * 0x1p-24f;
        mag = (u < p) ? 2u : 1u;
    } else {
        uint32_t rr = a + (uint32_t)(r & 0x3FFFFFu);
        rr = rr > 0x40C00000u ? 0x40C00000u : rr;
        mag = ((((rr >> 23) & 0xFFu) - 126u) << 1) | ((rr >> 22) & 1u);
    }
    return mag == 0 ? 0u : ((sign << 3) | mag);
}

// Counter-based draw for stochastic rounding: splitmix64's finaliser over
// (seed, backward-call counter, element position, lane 0 = weight /
// 1 = importance).  Independent per synapse, so the update kernel needs no
// ordered RNG stream; the CPU oracle uses the identical function.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t rng_draw(uint64_t call_key, uint64_t elem, uint32_t lane) {
    return mix64(call_key ^ (elem * 2u + lane) * 0xD1B54A32D192ED03ULL);
}
// call_key = mix64(seed ^ call * golden), computed once per launch on the host.
inline uint64_t host_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Inclusive prefix sum across the warp.
__device__ __forceinline__ uint32_t warp_inclusive_scan(uint32_t v) {
    const unsigned lane = lane_id();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= (unsigned)o) v += t;
    }
    return v;
}

// Warp-cooperative ULEB128 decoder for one delta-CSR row
// (format: delta_csr_types.hpp:211-241; first delta is the absolute column).
// Each call consumes the next window of 32 bytes starting at a value
// boundary, decodes every value that ends inside it (a value is at most 5
// bytes), prefix-sums the deltas onto the running column and hands value j of
// the window to lane j.  Returns how many values it produced (<= 32).
struct RowDecoder {
    int64_t pos, end;
    uint32_t col;
};

__device__ __forceinline__ int warp_decode_window(const uint8_t* __restrict__ buf, RowDecoder& d,
                                                  uint32_t* stage /* 32 words per warp */,
                                                  uint32_t& out_col) {
    const unsigned lane = lane_id();
    const int64_t p = d.pos + lane;
    const bool in = p < d.end;
    const uint32_t byte = in ? (uint32_t)__ldg(buf + p) : 0x80u;
    const unsigned term = __ballot_sync(0xffffffffu, in && !(byte & 0x80u));
    const int count = __popc(term);
    const unsigned below = term & ((1u << lane) - 1u);
    const int start = below ? (32 - __clz(below)) : 0;
    const int k = (int)lane - start;                       // byte index inside its value
    const uint32_t contrib = (k < 5) ? ((byte & 0x7Fu) << (7 * k)) : 0u;
    uint32_t v = contrib;
#pragma unroll
    for (int s = 1; s <= 4; ++s) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, contrib, s);
        if ((int)lane - s >= start) v |= t;
    }
    const bool is_end = (term >> lane) & 1u;
    const uint32_t inc = warp_inclusive_scan(is_end ? v : 0u);
    const uint32_t col_here = d.col + inc;
    if (is_end) stage[__popc(below)] = col_here;
    __syncwarp();
    out_col = (lane < (unsigned)count) ? stage[lane] : 0u;
    if (count > 0) {
        const int last = 31 - __clz(term);
        d.pos += last + 1;
        d.col = __shfl_sync(0xffffffffu, col_here, last);
    } else {
        d.pos = d.end;
    }
    __syncwarp();
    return count;
}

}  // namespace sili
