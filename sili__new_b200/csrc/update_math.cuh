// Device math shared by the scattered and block4 update kernels: the scale
// optimiser and the bounded per-synapse importance update, with the
// reference build's fused-multiply-add placement.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace sili {

// ── scale optimiser (RMSpropScalePolicy::update, delta_csr_types.hpp:445-466) ──
__device__ __forceinline__ float bias_pow(const UpdateParams& P, uint32_t step) {
    if ((int)step < P.pow_n) return P.pow_tab[step];
    return powf(P.beta2, (float)step);   // beyond the table powf(beta2, s) < 2^-25: 1 - p == 1
}

__device__ __forceinline__ void rmsprop_scale(float* scale, float* state, float g, float lr, float c,
                                              uint32_t* step, const UpdateParams& P) {
    if (!isfinite(g) || !isfinite(c)) return;
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float ns = __fmaf_rn(P.beta2, *state, __fmul_rn(onem, __fmaf_rn(g, g, __fmul_rn(c, c))));
    if (!isfinite(ns)) return;
    float hat = ns;
    const uint32_t st = *step + 1u;
    *step = st;
    const float bc = __fsub_rn(1.0f, bias_pow(P, st));
    if (bc > 0.0f) hat = __fdiv_rn(ns, bc);
    if (!isfinite(hat)) return;
    const float nsc = __fsub_rn(*scale, __fdiv_rn(__fmul_rn(lr, g), __fadd_rn(__fsqrt_rn(hat), P.eps)));
    if (!isfinite(nsc)) return;
    *state = ns;
    *scale = nsc;
}

// BoundedRMSpropSynapsePolicy::update_ci (delta_csr_types.hpp:707-713) at the
// production arguments min_decay_frac = 0, max_ci = 100 (cpu_backend.cpp:518-525).
__device__ __forceinline__ float bounded_ci(float ci, float g, float contrib, float beta2, float onem) {
    const float ema = __fmaf_rn(beta2, ci, __fmul_rn(onem, __fmaf_rn(g, g, __fmul_rn(contrib, contrib))));
    const float fl = __fmul_rn(0.0f, ci);
    float r = (ema < fl) ? fl : ema;
    return (100.0f < r) ? 100.0f : r;
}

// n steps of the x == 0 closed form of the importance update (ci = fma(beta2,
// ci, zterm), n < 64), as n sequential fmas in binary-sized runs: the runs
// between a row's non-zero inputs are short and vary, and warp-uniform tests
// of n's bits cost less than a counted loop
__device__ __forceinline__ float decay_run(float ci, int n, float beta2, float zterm) {
    if (n & 32) {
#pragma unroll
        for (int u = 0; u < 32; ++u) ci = __fmaf_rn(beta2, ci, zterm);
    }
    if (n & 16) {
#pragma unroll
        for (int u = 0; u < 16; ++u) ci = __fmaf_rn(beta2, ci, zterm);
    }
    if (n & 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) ci = __fmaf_rn(beta2, ci, zterm);
    }
    if (n & 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) ci = __fmaf_rn(beta2, ci, zterm);
    }
    if (n & 2) {
        ci = __fmaf_rn(beta2, ci, zterm);
        ci = __fmaf_rn(beta2, ci, zterm);
    }
    if (n & 1) ci = __fmaf_rn(beta2, ci, zterm);
    return ci;
}

}  // namespace sili
