// The fused dense backward at learning_rate != 0 for batches up to 128:
// disldo_backward's scattered non-deferred path (linear_disldo.hpp:625-925),
// with k_backward_update's arithmetic and summation orders (so codes, scales
// and dx are bit-identical to it), arranged to issue fewer instructions and
// keep more warps resident.
//
//  * One warp per input row, one synapse per lane, 32 synapses at a time.
//  * The dy tile [32 synapses][32 samples] reaches shared memory by cp.async
//    16-byte copies, one 128-byte line of dyT per synapse, with no staging
//    registers (pitch 36 floats keeps the lanes = samples reads of the dx
//    pass free of bank conflicts).
//  * x of the row sits in shared memory; dx[b, r] stays in registers for the
//    whole row (lanes = samples, one register per 32-sample block) and is
//    stored once, instead of a read-modify-write per tile.
//  * Whether dy holds an inf or NaN is known per call (a flag written by the
//    |dy| accumulation), not checked per tile.
//  * FP4 codes decode through a 16-entry shared table, and each run of
//    x == 0 samples decays the importance in binary-sized unrolled runs.
//  * The weight history cw (the weight after every sample that can change
//    it) is kept for at most kU2K such samples of a 32-sample block; a block
//    with more is processed as sub-blocks, each followed by the dx pass over
//    its own samples.  dx sums the synapses in stored order with fmaf, each
//    sample with the weight its synapse had after that sample.
//
// Floating point: compiled with --fmad=false like every kernel file here;
// each fused multiply-add is an explicit __fmaf_rn placed as the reference's
// build fuses it.
#include "common.cuh"
#include "kernels.cuh"
#include "update_math.cuh"

namespace sili {

// 2-warp CTAs with 13.5 KB of shared memory each; 14 resident per SM (28
// warps, 72 registers) at scale rank 1-2, 10 at rank 3-4 (their per-synapse
// state needs more registers).  12 weight-history segments: a 32-sample
// block of 20 %-dense inputs almost never needs a second dx pass (8
// segments: 0.356 -> 0.344 ms at config 2)
constexpr int kU2Warps = 2, kU2K = 12, kU2Pitch = 36;
constexpr int u2_min_ctas(int rank) { return rank <= 2 ? 14 : 10; }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem) : "memory");
}
// 16 bytes, or (take == false) 16 zero bytes without reading global memory
// (src-size 0; gmem must still be a valid address)
__device__ __forceinline__ void cp_async16_or_zero(void* smem, const void* gmem, bool take) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gmem), "r"(take ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// One synapse's running state through the batch.
template <int RANK>
struct SynChain {
    float ci, quant, cw, S, cw_orig;
    float cis;       // importance_scale[row] * output_importance_scale[column]
    uint32_t byte;   // the stored FP4BiPacked byte at entry
    int c;           // absolute column
    bool ok;         // finite S and weight, and the row's parameters allow the x == 0 closed form
    float osk[RANK], cg[RANK], cc[RANK];
};

// RESYNC: the DeferredScaleWrite update of the Resync classes (scale rank 1):
// the old true-units step cw += update_cw(g, ci, 1, ...) from
// cw = (cw_orig * vs) * os, component-0 scale sums from the stored code, the
// store deferred (def_cw / def_ci) and the importance statistics taken from
// the true-units ci (linear_disldo.hpp:686-790, 918-923).
template <bool STOCH, bool OST, int RANK, int NB, bool RESYNC>
__global__ void __launch_bounds__(kU2Warps * 32, u2_min_ctas(RANK)) k_backward_update_tiled(LayerView L, const float* __restrict__ xT,
                                                                             const float* __restrict__ dyT, int B,
                                                                             UpdateParams P, float* __restrict__ dxT) {
    __shared__ __align__(16) float dys_s[kU2Warps][32][kU2Pitch];   // [synapse][sample]
    // [segment][synapse]; pitch 36 puts the rows of different segments,
    // which the lanes (samples) of the dx pass read at once, in different banks
    __shared__ __align__(16) float cws_s[kU2Warps][kU2K + 1][kU2Pitch];
    __shared__ float xs_s[kU2Warps][NB * 32];
    __shared__ float ftab[16];   // fp4_decode of every code
    if (threadIdx.x < 16) ftab[threadIdx.x] = fp4_decode(threadIdx.x);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kU2Warps + warp;
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    float* dxr = dxT + r * (int64_t)B;
    if (nnz == 0) {
        for (int b = lane; b < B; b += 32) dxr[b] = 0.0f;
        return;
    }
    float (*dys)[kU2Pitch] = dys_s[warp];
    float (*cws)[kU2Pitch] = cws_s[warp];
    float* xs = xs_s[warp];
    const int f0 = L.rowptr[r];
    const int gnnz = P.row_nnz_g ? P.row_nnz_g[r] : nnz;   // a column shard divides by the global count
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)gnnz) : P.lr;
    const float beta2 = P.beta2;
    const float onem = __fsub_rn(1.0f, beta2);
    const float zterm = __fmul_rn(onem, 0.0f);
    const bool fast_ok = (!P.damp || P.eps > 0.0f) && isfinite(eff_lr) && beta2 >= 0.0f && beta2 <= 1.0f;
    const bool dy_finite = P.dy_flag != nullptr && *P.dy_flag != P.dy_tag;
    const float imp_scale = L.is[r];
    float vsr[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) vsr[k] = L.vs[r * RANK + k];
    const float* xr = xT + r * (int64_t)B;
    const bool vec4 = (B & 3) == 0;
    const int nblk = (B + 31) >> 5;
    float acc[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int t = k * 32 + lane;
        xs[t] = t < B ? __ldg(xr + t) : 0.0f;
        acc[k] = 0.0f;
    }
    __syncwarp();

    double sgs[RANK], sgc[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) { sgs[k] = 0.0; sgc[k] = 0.0; }
    // importance statistics: FP4 magnitudes are multiples of 1/2, so the
    // l1 and l2 changes are exact integers in units of 1/2 and 1/4
    int l1d = 0, l2d = 0;
    bool st_nan = false;
    float mx_new = 0.0f;
    double dsa = 0.0, dsq = 0.0;   // RESYNC: |ci| and ci^2 changes in true units

    auto init = [&](SynChain<RANK>& C, int e, bool valid) {
        C.c = 0;
        C.byte = 0;
        if (valid) {
            C.c = L.abs_cols[f0 + e];
            C.byte = L.val[es + e];
        }
        C.cw_orig = ftab[C.byte >> 4];
#pragma unroll
        for (int k = 0; k < RANK; ++k) C.osk[k] = valid ? L.os[(int64_t)C.c * RANK + k] : 0.0f;
        const float cis = valid ? __fmul_rn(imp_scale, L.ois[C.c]) : 1.0f;
        C.cis = cis;
        float S = 0.0f;
#pragma unroll
        for (int k = 0; k < RANK; ++k) S = __fmaf_rn(vsr[k], C.osk[k], S);
        C.S = S;
        C.ci = __fmul_rn(ftab[C.byte & 15u], cis);
        C.quant = C.cw_orig;
        if (RESYNC) {
            // true units in the reference build's association; an absent
            // lane holds +0 so that it never blocks the x == 0 closed form
            C.S = 1.0f;
            C.cw = valid ? __fmul_rn(__fmul_rn(C.cw_orig, vsr[0]), C.osk[0]) : 0.0f;
            // the closed form leaves cw as is only when cw is not -0
            C.ok = fast_ok && isfinite(S) && isfinite(C.cw_orig) && isfinite(vsr[0]) && isfinite(C.osk[0]) &&
                   !(C.cw == 0.0f && signbit(C.cw));
        } else {
            C.cw = __fmul_rn(C.quant, S);
            C.ok = fast_ok && isfinite(S) && isfinite(C.cw_orig);
        }
#pragma unroll
        for (int k = 0; k < RANK; ++k) { C.cg[k] = 0.0f; C.cc[k] = 0.0f; }
    };
    // one sample that can change the weight (x != 0, or any sample on the
    // general path)
    auto step = [&](SynChain<RANK>& C, float dyv, float iv) {
        const float g = __fmul_rn(dyv, iv);
        const float contrib = __fmul_rn(iv, C.cw_orig);
        C.ci = bounded_ci(C.ci, g, contrib, beta2, onem);
        if (RESYNC) {
            float raw = P.damp ? __fdiv_rn(-g, __fadd_rn(__fsqrt_rn(C.ci), P.eps)) : -g;
            if (raw > 2.0f) raw = 2.0f;
            if (raw < -2.0f) raw = -2.0f;
            C.cw = __fmaf_rn(eff_lr, raw, C.cw);
            const double qo = (double)C.cw_orig * (double)C.osk[0];
            sgs[0] = __fma_rn(qo, (double)g, sgs[0]);
            sgc[0] = __fma_rn(qo, (double)contrib, sgc[0]);
            if (OST) {
                const float qv = __fmul_rn(C.cw_orig, vsr[0]);
                C.cg[0] = __fmaf_rn(qv, g, C.cg[0]);
                C.cc[0] = __fmaf_rn(qv, contrib, C.cc[0]);
            }
            return;
        }
        const float ngS = __fmul_rn(-g, C.S);
        float raw = P.damp ? __fdiv_rn(ngS, __fadd_rn(__fsqrt_rn(C.ci), P.eps)) : ngS;
        if (raw > 2.0f) raw = 2.0f;
        if (raw < -2.0f) raw = -2.0f;
        C.quant = __fmaf_rn(eff_lr, raw, C.quant);
        C.cw = __fmul_rn(C.quant, C.S);
        const float qf = (C.quant == 0.0f) ? 0.1f : C.quant;
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            const double qo = (double)qf * (double)C.osk[k];
            sgs[k] = __fma_rn(qo, (double)g, sgs[k]);
            sgc[k] = __fma_rn(qo, (double)contrib, sgc[k]);
            if (OST) {
                const float qv = __fmul_rn(qf, vsr[k]);
                C.cg[k] = __fmaf_rn(qv, g, C.cg[k]);
                C.cc[k] = __fmaf_rn(qv, contrib, C.cc[k]);
            }
        }
    };
    // dy tile: row l = synapse e0 + l (its n synapses), samples [t0, t0 + nb);
    // rows of absent synapses read as dy = 0
    auto stage = [&](const SynChain<RANK>& C, int n, int t0, int nb) {
        if (vec4) {   // B % 4 == 0: every 16-byte group lies inside or outside [0, nb)
            // groups outside the tile are zero-filled by the copy itself (no
            // branch around the asm, no separate fill of absent rows)
            const int sub = lane >> 3, m4 = (lane & 7) * 4;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int l = q * 4 + sub;
                const int cl = __shfl_sync(0xffffffffu, C.c, l);
                const bool take = l < n && m4 < nb;
                cp_async16_or_zero(&dys[l][m4], take ? dyT + (int64_t)cl * B + t0 + m4 : dyT, take);
            }
            return;
        } else {
            for (int l = 0; l < n; ++l) {
                const int cl = __shfl_sync(0xffffffffu, C.c, l);
                if (lane < nb) cp_async4(&dys[l][lane], dyT + (int64_t)cl * B + t0 + lane);
            }
        }
        for (int l = n; l < 32; ++l) dys[l][lane] = 0.0f;
    };
    auto finish = [&](const SynChain<RANK>& C, int e) {
        if (RESYNC) {
            // deferred: the true-units state, stored by launch_resync_store
            P.def_cw[es + e] = C.cw;
            P.def_ci[es + e] = C.ci;
            const float ao = ftab[C.byte & 15u];
            dsa += fabs((double)C.ci) - fabs((double)ao);
            dsq += (double)C.ci * C.ci - (double)ao * ao;
            mx_new = fmaxf(mx_new, fabsf(C.ci));
            if (OST) {
                atomicAdd(P.colg + (int64_t)C.c * RANK, C.cg[0]);
                atomicAdd(P.colc + (int64_t)C.c * RANK, C.cc[0]);
            }
            return;
        }
        const float imp_st = __fdiv_rn(C.ci, C.cis);
        uint32_t nbyte;
        if (STOCH) {
            const uint64_t vp = (uint64_t)(es + e);
            nbyte = (fp4_quantize_stochastic(C.quant, rng_draw(P.call_key, vp, 0)) << 4) |
                    fp4_quantize_stochastic(imp_st, rng_draw(P.call_key, vp, 1));
        } else {
            nbyte = (fp4_encode(C.quant) << 4) | fp4_encode(imp_st);
        }
        L.val[es + e] = (uint8_t)nbyte;
        if (L.cpack_upd) L.cpack_upd[L.fcpos[f0 + e]] = (int)(((uint32_t)r << 4) | (nbyte >> 4));
        const float an = fabsf(ftab[nbyte & 15u]), ao = fabsf(ftab[C.byte & 15u]);
        if (an != an || ao != ao) {
            st_nan = true;
        } else {
            const int hn = (int)(2.0f * an), ho = (int)(2.0f * ao);
            l1d += hn - ho;
            l2d += hn * hn - ho * ho;
        }
        mx_new = fmaxf(mx_new, an);
        if (OST) {
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                atomicAdd(P.colg + (int64_t)C.c * RANK + k, C.cg[k]);
                atomicAdd(P.colc + (int64_t)C.c * RANK + k, C.cc[k]);
            }
        }
    };

    SynChain<RANK> A;   // synapse e0 + lane
    for (int e0 = 0; e0 < nnz; e0 += 32) {
        const int nA = min(32, nnz - e0);
        init(A, e0 + lane, lane < nA);
        for (int blk = 0; blk < nblk; ++blk) {
            const int t0 = blk * 32, nb = min(32, B - t0);
            float a = acc[0];
#pragma unroll
            for (int k = 1; k < NB; ++k)
                if (blk == k) a = acc[k];
            __syncwarp();   // the previous tile's readers are done
            stage(A, nA, t0, nb);
            const float* xb = xs + t0;
            const unsigned act = __ballot_sync(0xffffffffu, xb[lane] != 0.0f);   // zero beyond B
            cp_async_wait_all();
            __syncwarp();
            const unsigned full = nb >= 32 ? 0xffffffffu : ((1u << nb) - 1u);
            const bool fast = A.ok && A.ci >= 0.0f && A.ci <= 100.0f;
            // samples where some weight may change: x != 0, or all of them
            // when some lane cannot take the x == 0 closed form
            const unsigned bnd = (dy_finite && __all_sync(0xffffffffu, fast)) ? act : full;
            unsigned rem = bnd;
            int j = 0, s0 = 0;
            while (s0 < nb) {
                cws[0][lane] = A.cw;
                int seg = 0, s1 = nb;
                while (true) {
                    const int ja = rem ? (__ffs(rem) - 1) : nb;
                    A.ci = decay_run(A.ci, ja - j, beta2, zterm);   // x == 0 run: only the importance decays
                    j = ja;
                    if (ja >= nb) break;
                    rem &= rem - 1u;
                    const float iv = xb[ja];
                    step(A, dys[lane][ja], iv);
                    ++seg;
                    cws[seg][lane] = A.cw;
                    j = ja + 1;
                    if (seg == kU2K) { s1 = j; break; }
                }
                __syncwarp();
                // dx over this sub-block's samples, synapses in stored order
                if (lane >= s0 && lane < s1) {
                    const unsigned m = bnd & ((2u << lane) - 1u) & ~((1u << s0) - 1u);
                    const float* cwrow = cws[__popc(m)];
                    if (nA == 32) {
#pragma unroll
                        for (int l = 0; l < 32; l += 4) {
                            const float4 w = *reinterpret_cast<const float4*>(cwrow + l);
                            a = __fmaf_rn(w.x, dys[l][lane], a);
                            a = __fmaf_rn(w.y, dys[l + 1][lane], a);
                            a = __fmaf_rn(w.z, dys[l + 2][lane], a);
                            a = __fmaf_rn(w.w, dys[l + 3][lane], a);
                        }
                    } else {
                        for (int l = 0; l < nA; ++l) a = __fmaf_rn(cwrow[l], dys[l][lane], a);
                    }
                }
                __syncwarp();
                s0 = s1;
            }
#pragma unroll
            for (int k = 0; k < NB; ++k)
                if (blk == k) acc[k] = a;
        }
        if (lane < nA) finish(A, e0 + lane);
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int t = k * 32 + lane;
        if (t < B) dxr[t] = acc[k];
    }
    // value_scale update (linear_disldo.hpp:901-925)
#pragma unroll
    for (int k = 0; k < RANK; ++k) {
        sgs[k] = warp_sum(sgs[k]);
        sgc[k] = warp_sum(sgc[k]);
    }
    if (lane == 0) {
        const float scale_eff_lr = __fdiv_rn(P.lr, (float)gnnz);
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            const int64_t i = r * RANK + k;
            if (RESYNC) {
                // component 0 through value_scale[r] / value_scale_importance[r]
                // and the step counter of (r, 0), linear_disldo.hpp:918-923
                if (k == 0 && !P.scale_noop)
                    rmsprop_scale(L.vs + r, L.vsi + r, (float)sgs[0], scale_eff_lr, (float)sgc[0], L.vstep + r * RANK, P);
            } else if (P.row_part) {   // a column shard: its part of the row sums
                P.row_part[2 * i] = sgs[k];
                P.row_part[2 * i + 1] = sgc[k];
            } else if (!P.scale_noop) {
                rmsprop_scale(L.vs + i, L.vsi + i, (float)sgs[k], scale_eff_lr, (float)sgc[k], L.vstep + i, P);
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) mx_new = fmaxf(mx_new, __shfl_xor_sync(0xffffffffu, mx_new, o));
    if (RESYNC) {
        dsa = warp_sum(dsa);
        dsq = warp_sum(dsq);
        if (lane == 0) {
            atomicAdd(P.stats + 0, dsa);
            atomicAdd(P.stats + 1, dsq);
            atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx_new));
        }
        return;
    }
    l1d = warp_sum(l1d);
    l2d = warp_sum(l2d);
    const bool any_nan = __any_sync(0xffffffffu, st_nan);
    if (lane == 0) {
        const double nan = __longlong_as_double(0x7ff8000000000000LL);
        atomicAdd(P.stats + 0, any_nan ? nan : 0.5 * (double)l1d);
        atomicAdd(P.stats + 1, any_nan ? nan : 0.25 * (double)l2d);
        atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx_new));
    }
}

template <bool STOCH, bool OST, int RANK, bool RESYNC = false>
static void launch_tiled_nb(const LayerView& L, const float* xT, const float* dyT, int B, const UpdateParams& P,
                            float* dxT, cudaStream_t s) {
    const unsigned g = (unsigned)((L.n_in + kU2Warps - 1) / kU2Warps);
    if (B <= 64) k_backward_update_tiled<STOCH, OST, RANK, 2, RESYNC><<<g, kU2Warps * 32, 0, s>>>(L, xT, dyT, B, P, dxT);
    else k_backward_update_tiled<STOCH, OST, RANK, 4, RESYNC><<<g, kU2Warps * 32, 0, s>>>(L, xT, dyT, B, P, dxT);
}

template <bool STOCH, bool OST>
static void launch_tiled_rank(const LayerView& L, const float* xT, const float* dyT, int B, const UpdateParams& P,
                              float* dxT, cudaStream_t s) {
    if (P.resync) {   // scale rank 1 only (the host enforces it)
        launch_tiled_nb<STOCH, OST, 1, true>(L, xT, dyT, B, P, dxT, s);
        return;
    }
    switch (L.rank) {
    case 1: launch_tiled_nb<STOCH, OST, 1>(L, xT, dyT, B, P, dxT, s); break;
    case 2: launch_tiled_nb<STOCH, OST, 2>(L, xT, dyT, B, P, dxT, s); break;
    case 3: launch_tiled_nb<STOCH, OST, 3>(L, xT, dyT, B, P, dxT, s); break;
    default: launch_tiled_nb<STOCH, OST, 4>(L, xT, dyT, B, P, dxT, s); break;
    }
}

void launch_backward_update_tiled(const LayerView& L, const float* xT, const float* dyT, int B, const UpdateParams& P,
                                  float* dxT, cudaStream_t s) {
    if (L.n_in == 0) return;
    if (P.stochastic) {
        if (P.os_trainable) launch_tiled_rank<true, true>(L, xT, dyT, B, P, dxT, s);
        else launch_tiled_rank<true, false>(L, xT, dyT, B, P, dxT, s);
    } else {
        if (P.os_trainable) launch_tiled_rank<false, true>(L, xT, dyT, B, P, dxT, s);
        else launch_tiled_rank<false, false>(L, xT, dyT, B, P, dxT, s);
    }
    count_launch();
}

// The deferred stores of a Resync update (linear_disldo.hpp:2083-2112): every
// synapse of a row the update visited, under the scales now in effect --
// w = cw / (vs * os), imp = ci / (is * ois) -- stochastically or to nearest,
// with the same per-position draws as the immediate store.  A warp per row.
template <bool STOCH>
__global__ void k_resync_store(LayerView L, UpdateParams P) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    const int f0 = L.rowptr[r];
    const float vs0 = L.vs[r * L.rank], isr = L.is[r];
    for (int e = threadIdx.x & 31; e < nnz; e += 32) {
        const int c = L.abs_cols[f0 + e];
        const float w = __fdiv_rn(P.def_cw[es + e], __fmul_rn(vs0, L.os[(int64_t)c * L.rank]));
        const float imp = __fdiv_rn(P.def_ci[es + e], __fmul_rn(isr, L.ois[c]));
        uint32_t nbyte;
        if (STOCH) {
            const uint64_t vp = (uint64_t)(es + e);
            nbyte = (fp4_quantize_stochastic(w, rng_draw(P.call_key, vp, 0)) << 4) |
                    fp4_quantize_stochastic(imp, rng_draw(P.call_key, vp, 1));
        } else {
            nbyte = (fp4_encode(w) << 4) | fp4_encode(imp);
        }
        L.val[es + e] = (uint8_t)nbyte;
        if (L.cpack_upd) L.cpack_upd[L.fcpos[f0 + e]] = (int)(((uint32_t)r << 4) | (nbyte >> 4));
    }
}

void launch_resync_store(const LayerView& L, const UpdateParams& P, cudaStream_t s) {
    if (L.n_in == 0) return;
    const unsigned g = (unsigned)((L.n_in + 7) / 8);
    if (P.stochastic) k_resync_store<true><<<g, 256, 0, s>>>(L, P);
    else k_resync_store<false><<<g, 256, 0, s>>>(L, P);
    count_launch();
}

}  // namespace sili
