// Compute kernels of the FP4 delta-CSR sparse layer: forward, dense backward
// (dx and the fused per-synapse update), sparse-gradient backward and the
// row/column scale optimisers.
//
// Floating point: this file is compiled with --fmad=false; every fused
// multiply-add below is an explicit __fmaf_rn, placed where the reference's
// own build fuses (the CPU oracle uses the same placement and is pinned
// bit-exact against the reference), so codes and scales match bit for bit.
#include "common.cuh"
#include "kernels.cuh"
#include "update_math.cuh"

#include <atomic>
#include <cmath>

namespace sili {

static std::atomic<long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

// ── layout helpers ─────────────────────────────────────────────────────────
__global__ void k_transpose(const float* __restrict__ in, float* __restrict__ out, int64_t R, int64_t C) {
    __shared__ float tile[32][33];
    const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int64_t r = r0 + j, c = c0 + threadIdx.x;
        if (r < R && c < C) tile[j][threadIdx.x] = in[r * C + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int64_t c = c0 + j, r = r0 + threadIdx.x;
        if (r < R && c < C) out[c * R + r] = tile[threadIdx.x][j];
    }
}

void launch_transpose(const float* in, float* out, int64_t R, int64_t C, cudaStream_t s) {
    if (R == 0 || C == 0) return;
    dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32)), block(32, 8);
    k_transpose<<<grid, block, 0, s>>>(in, out, R, C); count_launch();
}

// A single row [1, C] is its own transpose: copy it and append the zero row
// (one element) in one launch.
__global__ void k_copy_pad(const float* __restrict__ in, float* __restrict__ out, int64_t C) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < C) out[i] = in[i];
    else if (i == C) out[i] = 0.0f;
}
void launch_copy_pad(const float* in, float* out, int64_t C, cudaStream_t s) {
    k_copy_pad<<<(unsigned)((C + 1 + 255) / 256), 256, 0, s>>>(in, out, C); count_launch();
}

// neuron_*_accum[j] += |x[b, j]| for b ascending (linear_disldo.hpp:515-520).
// With a flag pointer, a thread that meets an inf or NaN stores `tag` there
// (the update kernel reads it to choose its exact general path for the call).
__global__ void k_accum_abs(const float* __restrict__ x, float* __restrict__ acc, int B, int64_t n,
                            unsigned long long* __restrict__ nonfinite, unsigned long long tag) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float a = acc[j];
    const bool was_finite = isfinite(a);
    for (int b = 0; b < B; ++b) a = __fadd_rn(a, fabsf(x[(int64_t)b * n + j]));
    acc[j] = a;
    if (!nonfinite || isfinite(a)) return;   // a finite sum of |x| has only finite terms
    // a non-finite sum: an inf or NaN term, a sum that was already non-finite,
    // or an overflow of finite terms (which only costs the update its fast path)
    bool bad = was_finite;
    for (int b = 0; b < B && !bad; ++b) bad = !(fabsf(x[(int64_t)b * n + j]) <= 3.402823466e38f);
    if (bad) *nonfinite = tag;
}
void launch_accum_abs(const float* x, float* acc, int B, int64_t n, cudaStream_t s, unsigned long long* nonfinite,
                      unsigned long long tag) {
    if (n == 0 || B == 0) return;
    k_accum_abs<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, acc, B, n, nonfinite, tag); count_launch();
}

// The transpose of dy [B, n] into dyT [n, B] and, on the way, the |dy|
// accumulation and non-finite flag of k_accum_abs (same order: b ascending
// per column): one read of dy instead of two.  A CTA owns 32 columns and
// walks the samples in 32-row tiles; one thread per column carries the sum.
__global__ void k_transpose_accum(const float* __restrict__ in, float* __restrict__ out, int64_t R, int64_t C,
                                  float* __restrict__ acc, unsigned long long* __restrict__ nonfinite,
                                  unsigned long long tag) {
    __shared__ float tile[32][33];
    const int64_t c0 = (int64_t)blockIdx.x * 32;
    const int64_t cs = c0 + threadIdx.x;   // the column this thread sums (threadIdx.y == 0)
    const bool summer = threadIdx.y == 0 && cs < C;
    float a = summer ? acc[cs] : 0.0f;
    const bool was_finite = isfinite(a);
    bool term_bad = false;
    for (int64_t r0 = 0; r0 < R; r0 += 32) {
        __syncthreads();   // the previous tile's readers are done
        for (int j = threadIdx.y; j < 32; j += 8) {
            const int64_t r = r0 + j, c = c0 + threadIdx.x;
            if (r < R && c < C) tile[j][threadIdx.x] = in[r * C + c];
        }
        __syncthreads();
        if (summer) {
            const int nr = (int)(R - r0 < 32 ? R - r0 : 32);
            for (int j = 0; j < nr; ++j) {
                const float v = fabsf(tile[j][threadIdx.x]);
                a = __fadd_rn(a, v);
                term_bad |= !(v <= 3.402823466e38f);
            }
        }
        for (int j = threadIdx.y; j < 32; j += 8) {
            const int64_t c = c0 + j, r = r0 + threadIdx.x;
            if (r < R && c < C) out[c * R + r] = tile[threadIdx.x][j];
        }
    }
    if (!summer) return;
    acc[cs] = a;
    // as k_accum_abs: a non-finite sum that this call made non-finite, or
    // one with an inf or NaN term
    if (nonfinite && !isfinite(a) && (was_finite || term_bad)) *nonfinite = tag;
}
void launch_transpose_accum(const float* in, float* out, int64_t R, int64_t C, float* acc,
                            unsigned long long* nonfinite, unsigned long long tag, cudaStream_t s) {
    if (R == 0 || C == 0) return;
    k_transpose_accum<<<(unsigned)((C + 31) / 32), dim3(32, 8), 0, s>>>(in, out, R, C, acc, nonfinite, tag);
    count_launch();
}

// Same accumulation from the transposed input xT [n, B].
__global__ void k_accum_abs_t(const float* __restrict__ xT, float* __restrict__ acc, int B, int64_t n) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float a = acc[j];
    const float* row = xT + j * (int64_t)B;
    for (int b = 0; b < B; ++b) a = __fadd_rn(a, fabsf(row[b]));
    acc[j] = a;
}
void launch_accum_abs_t(const float* xT, float* acc, int B, int64_t n, cudaStream_t s) {
    if (n == 0 || B == 0) return;
    k_accum_abs_t<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(xT, acc, B, n); count_launch();
}

// ── forward ────────────────────────────────────────────────────────────────
// Output-stationary gather over the CSC shadow: one warp per output column,
// lanes over batch samples, rows visited in ascending order.  This is the
// reference's single-thread summation order, so y is bit-identical to
// disldo_forward (linear_disldo.hpp:93-120: w = stored*S(r,c); y += w*x,
// x == 0 skipped) or, with SPARSE, to sisldo_forward's (w*x)*(vs*os).
template <int NB, bool SPARSE>
__global__ void __launch_bounds__(256) k_forward_gather(LayerView L, const float* __restrict__ xT, int B,
                                                        float* __restrict__ y) {
    __shared__ float ys[8][32 * NB + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c0 = (int64_t)blockIdx.x * 8, c = c0 + warp;
    const int b0 = blockIdx.y * 32 * NB;
    float acc[NB];
#pragma unroll
    for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
    if (c < L.n_out) {
        float osk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) osk[k] = k < L.rank ? L.os[c * L.rank + k] : 0.0f;
        const int k0 = L.colptr[c], k1 = L.colptr[c + 1];
        for (int kb = k0; kb < k1; kb += 32) {
            const int kk = kb + lane;
            int r = 0;
            float w = 0.0f, cs = 0.0f;
            if (kk < k1) r = L.crow[kk];   // CSC padding: the zero input row, weight 0
            if (kk < k1 && L.cvpos[kk] >= 0) {
                const float wq = fp4_decode(L.val[L.cvpos[kk]] >> 4);
                if (SPARSE) {
                    w = wq;
                    cs = __fmul_rn(L.vs[(int64_t)r * L.rank], osk[0]);
                } else {
                    float sc = 0.0f;
                    for (int k = 0; k < L.rank; ++k) sc = __fmaf_rn(L.vs[(int64_t)r * L.rank + k], osk[k], sc);
                    w = __fmul_rn(wq, sc);
                }
            }
            const int n = min(32, k1 - kb);
            for (int j0 = 0; j0 < n; j0 += 8) {
                // issue 8 synapses' x loads first, then accumulate in row order
                float wj[8], csj[8], xv[8][NB];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int jj = (j0 + u) & 31;
                    wj[u] = __shfl_sync(0xffffffffu, w, jj);
                    const int rj = __shfl_sync(0xffffffffu, r, jj);
                    csj[u] = SPARSE ? __shfl_sync(0xffffffffu, cs, jj) : 0.0f;
                    const float* xr = xT + (int64_t)rj * B;
#pragma unroll
                    for (int t = 0; t < NB; ++t) {
                        const int b = b0 + t * 32 + lane;
                        xv[u][t] = (j0 + u < n && b < B) ? __ldg(xr + b) : 0.0f;
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
#pragma unroll
                    for (int t = 0; t < NB; ++t) {
                        if (xv[u][t] != 0.0f)
                            acc[t] = SPARSE ? __fadd_rn(acc[t], __fmul_rn(__fmul_rn(wj[u], xv[u][t]), csj[u]))
                                            : __fmaf_rn(wj[u], xv[u][t], acc[t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NB; ++t) ys[warp][t * 32 + lane] = acc[t];
    __syncthreads();
    for (int i = threadIdx.x; i < 8 * 32 * NB; i += 256) {
        const int w = i & 7, bl = i >> 3;
        const int b = b0 + bl;
        const int64_t cc = c0 + w;
        if (b < B && cc < L.n_out) y[(int64_t)b * L.n_out + cc] = ys[w][bl];
    }
}

// Vectorised gather for batches that are a multiple of 4: each lane carries 4
// samples (one float4 of the transposed input), LPC lanes cover 4*LPC
// samples of one column and a warp works 32/LPC columns at once.  Every
// (column, sample) keeps its own fma chain over the column's synapses in
// ascending row -- the reference's single-thread order -- so the result is
// bit-exact.  Columns come padded to a multiple of 8 entries whose row is the
// all-zero input row n_in and whose weight is 0, so the inner loop has no
// bounds tests.  The reference skips zero inputs; for a finite weight
// fma(w, 0, acc) == acc (acc, built from +0, is never -0), so the skip is
// only applied in a chunk holding a non-finite weight or scale.
template <int LPC, bool SPARSE>
__global__ void __launch_bounds__(256) k_forward_vec(LayerView L, const float* __restrict__ xT, int B,
                                                     float* __restrict__ y) {
    constexpr int CPW = 32 / LPC;          // columns per warp
    constexpr int CPB = 8 * CPW;           // columns per block
    constexpr int SPB = 4 * LPC;           // samples per block
    __shared__ float ys[CPB][SPB + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPC, lid = lane % LPC;
    const int gbase = grp * LPC;
    const int64_t cb = (int64_t)blockIdx.x * CPB;
    const int64_t c = cb + warp * CPW + grp;
    const int b0 = blockIdx.y * SPB;
    const int bl = b0 + lid * 4;
    const bool bok = bl < B;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int k0 = 0, len = 0;
    float osk[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c < L.n_out) {
        k0 = L.colptr[c];
        len = L.colptr[c + 1] - k0;
#pragma unroll
        for (int k = 0; k < 4; ++k) osk[k] = k < L.rank ? L.os[c * L.rank + k] : 0.0f;
    }
    int maxlen = len;
#pragma unroll
    for (int o = LPC; o < 32; o <<= 1) maxlen = max(maxlen, __shfl_xor_sync(0xffffffffu, maxlen, o));
    // lanes past the batch read the zero row: every lane stays on the fast path
    const float* xb = bok ? xT + bl : xT + (int64_t)L.n_in * B;
    const int omask = bok ? -1 : 0;
    for (int kb = 0; kb < maxlen; kb += 8) {
        // lanes lid < 8 load the chunk's metadata: row offset and weight
        int off = L.n_in * B;                  // zero row
        float w = 0.0f, cs = 0.0f;
        if (lid < 8 && kb < len) {
            const int kk = k0 + kb + lid;
            // packed word (row << 4 | weight code; padding = row n_in) when
            // present, else the row and value position separately
            int r;
            uint32_t code;
            if (L.cpack) {
                const int pk = L.cpack[kk];
                r = pk >> 4;
                code = (uint32_t)pk & 15u;
            } else {
                const int vp = L.cvpos[kk];
                r = vp >= 0 ? L.crow[kk] : L.n_in;
                code = vp >= 0 ? (uint32_t)(L.val[vp] >> 4) : 0u;
            }
            if (r < L.n_in) {
                off = r * B;
                const float wq = fp4_decode(code);
                if (SPARSE) {
                    w = wq;
                    cs = __fmul_rn(L.vs[(int64_t)r * L.rank], osk[0]);
                } else {
                    float sc = 0.0f;
                    for (int k = 0; k < L.rank; ++k) sc = __fmaf_rn(L.vs[(int64_t)r * L.rank + k], osk[k], sc);
                    w = __fmul_rn(wq, sc);
                }
            }
        }
        const bool careful = __any_sync(0xffffffffu, !isfinite(w) || (SPARSE && !isfinite(cs)));
        float4 xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int o = __shfl_sync(0xffffffffu, off, gbase + u) & omask;
            xv[u] = __ldg(reinterpret_cast<const float4*>(xb + o));
        }
        if (!careful) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float wj = __shfl_sync(0xffffffffu, w, gbase + u);
                if (SPARSE) {
                    const float cj = __shfl_sync(0xffffffffu, cs, gbase + u);
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(__fmul_rn(wj, xv[u].x), cj));
                    acc[1] = __fadd_rn(acc[1], __fmul_rn(__fmul_rn(wj, xv[u].y), cj));
                    acc[2] = __fadd_rn(acc[2], __fmul_rn(__fmul_rn(wj, xv[u].z), cj));
                    acc[3] = __fadd_rn(acc[3], __fmul_rn(__fmul_rn(wj, xv[u].w), cj));
                } else {
                    acc[0] = __fmaf_rn(wj, xv[u].x, acc[0]);
                    acc[1] = __fmaf_rn(wj, xv[u].y, acc[1]);
                    acc[2] = __fmaf_rn(wj, xv[u].z, acc[2]);
                    acc[3] = __fmaf_rn(wj, xv[u].w, acc[3]);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float wj = __shfl_sync(0xffffffffu, w, gbase + u);
                const float cj = SPARSE ? __shfl_sync(0xffffffffu, cs, gbase + u) : 0.0f;
                const float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    if (xs[v] == 0.0f) continue;
                    acc[v] = SPARSE ? __fadd_rn(acc[v], __fmul_rn(__fmul_rn(wj, xs[v]), cj))
                                    : __fmaf_rn(wj, xs[v], acc[v]);
                }
            }
        }
    }
#pragma unroll
    for (int v = 0; v < 4; ++v) ys[warp * CPW + grp][lid * 4 + v] = acc[v];
    __syncthreads();
    for (int i = threadIdx.x; i < CPB * SPB; i += 256) {
        const int bi = i / CPB, ci = i % CPB;
        const int b = b0 + bi;
        const int64_t cc = cb + ci;
        if (b < B && cc < L.n_out) y[(int64_t)b * L.n_out + cc] = ys[ci][bi];
    }
}

// Small batches: lanes over a column's synapses, per-lane partial sums over
// the batch, then a fixed warp tree (deterministic; not the reference's
// sequential order, so equal to it within fp32 rounding).
template <int BMAX, int U, bool SPARSE>
__global__ void __launch_bounds__(256) k_forward_small(LayerView L, const float* __restrict__ xT, int B,
                                                       float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c = (int64_t)blockIdx.x * 8 + warp;
    if (c >= L.n_out) return;
    float osk[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) osk[k] = k < L.rank ? L.os[c * L.rank + k] : 0.0f;
    float acc[BMAX];
#pragma unroll
    for (int b = 0; b < BMAX; ++b) acc[b] = 0.0f;
    const int k0 = L.colptr[c], k1 = L.colptr[c + 1];
    // one entry's contribution to the lane's sums (entries in ascending
    // position per lane: lane, lane + 32, ...)
    // vs0: the row's first value_scale component (the others, rank > 1,
    // are read here)
    auto add = [&](float wq, int r, float vs0, const float* xv) {
        float w, cs = 0.0f;
        if (SPARSE) {
            w = wq;
            cs = __fmul_rn(vs0, osk[0]);
        } else {
            float sc = __fmaf_rn(vs0, osk[0], 0.0f);
            for (int k = 1; k < L.rank; ++k) sc = __fmaf_rn(L.vs[(int64_t)r * L.rank + k], osk[k], sc);
            w = __fmul_rn(wq, sc);
        }
#pragma unroll
        for (int b = 0; b < BMAX; ++b) {
            if (b < B && xv[b] != 0.0f)
                acc[b] = SPARSE ? __fadd_rn(acc[b], __fmul_rn(__fmul_rn(w, xv[b]), cs)) : __fmaf_rn(w, xv[b], acc[b]);
        }
    };
    if (L.cpack) {
        // the packed column index (row << 4 | weight code, one coalesced word
        // per entry): U entries per lane in flight at once, their words
        // first, then their x values and row scales, then the sums in entry
        // order
        for (int kb = k0 + lane; kb < k1; kb += 32 * U) {
            int rr[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int kk = kb + 32 * u;
                rr[u] = kk < k1 ? __ldg(L.cpack + kk) : (L.n_in << 4);
            }
            float xv[U][BMAX], vs0[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int r = rr[u] >> 4;
                const bool live = r < L.n_in;   // not CSC padding
#pragma unroll
                for (int b = 0; b < BMAX; ++b) xv[u][b] = (live && b < B) ? __ldg(xT + (int64_t)r * B + b) : 0.0f;
                vs0[u] = live ? __ldg(L.vs + (int64_t)r * L.rank) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int r = rr[u] >> 4;
                if (r < L.n_in) add(fp4_decode((uint32_t)rr[u] & 15u), r, vs0[u], xv[u]);
            }
        }
    } else {
        for (int kk = k0 + lane; kk < k1; kk += 32) {
            const int vp = L.cvpos[kk];
            if (vp < 0) continue;        // CSC padding
            const int r = L.crow[kk];
            float xv[BMAX];
#pragma unroll
            for (int b = 0; b < BMAX; ++b) xv[b] = b < B ? __ldg(xT + (int64_t)r * B + b) : 0.0f;
            add(fp4_decode(L.val[vp] >> 4), r, L.vs[(int64_t)r * L.rank], xv);
        }
    }
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
        if (b < B) {
            const float v = warp_sum(acc[b]);
            if (lane == 0) y[(int64_t)b * L.n_out + c] = v;
        }
    }
}

void launch_forward(const LayerView& L, const float* xT, int B, float* y, bool sparse, cudaStream_t s) {
    if (L.n_out == 0 || B == 0) return;
    const unsigned gx = (unsigned)((L.n_out + 7) / 8);
    if (B == 1) {   // a vector: 8 entries per lane in flight
        if (sparse) k_forward_small<1, 8, true><<<gx, 256, 0, s>>>(L, xT, B, y);
        else k_forward_small<1, 8, false><<<gx, 256, 0, s>>>(L, xT, B, y);
        count_launch();
        return;
    }
    if (B <= 8) {
        if (sparse) k_forward_small<8, 4, true><<<gx, 256, 0, s>>>(L, xT, B, y);
        else k_forward_small<8, 4, false><<<gx, 256, 0, s>>>(L, xT, B, y);
        count_launch();
        return;
    }
    if (B % 4 == 0) {
        // lanes per column: 4 samples each, up to one warp per column
        const int lpc = B <= 32 ? 8 : (B <= 64 ? 16 : 32);
        const int cpb = 8 * (32 / lpc), spb = 4 * lpc;
        dim3 g((unsigned)((L.n_out + cpb - 1) / cpb), (unsigned)((B + spb - 1) / spb));
        if (lpc == 8) {
            if (sparse) k_forward_vec<8, true><<<g, 256, 0, s>>>(L, xT, B, y);
            else k_forward_vec<8, false><<<g, 256, 0, s>>>(L, xT, B, y);
        } else if (lpc == 16) {
            if (sparse) k_forward_vec<16, true><<<g, 256, 0, s>>>(L, xT, B, y);
            else k_forward_vec<16, false><<<g, 256, 0, s>>>(L, xT, B, y);
        } else {
            if (sparse) k_forward_vec<32, true><<<g, 256, 0, s>>>(L, xT, B, y);
            else k_forward_vec<32, false><<<g, 256, 0, s>>>(L, xT, B, y);
        }
    } else if (B <= 32) {
        dim3 g(gx, 1);
        if (sparse) k_forward_gather<1, true><<<g, 256, 0, s>>>(L, xT, B, y);
        else k_forward_gather<1, false><<<g, 256, 0, s>>>(L, xT, B, y);
    } else {
        dim3 g(gx, (unsigned)((B + 63) / 64));
        if (sparse) k_forward_gather<2, true><<<g, 256, 0, s>>>(L, xT, B, y);
        else k_forward_gather<2, false><<<g, 256, 0, s>>>(L, xT, B, y);
    }
    count_launch();
}

// ── dense backward, learning_rate == 0 ─────────────────────────────────────
// dx[b, r] = sum over the row's synapses, in stored order, of
// fma(w*S(r,c), dy[b,c], .) -- linear_disldo.hpp:884 with cw = quant*S and no
// update.  Lanes over batch samples, so the sum order is the reference's.
template <int NB>
__global__ void __launch_bounds__(256) k_backward_dx(LayerView L, const float* __restrict__ dyT, int B,
                                                     float* __restrict__ dx) {
    __shared__ float xs[8][32 * NB + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * 8, r = r0 + warp;
    const int b0 = blockIdx.y * 32 * NB;
    float acc[NB];
#pragma unroll
    for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
    if (r < L.n_in) {
        const int64_t es = L.es[r];
        const int nnz = (int)(L.ee[r] - es);
        const int f0 = L.rowptr[r];
        float vsk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) vsk[k] = k < L.rank ? L.vs[r * L.rank + k] : 0.0f;
        for (int eb = 0; eb < nnz; eb += 32) {
            const int e = eb + lane;
            int c = 0;
            float cw = 0.0f;
            if (e < nnz) {
                c = L.abs_cols[f0 + e];
                const float wq = fp4_decode(L.val[es + e] >> 4);
                if (L.true_units) {
                    cw = __fmul_rn(__fmul_rn(wq, vsk[0]), L.os[(int64_t)c * L.rank]);
                } else {
                    float sc = 0.0f;
                    for (int k = 0; k < L.rank; ++k) sc = __fmaf_rn(vsk[k], L.os[(int64_t)c * L.rank + k], sc);
                    cw = __fmul_rn(wq, sc);
                }
            }
            const int n = min(32, nnz - eb);
            for (int j0 = 0; j0 < n; j0 += 8) {
                float cwj[8], dv[8][NB];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int jj = (j0 + u) & 31;
                    cwj[u] = __shfl_sync(0xffffffffu, cw, jj);
                    const int cj = __shfl_sync(0xffffffffu, c, jj);
                    const float* dr = dyT + (int64_t)cj * B;
#pragma unroll
                    for (int t = 0; t < NB; ++t) {
                        const int b = b0 + t * 32 + lane;
                        dv[u][t] = (j0 + u < n && b < B) ? __ldg(dr + b) : 0.0f;
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (j0 + u < n) {
#pragma unroll
                        for (int t = 0; t < NB; ++t) acc[t] = __fmaf_rn(cwj[u], dv[u][t], acc[t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NB; ++t) xs[warp][t * 32 + lane] = acc[t];
    __syncthreads();
    for (int i = threadIdx.x; i < 8 * 32 * NB; i += 256) {
        const int w = i & 7, bl = i >> 3;
        const int b = b0 + bl;
        const int64_t rr = r0 + w;
        if (b < B && rr < L.n_in) dx[(int64_t)b * L.n_in + rr] = xs[w][bl];
    }
}

void launch_backward_dx(const LayerView& L, const float* dyT, int B, float* dx, cudaStream_t s) {
    if (L.n_in == 0 || B == 0) return;
    const unsigned gx = (unsigned)((L.n_in + 7) / 8);
    if (B <= 32) {
        k_backward_dx<1><<<dim3(gx, 1), 256, 0, s>>>(L, dyT, B, dx); count_launch();
    } else {
        k_backward_dx<2><<<dim3(gx, (unsigned)((B + 63) / 64)), 256, 0, s>>>(L, dyT, B, dx); count_launch();
    }
}

// ── dense backward, learning_rate != 0: the fused update ───────────────────
// disldo_backward's scattered non-deferred path (linear_disldo.hpp:625-925).
// One warp per input row, synapses in chunks of 32, samples in blocks of 32.
// Per (chunk, block):
//  1. stage dy[block, chunk columns] in shared memory, one coalesced
//     128-byte line per synapse (dyT is [n_out, B]);
//  2. lanes = synapses: each lane runs its synapse's recurrence over the
//     block's samples IN ORDER (ci, quant, cw evolve per sample, exactly as
//     the reference); samples with x == 0 take the closed form of the same
//     arithmetic, and the lane's cw after every x != 0 sample is recorded;
//  3. lanes = samples: dx[b, r] += cw_e(b) * dy[b, c_e] over the chunk's
//     synapses in stored order with fmaf, cw_e(b) being synapse e's weight
//     after sample b -- the reference's summation order, so dx is bit-exact.
// The row's value_scale is updated at the end by lane 0 from double sums.
constexpr int kUpdWarps = 4;
template <bool STOCH, int RANK>
__global__ void __launch_bounds__(kUpdWarps * 32, 6) k_backward_update(LayerView L, const float* __restrict__ xT,
                                                                       const float* __restrict__ dyT, int B,
                                                                       UpdateParams P, float* __restrict__ dxT) {
    __shared__ float dys_s[kUpdWarps][32][33];   // [synapse][sample]
    __shared__ float cws_s[kUpdWarps][33][33];   // [segment][synapse]
    __shared__ float xs_s[kUpdWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kUpdWarps + warp;
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    float* dxr = dxT + r * (int64_t)B;
    if (nnz == 0) {
        for (int b = lane; b < B; b += 32) dxr[b] = 0.0f;
        return;
    }
    float (*dys)[33] = dys_s[warp];
    float (*cws)[33] = cws_s[warp];
    float* xs = xs_s[warp];
    const int f0 = L.rowptr[r];
    const int gnnz = P.row_nnz_g ? P.row_nnz_g[r] : nnz;   // a column shard divides by the global count
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)gnnz) : P.lr;
    const float scale_eff_lr = __fdiv_rn(P.lr, (float)gnnz);
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float zterm = __fmul_rn(onem, 0.0f);
    const bool fast_ok = (!P.damp || P.eps > 0.0f) && isfinite(eff_lr) && P.beta2 >= 0.0f && P.beta2 <= 1.0f;
    const float imp_scale = L.is[r];
    float vsr[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) vsr[k] = L.vs[r * RANK + k];
    const float* xr = xT + r * (int64_t)B;
    const bool vec4 = (B & 3) == 0;

    double sgs[RANK], sgc[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) { sgs[k] = 0.0; sgc[k] = 0.0; }
    double sa_new = 0.0, sa_old = 0.0, sq_new = 0.0, sq_old = 0.0;
    float mx_new = 0.0f;

    for (int e0 = 0; e0 < nnz; e0 += 32) {
        const int e = e0 + lane;
        const int nsyn = min(32, nnz - e0);
        const bool valid = lane < nsyn;
        int c = 0;
        uint32_t byte = 0;
        if (valid) {
            c = L.abs_cols[f0 + e];
            byte = L.val[es + e];
        }
        const float cw_orig = fp4_decode(byte >> 4), ci_orig = fp4_decode(byte & 15u);
        float osk[RANK];
#pragma unroll
        for (int k = 0; k < RANK; ++k) osk[k] = valid ? L.os[(int64_t)c * RANK + k] : 0.0f;
        const float cis = valid ? __fmul_rn(imp_scale, L.ois[c]) : 1.0f;
        float S = 0.0f;
#pragma unroll
        for (int k = 0; k < RANK; ++k) S = __fmaf_rn(vsr[k], osk[k], S);
        float ci = __fmul_rn(ci_orig, cis);
        float quant = cw_orig;
        float cw = __fmul_rn(quant, S);
        const bool lane_static_ok = fast_ok && isfinite(S) && isfinite(cw_orig);
        float cg[RANK], cc[RANK];
#pragma unroll
        for (int k = 0; k < RANK; ++k) { cg[k] = 0.0f; cc[k] = 0.0f; }

        for (int t0 = 0; t0 < B; t0 += 32) {
            const int nb = min(32, B - t0);
            __syncwarp();
            // 1. stage dy: row l of the tile is synapse l's column.  Full
            //    blocks load 16 bytes per lane with 8 lanes covering one
            //    128-byte line (synapse q*4 + lane/8, samples 4*(lane%8)..+3).
            float nf = 0.0f;   // NaN iff a staged dy is inf / NaN (0 * inf = NaN)
            if (vec4 && nb == 32) {
                const int sub = lane >> 3, s4 = (lane & 7) * 4;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int l = q * 4 + sub;
                    const int cl = __shfl_sync(0xffffffffu, c, l);
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (l < nsyn) v = __ldg(reinterpret_cast<const float4*>(dyT + (int64_t)cl * B + t0 + s4));
                    dys[l][s4 + 0] = v.x; dys[l][s4 + 1] = v.y; dys[l][s4 + 2] = v.z; dys[l][s4 + 3] = v.w;
                    nf = __fmaf_rn(v.x, 0.0f, nf); nf = __fmaf_rn(v.y, 0.0f, nf);
                    nf = __fmaf_rn(v.z, 0.0f, nf); nf = __fmaf_rn(v.w, 0.0f, nf);
                }
            } else {
                for (int l = 0; l < 32; ++l) {
                    const int cl = __shfl_sync(0xffffffffu, c, l);
                    const float v = (l < nsyn && lane < nb) ? __ldg(dyT + (int64_t)cl * B + t0 + lane) : 0.0f;
                    dys[l][lane] = v;
                    nf = __fmaf_rn(v, 0.0f, nf);
                }
            }
            const float xl = (lane < nb) ? __ldg(xr + t0 + lane) : 0.0f;
            xs[lane] = xl;
            const unsigned act = __ballot_sync(0xffffffffu, xl != 0.0f);
            const bool dy_finite = __all_sync(0xffffffffu, nf == 0.0f);
            const bool lane_fast = lane_static_ok && ci >= 0.0f && ci <= 100.0f;
            // Samples where some lane's weight may change: x != 0, or every
            // sample when a lane cannot use the x == 0 closed form.
            const unsigned full_mask = nb >= 32 ? 0xffffffffu : ((1u << nb) - 1u);
            const unsigned bnd = (dy_finite && __all_sync(0xffffffffu, lane_fast)) ? act : full_mask;
            __syncwarp();
            // 2. lanes = synapses: the recurrence, recording cw after each boundary sample
            cws[0][lane] = cw;
            unsigned rem = bnd;
            int j = 0, seg = 0;
            while (true) {
                const int ja = rem ? (__ffs(rem) - 1) : nb;
                for (; j + 4 <= ja; j += 4) {                                // x == 0 run
                    ci = __fmaf_rn(P.beta2, ci, zterm); ci = __fmaf_rn(P.beta2, ci, zterm);
                    ci = __fmaf_rn(P.beta2, ci, zterm); ci = __fmaf_rn(P.beta2, ci, zterm);
                }
                for (; j < ja; ++j) ci = __fmaf_rn(P.beta2, ci, zterm);
                if (ja >= nb) break;
                rem &= rem - 1u;
                const float dyv = dys[lane][ja];
                const float iv = xs[ja];
                const float g = __fmul_rn(dyv, iv);
                const float contrib = __fmul_rn(iv, cw_orig);
                ci = bounded_ci(ci, g, contrib, P.beta2, onem);
                const float ngS = __fmul_rn(-g, S);
                float raw = P.damp ? __fdiv_rn(ngS, __fadd_rn(__fsqrt_rn(ci), P.eps)) : ngS;
                if (raw > 2.0f) raw = 2.0f;
                if (raw < -2.0f) raw = -2.0f;
                quant = __fmaf_rn(eff_lr, raw, quant);
                cw = __fmul_rn(quant, S);
                const float qf = (quant == 0.0f) ? 0.1f : quant;
#pragma unroll
                for (int k = 0; k < RANK; ++k) {
                    const double qo = (double)qf * (double)osk[k];
                    sgs[k] = __fma_rn(qo, (double)g, sgs[k]);
                    sgc[k] = __fma_rn(qo, (double)contrib, sgc[k]);
                    if (P.os_trainable) {
                        const float qv = __fmul_rn(qf, vsr[k]);
                        cg[k] = __fmaf_rn(qv, g, cg[k]);
                        cc[k] = __fmaf_rn(qv, contrib, cc[k]);
                    }
                }
                cws[++seg][lane] = cw;
                j = ja + 1;
            }
            __syncwarp();
            // 3. lanes = samples: dx in the reference's order (synapses ascending)
            if (lane < nb) {
                const int sg = __popc(bnd & ((2u << lane) - 1u));
                float* d = dxr + t0 + lane;
                float acc = (e0 == 0) ? 0.0f : *d;
                const float* cwrow = cws[sg];
                if (nsyn == 32) {
#pragma unroll
                    for (int l = 0; l < 32; ++l) acc = __fmaf_rn(cwrow[l], dys[l][lane], acc);
                } else {
                    for (int l = 0; l < nsyn; ++l) acc = __fmaf_rn(cwrow[l], dys[l][lane], acc);
                }
                *d = acc;
            }
        }
        if (valid) {
            const float imp_st = __fdiv_rn(ci, cis);
            uint32_t nbyte;
            if (STOCH) {
                const uint64_t vp = (uint64_t)(es + e);
                nbyte = (fp4_quantize_stochastic(quant, rng_draw(P.call_key, vp, 0)) << 4) |
                        fp4_quantize_stochastic(imp_st, rng_draw(P.call_key, vp, 1));
            } else {
                nbyte = (fp4_encode(quant) << 4) | fp4_encode(imp_st);
            }
            L.val[es + e] = (uint8_t)nbyte;
            if (L.cpack_upd) L.cpack_upd[L.fcpos[f0 + e]] = (int)(((uint32_t)r << 4) | (nbyte >> 4));
            const float ai = fp4_decode(nbyte & 15u);
            sa_new += fabs((double)ai);
            sa_old += fabs((double)ci_orig);
            sq_new += (double)ai * (double)ai;
            sq_old += (double)ci_orig * (double)ci_orig;
            mx_new = fmaxf(mx_new, fabsf(ai));
            if (P.os_trainable) {
#pragma unroll
                for (int k = 0; k < RANK; ++k) {
                    atomicAdd(P.colg + (int64_t)c * RANK + k, cg[k]);
                    atomicAdd(P.colc + (int64_t)c * RANK + k, cc[k]);
                }
            }
        }
    }
    // value_scale update (linear_disldo.hpp:901-925)
#pragma unroll
    for (int k = 0; k < RANK; ++k) {
        sgs[k] = warp_sum(sgs[k]);
        sgc[k] = warp_sum(sgc[k]);
    }
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            const int64_t i = r * RANK + k;
            if (P.row_part) {   // a column shard: its part of the row sums
                P.row_part[2 * i] = sgs[k];
                P.row_part[2 * i + 1] = sgc[k];
            } else if (!P.scale_noop) {
                rmsprop_scale(L.vs + i, L.vsi + i, (float)sgs[k], scale_eff_lr, (float)sgc[k], L.vstep + i, P);
            }
        }
    }
    sa_new = warp_sum(sa_new); sa_old = warp_sum(sa_old);
    sq_new = warp_sum(sq_new); sq_old = warp_sum(sq_old);
    for (int o = 16; o > 0; o >>= 1) mx_new = fmaxf(mx_new, __shfl_xor_sync(0xffffffffu, mx_new, o));
    if (lane == 0) {
        atomicAdd(P.stats + 0, sa_new - sa_old);
        atomicAdd(P.stats + 1, sq_new - sq_old);
        atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx_new));
    }
}

void launch_backward_update(const LayerView& L, const float* xT, const float* dyT, int B,
                            const UpdateParams& P, float* dxT, cudaStream_t s) {
    if (L.n_in == 0) return;
    if (B <= 128) {   // x and dx of a row fit in registers: the tiled two-chain kernel
        launch_backward_update_tiled(L, xT, dyT, B, P, dxT, s);
        return;
    }
    const unsigned g = (unsigned)((L.n_in + kUpdWarps - 1) / kUpdWarps);
#define SILI_BWD(R)                                                                         \
    if (P.stochastic) k_backward_update<true, R><<<g, kUpdWarps * 32, 0, s>>>(L, xT, dyT, B, P, dxT);  \
    else k_backward_update<false, R><<<g, kUpdWarps * 32, 0, s>>>(L, xT, dyT, B, P, dxT);
    switch (L.rank) {
    case 1: SILI_BWD(1) break;
    case 2: SILI_BWD(2) break;
    case 3: SILI_BWD(3) break;
    default: SILI_BWD(4) break;
    }
#undef SILI_BWD
    count_launch();
}

// output_scale update, linear_disldo.hpp:2051-2080
__global__ void k_output_scale_update(LayerView L, const int* __restrict__ out_degree, UpdateParams P) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= L.n_out) return;
    const int deg = out_degree[c];
    if (deg == 0) return;
    const float col_lr = __fdiv_rn(P.lr, (float)deg);
    for (int k = 0; k < L.rank; ++k) {
        const int64_t i = c * L.rank + k;
        rmsprop_scale(L.os + i, L.osi + i, P.colg[i], col_lr, P.colc[i], L.ostep + i, P);
    }
}
void launch_output_scale_update(const LayerView& L, const int* out_degree, const UpdateParams& P,
                                cudaStream_t s) {
    if (L.n_out == 0 || P.scale_noop) return;
    k_output_scale_update<<<(unsigned)((L.n_out + 255) / 256), 256, 0, s>>>(L, out_degree, P); count_launch();
}

// Dead-row bootstrap, linear_disldo.hpp:1985-2042: S[b,k] = sum_c os[c,k]*dy[b,c]
// in double, then an Adam step on value_scale of every row with no synapse.
// The sum runs over the columns in order, each term a rounded double product
// then a rounded add (the reference build's evaluation, pinned through the
// oracle): a thread per (b, k), the loads of the next columns in flight
// while the chain adds.
__global__ void k_dead_S(LayerView L, const float* __restrict__ dy, int B, double* __restrict__ S) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)B * L.rank) return;
    const int b = (int)(t / L.rank), k = (int)(t % L.rank);
    const float* d = dy + (int64_t)b * L.n_out;
    double s = 0.0;
    int64_t c = 0;
    for (; c + 4 <= L.n_out; c += 4) {
        double p[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) p[u] = __dmul_rn((double)L.os[(c + u) * L.rank + k], (double)d[c + u]);
#pragma unroll
        for (int u = 0; u < 4; ++u) s = __dadd_rn(s, p[u]);
    }
    for (; c < L.n_out; ++c) s = __dadd_rn(s, __dmul_rn((double)L.os[c * L.rank + k], (double)d[c]));
    S[t] = s;
}
// the Adam step of one dead row from S (linear_disldo.hpp:2000-2040)
__device__ void dead_row_step(const LayerView& L, const float* __restrict__ xT, int B, const double* __restrict__ S,
                              int64_t r, float dead_lr, const UpdateParams& P) {
    const float onem = __fsub_rn(1.0f, P.beta2);
    for (int k = 0; k < L.rank; ++k) {
        double sum = 0.0;
        for (int b = 0; b < B; ++b) {
            const float iv = xT[r * B + b];
            if (iv == 0.0f) continue;
            sum = __dadd_rn(sum, __dmul_rn((double)iv, S[(int64_t)b * L.rank + k]));
        }
        if (sum == 0.0) continue;
        const float g = (float)sum;
        if (!isfinite(g)) continue;
        const int64_t i = r * L.rank + k;
        const float m = L.vsm[i], v = L.vsi[i];
        const float nm = __fmaf_rn(0.9f, m, __fmul_rn(__fsub_rn(1.0f, 0.9f), g));
        // new_v = beta2 * v + (1 - beta2) * g * g as the reference build
        // evaluates it: fma(1 - beta2, g * g, beta2 * v)
        const float nv = __fmaf_rn(onem, __fmul_rn(g, g), __fmul_rn(P.beta2, v));
        if (!isfinite(nm) || !isfinite(nv)) continue;
        const float nvs = __fsub_rn(L.vs[i], __fdiv_rn(__fmul_rn(dead_lr, nm), __fadd_rn(__fsqrt_rn(nv), P.eps)));
        if (!isfinite(nvs)) continue;
        L.vsm[i] = nm;
        L.vsi[i] = nv;
        L.vs[i] = nvs;
    }
}
__global__ void k_dead_rows(LayerView L, const float* __restrict__ xT, int B, const double* __restrict__ S,
                            UpdateParams P) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= L.n_in) return;
    if (L.ee[r] != L.es[r]) return;
    if (L.b4_nt && L.b4_nt[r >> 2] > 0) return;   // block4 slots make the row live (:1961-1967)
    dead_row_step(L, xT, B, S, r, __fdiv_rn(P.lr, (float)L.n_out), P);
}
void launch_dead_rows(const LayerView& L, const float* xT, const float* dy, int B, double* S,
                      const UpdateParams& P, cudaStream_t s) {
    if (L.n_in == 0 || B == 0) return;
    k_dead_S<<<(unsigned)(((int64_t)B * L.rank + 127) / 128), 128, 0, s>>>(L, dy, B, S); count_launch();
    k_dead_rows<<<(unsigned)((L.n_in + 127) / 128), 128, 0, s>>>(L, xT, B, S, P); count_launch();
}
void launch_dead_S(const LayerView& L, const float* dy, int B, double* S, cudaStream_t s) {
    if (B == 0) return;
    k_dead_S<<<(unsigned)(((int64_t)B * L.rank + 127) / 128), 128, 0, s>>>(L, dy, B, S); count_launch();
}

// Column shards: the row steps every shard takes after the parts are summed,
// the value_scale step of a row with synapses on some shard (the row sums of
// linear_disldo.hpp:901-925 over all its synapses) and the dead-row step of a
// row with none on any shard (S over every column, lr / global n_out).
__global__ void k_apply_row_part(LayerView L, const int* __restrict__ row_nnz_g, float dead_lr,
                                 const double* __restrict__ part, const float* __restrict__ xT, int B,
                                 UpdateParams P) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= L.n_in) return;
    const int gnnz = row_nnz_g[r];
    if (gnnz == 0) {
        dead_row_step(L, xT, B, part + 2 * L.n_in * L.rank, r, dead_lr, P);
        return;
    }
    if (P.scale_noop) return;
    const float se = __fdiv_rn(P.lr, (float)gnnz);
    for (int k = 0; k < L.rank; ++k) {
        const int64_t i = r * L.rank + k;
        rmsprop_scale(L.vs + i, L.vsi + i, (float)part[2 * i], se, (float)part[2 * i + 1], L.vstep + i, P);
    }
}
void launch_apply_row_part(const LayerView& L, const int* row_nnz_g, int64_t g_n_out, const double* part,
                           const float* xT, int B, const UpdateParams& P, cudaStream_t s) {
    if (L.n_in == 0) return;
    const float dead_lr = P.lr / (float)g_n_out;   // IEEE division, as __fdiv_rn
    k_apply_row_part<<<(unsigned)((L.n_in + 127) / 128), 128, 0, s>>>(L, row_nnz_g, dead_lr, part, xT, B, P);
    count_launch();
}

// ── sparse-gradient backward (disldo_backward_sparse_grad, sisldo_ops.hpp:589-799) ──
// One warp per row, batch samples in order (each sample requantizes the
// row's codes before the next reads them), lanes over the row's synapses.
// A synapse takes part in sample b only if dy's CSR holds an entry at its
// column (presT), whatever that entry's value.
__global__ void __launch_bounds__(256) k_backward_sparse(LayerView L, const float* __restrict__ xT,
                                                         const float* __restrict__ dyT,
                                                         const uint8_t* __restrict__ presT, int B,
                                                         UpdateParams P, double* __restrict__ sgs_out,
                                                         double* __restrict__ sgc_out, float* __restrict__ dxT) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + warp;
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    float* dxr = dxT + r * (int64_t)B;
    if (nnz == 0) {
        for (int b = lane; b < B; b += 32) dxr[b] = 0.0f;
        return;
    }
    const int f0 = L.rowptr[r];
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)nnz) : P.lr;
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float imp_scale = L.is[r];
    const float val_scale = L.vs[r * L.rank];
    double sgs = 0.0, sgc = 0.0, sa_new = 0.0, sa_old = 0.0, sq_new = 0.0, sq_old = 0.0;
    float mx_new = 0.0f;
    for (int b = 0; b < B; ++b) {
        const float in_val = xT[r * B + b];
        float dxa = 0.0f;
        for (int e0 = 0; e0 < nnz; e0 += 32) {
            const int e = e0 + lane;
            if (e >= nnz) continue;
            const int c = L.abs_cols[f0 + e];
            if (!presT[(int64_t)c * B + b]) continue;
            const uint8_t byte = L.val[es + e];
            const float w_stored = fp4_decode(byte >> 4);
            const float out_scale = L.os[(int64_t)c * L.rank];
            const float cs = __fmul_rn(val_scale, out_scale);
            const float w = __fmul_rn(w_stored, cs);
            const float dyv = dyT[(int64_t)c * B + b];
            dxa = __fmaf_rn(w, dyv, dxa);
            if (P.lr != 0.0f) {
                const float cis = __fmul_rn(imp_scale, L.ois[c]);
                const float grad = __fmul_rn(dyv, in_val);
                const float stored_imp = fp4_decode(byte & 15u);
                float imp = __fmul_rn(stored_imp, cis);
                const float contrib = __fmul_rn(in_val, w);
                imp = __fmaf_rn(P.beta2, imp, __fmul_rn(onem, __fmaf_rn(grad, grad, __fmul_rn(contrib, contrib))));
                const float num = __fmul_rn(-eff_lr, grad);
                const float step = P.damp ? __fdiv_rn(num, __fadd_rn(__fsqrt_rn(imp), P.eps)) : num;
                const float new_w = __fadd_rn(w, step);
                const uint32_t nbyte = (fp4_encode(__fdiv_rn(new_w, cs)) << 4) | fp4_encode(__fdiv_rn(imp, cis));
                L.val[es + e] = (uint8_t)nbyte;
                if (L.cpack_upd) L.cpack_upd[L.fcpos[f0 + e]] = (int)(((uint32_t)r << 4) | (nbyte >> 4));
                const float ai = fp4_decode(nbyte & 15u);
                sa_new += fabs((double)ai); sa_old += fabs((double)stored_imp);
                sq_new += (double)ai * (double)ai; sq_old += (double)stored_imp * (double)stored_imp;
                mx_new = fmaxf(mx_new, fabsf(ai));
                sgs += (double)w_stored * (double)out_scale * (double)grad;
                sgc += (double)w_stored * (double)out_scale * (double)contrib;
            }
        }
        dxa = warp_sum(dxa);
        if (lane == 0) dxr[b] = dxa;
        __syncwarp();
    }
    sgs = warp_sum(sgs); sgc = warp_sum(sgc);
    sa_new = warp_sum(sa_new); sa_old = warp_sum(sa_old);
    sq_new = warp_sum(sq_new); sq_old = warp_sum(sq_old);
    for (int o = 16; o > 0; o >>= 1) mx_new = fmaxf(mx_new, __shfl_xor_sync(0xffffffffu, mx_new, o));
    if (lane == 0) {
        sgs_out[r] = sgs;
        sgc_out[r] = sgc;
        if (P.lr != 0.0f) {
            atomicAdd(P.stats + 0, sa_new - sa_old);
            atomicAdd(P.stats + 1, sq_new - sq_old);
            atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx_new));
        }
    }
}
// The same for B <= 64, arranged around dy's sparsity: a lane keeps its
// synapse's column, scales and current byte in registers across the samples,
// reads its 64 presence flags once as a bit mask and visits only its own
// present samples (about 3 % of them at a 3 % top-k dy).  Each
// (synapse, sample) step is k_backward_sparse's, in the same sample order; a
// lane's dx partial for sample b accumulates over its synapses in the same
// order (shared memory, [sample][lane]) and the per-sample warp tree is the
// same, so dx and every code and sum match k_backward_sparse.
constexpr int kBs64Warps = 4;
__global__ void __launch_bounds__(kBs64Warps * 32) k_backward_sparse64(LayerView L, const float* __restrict__ xT,
                                                                      const float* __restrict__ dyT,
                                                                      const uint8_t* __restrict__ presT, int B,
                                                                      UpdateParams P, double* __restrict__ sgs_out,
                                                                      double* __restrict__ sgc_out,
                                                                      float* __restrict__ dxT) {
    __shared__ float dxa_s[kBs64Warps][64][32];
    __shared__ float xs_s[kBs64Warps][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kBs64Warps + warp;
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    float* dxr = dxT + r * (int64_t)B;
    if (nnz == 0) {
        for (int b = lane; b < B; b += 32) dxr[b] = 0.0f;
        return;
    }
    float (*dxa)[32] = dxa_s[warp];
    float* xs = xs_s[warp];
    for (int b = 0; b < 64; ++b) dxa[b][lane] = 0.0f;
    for (int b = lane; b < 64; b += 32) xs[b] = b < B ? xT[r * B + b] : 0.0f;
    __syncwarp();
    const int f0 = L.rowptr[r];
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)nnz) : P.lr;
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float imp_scale = L.is[r];
    const float val_scale = L.vs[r * L.rank];
    const bool train = P.lr != 0.0f;
    double sgs = 0.0, sgc = 0.0, sa_new = 0.0, sa_old = 0.0, sq_new = 0.0, sq_old = 0.0;
    float mx_new = 0.0f;
    for (int e0 = 0; e0 < nnz; e0 += 32) {
        const int e = e0 + lane;
        const bool valid = e < nnz;
        int c = 0;
        uint32_t byte = 0;
        unsigned long long mask = 0ull;
        float out_scale = 0.0f, cs = 0.0f, cis = 0.0f;
        if (valid) {
            c = L.abs_cols[f0 + e];
            byte = L.val[es + e];
            out_scale = L.os[(int64_t)c * L.rank];
            cs = __fmul_rn(val_scale, out_scale);
            cis = __fmul_rn(imp_scale, L.ois[c]);
            const uint8_t* pr = presT + (int64_t)c * B;
            if (B == 64) {
                const uint4* p4 = reinterpret_cast<const uint4*>(pr);   // c * 64 bytes: 16-byte aligned
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 v = __ldg(p4 + q);
                    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k)
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            if ((wv[k] >> (8 * t)) & 0xFFu) mask |= 1ull << (q * 16 + k * 4 + t);
                }
            } else {
                for (int b = 0; b < B; ++b)
                    if (pr[b]) mask |= 1ull << b;
            }
        }
        // this synapse's present samples, in order (lanes independent)
        while (mask) {
            const int b = __ffsll((long long)mask) - 1;
            mask &= mask - 1ull;
            const float in_val = xs[b];
            const float w_stored = fp4_decode(byte >> 4);
            const float w = __fmul_rn(w_stored, cs);
            const float dyv = dyT[(int64_t)c * B + b];
            dxa[b][lane] = __fmaf_rn(w, dyv, dxa[b][lane]);
            if (train) {
                const float grad = __fmul_rn(dyv, in_val);
                const float stored_imp = fp4_decode(byte & 15u);
                float imp = __fmul_rn(stored_imp, cis);
                const float contrib = __fmul_rn(in_val, w);
                imp = __fmaf_rn(P.beta2, imp, __fmul_rn(onem, __fmaf_rn(grad, grad, __fmul_rn(contrib, contrib))));
                const float num = __fmul_rn(-eff_lr, grad);
                const float step = P.damp ? __fdiv_rn(num, __fadd_rn(__fsqrt_rn(imp), P.eps)) : num;
                const float new_w = __fadd_rn(w, step);
                const uint32_t nbyte = (fp4_encode(__fdiv_rn(new_w, cs)) << 4) | fp4_encode(__fdiv_rn(imp, cis));
                const float ai = fp4_decode(nbyte & 15u);
                sa_new += fabs((double)ai); sa_old += fabs((double)stored_imp);
                sq_new += (double)ai * (double)ai; sq_old += (double)stored_imp * (double)stored_imp;
                mx_new = fmaxf(mx_new, fabsf(ai));
                sgs += (double)w_stored * (double)out_scale * (double)grad;
                sgc += (double)w_stored * (double)out_scale * (double)contrib;
                byte = nbyte;
            }
        }
        if (valid && train) L.val[es + e] = (uint8_t)byte;
    }
    __syncwarp();
    for (int b = 0; b < B; ++b) {
        const float v = warp_sum(dxa[b][lane]);
        if (lane == 0) dxr[b] = v;
    }
    sgs = warp_sum(sgs); sgc = warp_sum(sgc);
    sa_new = warp_sum(sa_new); sa_old = warp_sum(sa_old);
    sq_new = warp_sum(sq_new); sq_old = warp_sum(sq_old);
    for (int o = 16; o > 0; o >>= 1) mx_new = fmaxf(mx_new, __shfl_xor_sync(0xffffffffu, mx_new, o));
    if (lane == 0) {
        sgs_out[r] = sgs;
        sgc_out[r] = sgc;
        if (train) {
            atomicAdd(P.stats + 0, sa_new - sa_old);
            atomicAdd(P.stats + 1, sq_new - sq_old);
            atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx_new));
        }
    }
}

void launch_backward_sparse(const LayerView& L, const float* xT, const float* dyT, const uint8_t* presT, int B,
                            const UpdateParams& P, double* sgs, double* sgc, float* dxT, cudaStream_t s) {
    if (L.n_in == 0) return;
    if (B <= 64) {
        k_backward_sparse64<<<(unsigned)((L.n_in + kBs64Warps - 1) / kBs64Warps), kBs64Warps * 32, 0, s>>>(
            L, xT, dyT, presT, B, P, sgs, sgc, dxT);
    } else {
        k_backward_sparse<<<(unsigned)((L.n_in + 7) / 8), 256, 0, s>>>(L, xT, dyT, presT, B, P, sgs, sgc, dxT);
    }
    count_launch();
}

// value_scale after all samples, sisldo_ops.hpp:772-797 (no finiteness guards there).
__global__ void k_sparse_scale_update(LayerView L, const double* __restrict__ sgs, const double* __restrict__ sgc,
                                      UpdateParams P) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= L.n_in) return;
    if (sgs[r] == 0.0 && sgc[r] == 0.0) return;
    const int64_t nnz = L.ee[r] - L.es[r];
    if (nnz == 0) return;
    const float se = __fdiv_rn(P.lr, (float)nnz);
    const float g = (float)sgs[r], cg = (float)sgc[r];
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float nv = __fmaf_rn(P.beta2, L.vsi[r], __fmul_rn(onem, __fmaf_rn(g, g, __fmul_rn(cg, cg))));
    const uint32_t st = L.vstep[r * L.rank] + 1u;
    L.vstep[r * L.rank] = st;
    const float bc = __fsub_rn(1.0f, bias_pow(P, st));
    const float hat = bc > 0.0f ? __fdiv_rn(nv, bc) : nv;
    L.vsi[r] = nv;
    L.vs[r] = __fsub_rn(L.vs[r], __fdiv_rn(__fmul_rn(se, g), __fadd_rn(__fsqrt_rn(hat), P.eps)));
}
void launch_sparse_scale_update(const LayerView& L, const double* sgs, const double* sgc, const UpdateParams& P,
                                cudaStream_t s) {
    if (L.n_in == 0) return;
    k_sparse_scale_update<<<(unsigned)((L.n_in + 255) / 256), 256, 0, s>>>(L, sgs, sgc, P); count_launch();
}

__global__ void k_csr_to_dense_t(const int* __restrict__ ptrs, const int* __restrict__ idx,
                                 const float* __restrict__ vals, int rows, int cols, float* __restrict__ outT,
                                 uint8_t* __restrict__ presT) {
    const int b = blockIdx.x;
    if (b >= rows) return;
    for (int j = ptrs[b] + threadIdx.x; j < ptrs[b + 1]; j += blockDim.x) {
        const int c = idx[j];
        if (c < 0 || c >= cols) continue;   // out-of-range entries are rejected on the host for host input
        const int64_t o = (int64_t)c * rows + b;
        outT[o] = vals[j];
        if (presT) presT[o] = 1;
    }
}
void launch_csr_to_dense_t(const int* ptrs, const int* idx, const float* vals, int rows, int cols, float* outT,
                           uint8_t* presT, cudaStream_t s) {
    if (rows == 0) return;
    k_csr_to_dense_t<<<(unsigned)rows, 128, 0, s>>>(ptrs, idx, vals, rows, cols, outT, presT); count_launch();
}

}  // namespace sili
