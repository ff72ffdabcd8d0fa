// The dense forward with x staged in shared memory (disldo_forward,
// linear_disldo.hpp:289-308 / sisldo_forward for the sparse formula), for
// scale rank 1 and batches that are a multiple of 4.
//
// k_forward_vec gathers one x row per synapse from L2 (nnz x B x 4 bytes per
// launch), reaches the weight byte through cvpos, and spends most of its
// instructions broadcasting each synapse to the lanes of its column.  Here a
// thread owns one output column and 32 samples, the CTA walks the input rows
// in tiles whose x rows are staged into shared memory once (xT is read from
// L2 once per CTA instead of once per synapse), and each thread consumes its
// column's entries of the tile from the packed column index cpack (row << 4
// | weight code: one 4-byte load per synapse, no cvpos -> val gather).  The
// entries of a column are taken in ascending row order across tiles, so y is
// the same fma chain as k_forward_vec and the reference's single-thread loop:
// bit-exact.
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace sili {

// cpack over the padded CSC: real entries row << 4 | weight code, padding
// entries (cvpos -1) n_in << 4 (the zero input row, code 0 = weight 0)
__global__ void k_pack_csc(const int* __restrict__ colptr, int64_t n_out, const int* __restrict__ crow,
                           const int* __restrict__ cvpos, const uint8_t* __restrict__ val, int n_in,
                           int* __restrict__ cpack, int64_t bound) {
    const int64_t total = min((int64_t)colptr[n_out], bound);
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        const int vp = cvpos[k];
        cpack[k] = vp >= 0 ? ((crow[k] << 4) | (int)(val[vp] >> 4)) : (n_in << 4);
    }
}
void launch_pack_csc(const LayerView& L, int64_t bound, int* cpack, cudaStream_t s) {
    if (L.n_out == 0 || bound <= 0) return;
    const int64_t blocks = std::min<int64_t>((bound + 255) / 256, 148 * 16);
    k_pack_csc<<<(unsigned)blocks, 256, 0, s>>>(L.colptr, L.n_out, L.crow, L.cvpos, L.val, (int)L.n_in, cpack,
                                                bound);
    count_launch();
}

// ── lane-per-column forward ───────────────────────────────────────────────
// One thread per output column and SG samples (acc[SG] in registers; SG =
// 32, or 16 / 8 / 4 for narrow layers -- a column shard of a folded stack on
// many GPUs -- so that the grid still fills every SM).  Per tile of RT input
// rows the CTA stages x[rows][SG samples] into shared memory (SG / 4 float4
// chunks of an SG * 4-byte row); each thread then consumes its column's
// entries whose row lies in the tile, in ascending row order, SG fmas per
// entry, the next entry's packed word loaded ahead.  Lane l reads chunk
// q ^ (l mod C) at step q (C = SG / 4 chunks per row; its accumulator 4q + v
// holds sample 4 (q ^ (l mod C)) + v): for SG = 32 the 8 lanes of a quarter-
// warp then always touch 8 different bank groups, whatever rows they read,
// and with the tile 128-byte aligned the chunk address is one xor of the row
// address.  Weight codes are decoded through a 16-entry table in shared
// memory.
__device__ __forceinline__ float4 lds128(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

template <bool SPARSE, int SG>
__global__ void __launch_bounds__(256, 3) k_forward_cols(LayerView L, const float* __restrict__ xT, int B, int RT,
                                                      float* __restrict__ y) {
    constexpr int C = SG / 4;              // float4 chunks per staged row
    constexpr int ROWB = SG * 4;           // bytes per staged row
    // [pad to 128 B][RT][C] chunks of 4 samples, then vs of the RT rows, then the code table
    extern __shared__ __align__(16) unsigned char fc_smem[];
    const uint32_t raw32 = (uint32_t)__cvta_generic_to_shared(fc_smem);
    const uint32_t pad = (128u - (raw32 & 127u)) & 127u;
    float4* xs4 = reinterpret_cast<float4*>(fc_smem + pad);
    const uint32_t xs32 = raw32 + pad;
    float* vs_t = reinterpret_cast<float*>(xs4 + RT * C);
    float* ftab = vs_t + RT;
    if (threadIdx.x < 16) ftab[threadIdx.x] = fp4_decode(threadIdx.x);
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int b0 = blockIdx.y * SG;
    const int n_in = (int)L.n_in;
    const uint32_t rot16 = (threadIdx.x & (C - 1)) << 4;
    int cur = 0, end = 0;
    float oc = 0.0f;
    if (c < L.n_out) {
        cur = L.colptr[c];
        end = cur + (L.colptr_x[c + 1] - L.colptr_x[c]);
        oc = L.os[c];
    }
    float acc[SG];
#pragma unroll
    for (int v = 0; v < SG; ++v) acc[v] = 0.0f;
    // packed words four at a time (columns start on 8-entry boundaries of
    // the padded CSC, so cur & ~3 is 16-byte aligned)
    const int4* cp4 = reinterpret_cast<const int4*>(L.cpack);
    const int4 none = make_int4(n_in << 4, n_in << 4, n_in << 4, n_in << 4);
    // the group holding cur, and the next one already in flight
    int4 nb = cur < end ? __ldg(cp4 + (cur >> 2)) : none;
    int4 nb2 = (cur | 3) + 1 < end ? __ldg(cp4 + (cur >> 2) + 1) : none;
    auto word = [&](int k) { return k == 0 ? nb.x : k == 1 ? nb.y : k == 2 ? nb.z : nb.w; };
    int pk = word(cur & 3);

    for (int R0 = 0; R0 < n_in; R0 += RT) {
        const int nr = min(RT, n_in - R0), R1 = R0 + nr;
        __syncthreads();   // the previous tile's readers are done
#pragma unroll 4
        for (int t = threadIdx.x; t < nr * C; t += blockDim.x) {
            const int i = t / C, q = t % C;
            const int b = b0 + 4 * q;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (b < B) v = __ldg(reinterpret_cast<const float4*>(xT + (int64_t)(R0 + i) * B + b));
            xs4[i * C + q] = v;
        }
        for (int i = threadIdx.x; i < nr; i += blockDim.x) vs_t[i] = __ldg(L.vs + R0 + i);
        __syncthreads();
        while (cur < end && (pk >> 4) < R1) {
            const int ri = (pk >> 4) - R0, code = pk & 15;
            ++cur;
            // the next entry's word, ahead of this one's fmas
            if ((cur & 3) == 0) {
                nb = nb2;
                nb2 = cur + 4 < end ? __ldg(cp4 + (cur >> 2) + 1) : none;
            }
            pk = cur < end ? word(cur & 3) : (n_in << 4);
            const float wq = ftab[code];
            const float vr = vs_t[ri];
            float w, cs = 0.0f;
            if (SPARSE) {
                w = wq;
                cs = __fmul_rn(vr, oc);
            } else {
                w = __fmul_rn(wq, __fmaf_rn(vr, oc, 0.0f));
            }
            const uint32_t rowa = (xs32 + (uint32_t)ri * ROWB) ^ rot16;
            if (isfinite(w) && (!SPARSE || isfinite(cs))) {
#pragma unroll
                for (int q = 0; q < C; ++q) {
                    const float4 xv = lds128(rowa ^ ((uint32_t)q << 4));
                    if (SPARSE) {
                        acc[4 * q + 0] = __fadd_rn(acc[4 * q + 0], __fmul_rn(__fmul_rn(w, xv.x), cs));
                        acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __fmul_rn(__fmul_rn(w, xv.y), cs));
                        acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __fmul_rn(__fmul_rn(w, xv.z), cs));
                        acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __fmul_rn(__fmul_rn(w, xv.w), cs));
                    } else {
                        acc[4 * q + 0] = __fmaf_rn(w, xv.x, acc[4 * q + 0]);
                        acc[4 * q + 1] = __fmaf_rn(w, xv.y, acc[4 * q + 1]);
                        acc[4 * q + 2] = __fmaf_rn(w, xv.z, acc[4 * q + 2]);
                        acc[4 * q + 3] = __fmaf_rn(w, xv.w, acc[4 * q + 3]);
                    }
                }
            } else {
                // a non-finite weight: the reference skips x == 0 inputs, so
                // 0 * inf never reaches the sum
#pragma unroll
                for (int q = 0; q < C; ++q) {
                    const float4 xv = lds128(rowa ^ ((uint32_t)q << 4));
                    const float xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        if (xq[v] == 0.0f) continue;
                        acc[4 * q + v] = SPARSE ? __fadd_rn(acc[4 * q + v], __fmul_rn(__fmul_rn(w, xq[v]), cs))
                                                : __fmaf_rn(w, xq[v], acc[4 * q + v]);
                    }
                }
            }
        }
    }
    if (c < L.n_out) {
        const int rot = threadIdx.x & (C - 1);
#pragma unroll
        for (int k = 0; k < SG; ++k) {
            const int b = b0 + 4 * ((k >> 2) ^ rot) + (k & 3);
            if (b < B) y[(int64_t)b * L.n_out + c] = acc[k];
        }
    }
}

namespace {
struct ColsPlan {
    int threads = 0, rt = 0, sg = 0;
};

// A plan forced through the environment (SILI_FORWARD_COLS_PLAN="vec" for
// the per-synapse gather kernels, or "sg,threads,rows_per_tile"), read once:
// a tuning override for measuring the plans against each other.
struct PlanOverride {
    bool set = false, vec = false;
    ColsPlan p;
    PlanOverride() {
        const char* e = getenv("SILI_FORWARD_COLS_PLAN");
        if (!e || !*e) return;
        set = true;
        if (e[0] == 'v') { vec = true; return; }
        int a = 0, b = 0, c = 0;
        if (sscanf(e, "%d,%d,%d", &a, &b, &c) == 3 && (a == 32 || a == 16 || a == 8 || a == 4) &&
            (b == 256 || b == 128 || b == 64 || b == 32) && c >= 16 && c <= 2048) {
            p.sg = a; p.threads = b; p.rt = c;
        } else {
            set = false;
        }
    }
};
const PlanOverride& plan_override() {
    static PlanOverride o;
    return o;
}

// 32 samples per thread in 256-thread CTAs when that gives every SM two CTAs;
// no plan (threads 0) for narrower layers, where the per-synapse gathers of
// k_forward_vec win (a CTA re-reads all of x).  128-thread CTAs for layers
// between 148 and 296 CTAs wide measured slower than k_forward_vec on every
// config-5 shard they served (q / o / down at 4 ranks: 0.213 / 0.178 / 1.736
// ms against about 0.18 / 0.17 / 1.13).
ColsPlan cols_plan(const LayerView& L, int B) {
    ColsPlan p;
    if (L.rank != 1 || B < 16 || (B & 3) != 0 || L.n_in >= (1 << 27) || L.n_out == 0 || L.n_in == 0) return p;
    const PlanOverride& o = plan_override();
    if (o.set) {
        if (o.vec) return p;
        p = o.p;
        p.rt = (int)std::min<int64_t>(L.n_in, p.rt);
        return p;
    }
    const int sg = 32;
    const int64_t sgroups = (B + sg - 1) / sg;
    const int t = 256;
    // 3 CTAs fit per SM (64 KB x tile each): a grid whose last wave is
    // mostly empty loses to the per-synapse kernel (measured on the 8-way
    // shard of a 163840-column gate projection: 640 CTAs, 1.44 waves, 9 %
    // slower; the 4-way shard's 1280 CTAs, 2.9 waves, 13 % faster)
    const int64_t ctas = ((L.n_out + t - 1) / t) * sgroups;
    const int64_t wave = 3 * 148;
    if (ctas < 2 * 148 || ctas * 10 < ((ctas + wave - 1) / wave) * wave * 8) return p;
    p.threads = t;
    p.sg = sg;
    // x tile: 128 bytes per row, 64 KB (3 CTAs per SM)
    p.rt = (int)std::min<int64_t>(L.n_in, 512);
    return p;
}

template <bool SPARSE>
void launch_cols(const ColsPlan& p, dim3 g, size_t smem, const LayerView& L, const float* xT, int B, float* y,
                 cudaStream_t s) {
    switch (p.sg) {
    case 32: k_forward_cols<SPARSE, 32><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y); break;
    case 16: k_forward_cols<SPARSE, 16><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y); break;
    case 8: k_forward_cols<SPARSE, 8><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y); break;
    default: k_forward_cols<SPARSE, 4><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y); break;
    }
}
}  // namespace

// ── FoldedLayer.forward in one launch ─────────────────────────────────────
// sili/sparse_rnn.py:1096-1125: raw = sum over the suffix layers (all on the
// same x, Python's sum: 0 + raw_0 + raw_1 + ...) of forward_dense(x), then
// the fold sum y[b, j] = sum over f ascending of raw[b, f * out_dim + j]
// (FoldedColumnLayer.in_proj, :1340-1362, keeps raw).  A thread owns one
// stacked column and SG samples of every suffix layer: each suffix's column
// chain is k_forward_cols's (rows ascending, the same fma order), all of
// them fed from one staged x tile.  With the fold sum the CTA holds all
// n_folds columns of J output columns (thread t: fold t / J, column t % J)
// and adds their raw values in fold order in shared memory after the sweep.
template <int SG, int NS, bool FOLDSUM>
__global__ void __launch_bounds__(256, NS == 1 ? 3 : 2) k_folded_cols(FoldedView F, const float* __restrict__ xT, int B, int RT,
                                                     float* __restrict__ y) {
    constexpr int C = SG / 4;
    constexpr int ROWB = SG * 4;
    extern __shared__ __align__(16) unsigned char fc_smem[];
    const uint32_t raw32 = (uint32_t)__cvta_generic_to_shared(fc_smem);
    const uint32_t pad = (128u - (raw32 & 127u)) & 127u;
    float4* xs4 = reinterpret_cast<float4*>(fc_smem + pad);
    const uint32_t xs32 = raw32 + pad;
    float* vs_t = reinterpret_cast<float*>(xs4 + RT * C);     // [NS][RT]
    float* ftab = vs_t + NS * RT;
    if (threadIdx.x < 16) ftab[threadIdx.x] = fp4_decode(threadIdx.x);
    const int t = threadIdx.x;
    int64_t c;                  // stacked column of this thread
    bool live;
    int f = 0, jl = 0;
    if (FOLDSUM) {
        f = t / F.J;
        jl = t % F.J;
        const int64_t j = (int64_t)blockIdx.x * F.J + jl;
        live = f < F.n_folds && j < F.out_dim;
        c = (int64_t)f * F.out_dim + j;
    } else {
        c = (int64_t)blockIdx.x * blockDim.x + t;
        live = c < F.n_cols;
    }
    const int b0 = blockIdx.y * SG;
    const int n_in = F.n_in;
    const uint32_t rot16 = (t & (C - 1)) << 4;
    const int4 none = make_int4(n_in << 4, n_in << 4, n_in << 4, n_in << 4);
    int cur[NS], end[NS], pk[NS];
    int4 nb[NS], nb2[NS];
    float oc[NS];
    float acc[NS][SG];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        cur[s] = end[s] = 0;
        oc[s] = 0.0f;
        if (live) {
            cur[s] = F.colptr[s][c];
            end[s] = cur[s] + (F.colptr_x[s][c + 1] - F.colptr_x[s][c]);
            oc[s] = F.os[s][c];
        }
        const int4* cp4 = reinterpret_cast<const int4*>(F.cpack[s]);
        nb[s] = cur[s] < end[s] ? __ldg(cp4 + (cur[s] >> 2)) : none;
        nb2[s] = (cur[s] | 3) + 1 < end[s] ? __ldg(cp4 + (cur[s] >> 2) + 1) : none;
        const int k = cur[s] & 3;
        pk[s] = k == 0 ? nb[s].x : k == 1 ? nb[s].y : k == 2 ? nb[s].z : nb[s].w;
#pragma unroll
        for (int v = 0; v < SG; ++v) acc[s][v] = 0.0f;
    }
    for (int R0 = 0; R0 < n_in; R0 += RT) {
        const int nr = min(RT, n_in - R0), R1 = R0 + nr;
        __syncthreads();
        for (int u = t; u < nr * C; u += blockDim.x) {
            const int i = u / C, q = u % C;
            const int b = b0 + 4 * q;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (b < B) v = __ldg(reinterpret_cast<const float4*>(xT + (int64_t)(R0 + i) * B + b));
            xs4[i * C + q] = v;
        }
#pragma unroll
        for (int s = 0; s < NS; ++s)
            for (int i = t; i < nr; i += blockDim.x) vs_t[s * RT + i] = __ldg(F.vs[s] + R0 + i);
        __syncthreads();
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            const int4* cp4 = reinterpret_cast<const int4*>(F.cpack[s]);
            while (cur[s] < end[s] && (pk[s] >> 4) < R1) {
                const int ri = (pk[s] >> 4) - R0, code = pk[s] & 15;
                ++cur[s];
                if ((cur[s] & 3) == 0) {
                    nb[s] = nb2[s];
                    nb2[s] = cur[s] + 4 < end[s] ? __ldg(cp4 + (cur[s] >> 2) + 1) : none;
                }
                const int k = cur[s] & 3;
                pk[s] = cur[s] < end[s] ? (k == 0 ? nb[s].x : k == 1 ? nb[s].y : k == 2 ? nb[s].z : nb[s].w)
                                        : (n_in << 4);
                const float w = __fmul_rn(ftab[code], __fmaf_rn(vs_t[s * RT + ri], oc[s], 0.0f));
                const uint32_t rowa = (xs32 + (uint32_t)ri * ROWB) ^ rot16;
                if (isfinite(w)) {
#pragma unroll
                    for (int q = 0; q < C; ++q) {
                        const float4 xv = lds128(rowa ^ ((uint32_t)q << 4));
                        acc[s][4 * q + 0] = __fmaf_rn(w, xv.x, acc[s][4 * q + 0]);
                        acc[s][4 * q + 1] = __fmaf_rn(w, xv.y, acc[s][4 * q + 1]);
                        acc[s][4 * q + 2] = __fmaf_rn(w, xv.z, acc[s][4 * q + 2]);
                        acc[s][4 * q + 3] = __fmaf_rn(w, xv.w, acc[s][4 * q + 3]);
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < C; ++q) {
                        const float4 xv = lds128(rowa ^ ((uint32_t)q << 4));
                        const float xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            if (xq[v] != 0.0f) acc[s][4 * q + v] = __fmaf_rn(w, xq[v], acc[s][4 * q + v]);
                    }
                }
            }
        }
    }
    // the suffix sum, in suffix order from 0 (Python's sum)
    float raw[SG];
#pragma unroll
    for (int v = 0; v < SG; ++v) {
        float r = __fadd_rn(0.0f, acc[0][v]);
#pragma unroll
        for (int s = 1; s < NS; ++s) r = __fadd_rn(r, acc[s][v]);
        raw[v] = r;
    }
    const int rot = t & (C - 1);
    if (!FOLDSUM) {
        if (live) {
#pragma unroll
            for (int k = 0; k < SG; ++k) {
                const int b = b0 + 4 * ((k >> 2) ^ rot) + (k & 3);
                if (b < B) y[(int64_t)b * F.n_cols + c] = raw[k];
            }
        }
        return;
    }
    // fold sum through shared memory: red[f][jl][sample], then thread
    // (jl, sample) adds its column's folds in order
    __syncthreads();
    float* red = reinterpret_cast<float*>(fc_smem + pad);
    if (live) {
#pragma unroll
        for (int k = 0; k < SG; ++k) red[((int64_t)f * F.J + jl) * SG + 4 * ((k >> 2) ^ rot) + (k & 3)] = raw[k];
    }
    __syncthreads();
    for (int u = t; u < F.J * SG; u += blockDim.x) {
        const int jj = u / SG, v = u % SG;
        const int64_t j = (int64_t)blockIdx.x * F.J + jj;
        const int b = b0 + v;
        if (j >= F.out_dim || b >= B) continue;
        float a = red[(int64_t)jj * SG + v];
        for (int ff = 1; ff < F.n_folds; ++ff) a = __fadd_rn(a, red[((int64_t)ff * F.J + jj) * SG + v]);
        y[(int64_t)b * F.out_dim + j] = a;
    }
}

bool folded_forward_applies(const FoldedView& F, int B) {
    if (F.ns < 1 || F.ns > kFoldedMaxSuffixes || B < 16 || (B & 3) != 0 || F.n_in >= (1 << 27) || F.n_in <= 0) return false;
    if (F.fold_sum && F.n_folds > 256) return false;
    return F.n_cols > 0;
}

template <int SG, int NS, bool FS>
void folded_launch(dim3 g, int threads, size_t smem, const FoldedView& F, const float* xT, int B, int RT, float* y,
                   cudaStream_t s) {
    static unsigned long long attr_devices = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(attr_devices & (1ull << dev))) {
        cudaFuncSetAttribute(k_folded_cols<SG, NS, FS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr_devices |= 1ull << dev;
    }
    k_folded_cols<SG, NS, FS><<<g, threads, smem, s>>>(F, xT, B, RT, y);
}

template <int SG, int NS>
void folded_launch_fs(dim3 g, int threads, size_t smem, const FoldedView& F, const float* xT, int B, int RT,
                      float* y, cudaStream_t s) {
    if (F.fold_sum) folded_launch<SG, NS, true>(g, threads, smem, F, xT, B, RT, y, s);
    else folded_launch<SG, NS, false>(g, threads, smem, F, xT, B, RT, y, s);
}

template <int SG>
void folded_launch_ns(dim3 g, int threads, size_t smem, const FoldedView& F, const float* xT, int B, int RT,
                      float* y, cudaStream_t s) {
    switch (F.ns) {
    case 1: folded_launch_fs<SG, 1>(g, threads, smem, F, xT, B, RT, y, s); break;
    case 2: folded_launch_fs<SG, 2>(g, threads, smem, F, xT, B, RT, y, s); break;
    case 3: folded_launch_fs<(SG > 16 ? 16 : SG), 3>(g, threads, smem, F, xT, B, RT, y, s); break;
    default: folded_launch_fs<(SG > 16 ? 16 : SG), 4>(g, threads, smem, F, xT, B, RT, y, s); break;
    }
}

bool launch_folded_forward(FoldedView F, const float* xT, int B, float* y, cudaStream_t s) {
    if (!folded_forward_applies(F, B)) return false;
    int threads;
    unsigned gx;
    if (F.fold_sum) {
        // J output columns per CTA, n_folds * J threads (at most 256)
        F.J = (int)std::max<int64_t>(1, std::min<int64_t>(F.out_dim, 256 / F.n_folds));
        threads = ((F.n_folds * F.J + 31) / 32) * 32;
        gx = (unsigned)((F.out_dim + F.J - 1) / F.J);
    } else {
        threads = 256;
        gx = (unsigned)((F.n_cols + threads - 1) / threads);
    }
    // samples per thread: the most (up to 32; 16 with three or four
    // suffixes, whose accumulators share the thread's registers) that still
    // gives two CTAs per SM -- a narrow column shard splits its samples
    // instead (measured on config 5's shards at 1-8 ranks); x tiles of 32 KB.
    // The tuning override of cols_plan applies its samples and tile rows here.
    int sg = F.ns >= 3 ? 16 : 32;
    while (sg > 4 && (int64_t)gx * ((B + sg - 1) / sg) < 2 * 148) sg >>= 1;
    int rt_max = 256 * 32 / sg / (F.ns > 1 ? 2 : 1);
    const PlanOverride& o = plan_override();
    if (o.set && !o.vec) {
        sg = F.ns >= 3 ? std::min(o.p.sg, 16) : o.p.sg;
        rt_max = o.p.rt;
    }
    const int rt = (int)std::min<int64_t>(F.n_in, rt_max);
    size_t smem = 128 + (size_t)rt * (sg * sizeof(float) + F.ns * sizeof(float)) + 16 * sizeof(float);
    if (F.fold_sum) smem = std::max(smem, 128 + (size_t)F.n_folds * F.J * sg * sizeof(float));
    dim3 g(gx, (unsigned)((B + sg - 1) / sg));
    switch (sg) {
    case 32: folded_launch_ns<32>(g, threads, smem, F, xT, B, rt, y, s); break;
    case 16: folded_launch_ns<16>(g, threads, smem, F, xT, B, rt, y, s); break;
    case 8: folded_launch_ns<8>(g, threads, smem, F, xT, B, rt, y, s); break;
    default: folded_launch_ns<4>(g, threads, smem, F, xT, B, rt, y, s); break;
    }
    count_launch();
    return true;
}

bool forward_rows_applies(const LayerView& L, int B) { return cols_plan(L, B).threads > 0; }

bool launch_forward_rows(const LayerView& L, const float* xT, int B, float* y, bool sparse, cudaStream_t s) {
    const ColsPlan p = cols_plan(L, B);
    if (p.threads == 0 || !L.cpack || !L.colptr_x) return false;
    const size_t smem = 128 + (size_t)p.rt * (p.sg * sizeof(float) + sizeof(float)) + 16 * sizeof(float);
    static unsigned long long attr_devices = 0;   // the attribute is per device and kernel
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(attr_devices & (1ull << dev))) {
        for (const void* f : {(const void*)k_forward_cols<false, 32>, (const void*)k_forward_cols<true, 32>,
                              (const void*)k_forward_cols<false, 16>, (const void*)k_forward_cols<true, 16>,
                              (const void*)k_forward_cols<false, 8>, (const void*)k_forward_cols<true, 8>,
                              (const void*)k_forward_cols<false, 4>, (const void*)k_forward_cols<true, 4>})
            cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        attr_devices |= 1ull << dev;
    }
    dim3 g((unsigned)((L.n_out + p.threads - 1) / p.threads), (unsigned)((B + p.sg - 1) / p.sg));
    if (sparse) launch_cols<true>(p, g, smem, L, xT, B, y, s);
    else launch_cols<false>(p, g, smem, L, xT, B, y, s);
    count_launch();
    return true;
}

}  // namespace sili
