// block4 kernels: 4x4 dense FP4 tiles (block4.hpp) beside the scattered
// delta-CSR synapses.  Loading (block4_load_dense), the forward part of
// disldo_forward (linear_disldo.hpp:128-339), the backward part of
// disldo_backward (linear_disldo.hpp:939-1951) with the per-row workspace
// merge and its eviction (Block4Store::merge_row_workspace,
// block4.hpp:1368-1465), and the tile column index.
//
// Floating point: compiled with --fmad=false; each fused multiply-add and
// each horizontal-sum order below is the one the reference's own build
// evaluates (pinned through the CPU oracle against that build).
#include "common.cuh"
#include "kernels.cuh"
#include "update_math.cuh"

#include <algorithm>

namespace sili {

namespace {

__device__ __forceinline__ uint32_t tile_byte(const uint4& t, int s) {
    const uint32_t w = s < 8 ? (s < 4 ? t.x : t.y) : (s < 12 ? t.z : t.w);
    return (w >> ((s & 3) * 8)) & 0xFFu;
}
__device__ __forceinline__ void set_tile_byte(uint4& t, int s, uint32_t b) {
    const uint32_t sh = (uint32_t)(s & 3) * 8u, m = ~(0xFFu << sh), v = (b & 0xFFu) << sh;
    if (s < 4) t.x = (t.x & m) | v;
    else if (s < 8) t.y = (t.y & m) | v;
    else if (s < 12) t.z = (t.z & m) | v;
    else t.w = (t.w & m) | v;
}
// live slots (non-zero bytes) of a tile (Block4Tile::count_live, block4.hpp:314-319)
__device__ __forceinline__ int nz_bytes(uint32_t w) {
    const uint32_t t = ((w & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | w;
    return __popc(t & 0x80808080u);
}
__device__ __forceinline__ int tile_live(const uint4& t) {
    return nz_bytes(t.x) + nz_bytes(t.y) + nz_bytes(t.z) + nz_bytes(t.w);
}
// block4_stored_tile_len (block4.hpp:340-343, 386-388)
__device__ __forceinline__ int tile_len(int live, bool sparse) { return sparse ? 1 + (live + 1) / 2 + live : 16; }

// S(row, col) = sum_k value_scale_k(row) * output_scale_k(col)
// (SparseLinearWeightsDelta::get_scale, delta_csr_types.hpp:1235-1240)
__device__ __forceinline__ float scale_of(const LayerView& L, int64_t row, int64_t col) {
    float s = 0.0f;
    for (int k = 0; k < L.rank; ++k) s = __fmaf_rn(L.vs[row * L.rank + k], L.os[col * L.rank + k], s);
    return s;
}

}  // namespace

// ── load_dense_codes ────────────────────────────────────────────────────────
// block4_load_dense (delta_csr_memory.hpp:843-945): a tile for every
// (br, bc), bytes weight | importance << 4 straight from the codes, packed
// sparse when live <= switch_point (commit_dirty_sparse_tile of a new tile).
__global__ void k_b4_load_dense(const uint8_t* __restrict__ wc, const uint8_t* __restrict__ ic, int64_t n_in,
                                int64_t n_out, B4View V, unsigned long long* __restrict__ row_used) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= V.BR * V.BC) return;
    const int64_t br = t / V.BC, bc = t % V.BC;
    uint4 tile = make_uint4(0, 0, 0, 0);
    for (int li = 0; li < 4; ++li) {
        const int64_t row = br * 4 + li;
        if (row >= n_in) break;
        for (int lj = 0; lj < 4; ++lj) {
            const int64_t col = bc * 4 + lj;
            if (col >= n_out) break;
            const int64_t i = row * n_out + col;
            set_tile_byte(tile, lj * 4 + li, (uint32_t)(uint8_t)(wc[i] | (ic[i] << 4)));
        }
    }
    const int64_t slot = V.es[br] + bc;
    V.tile[slot] = tile;
    V.bc[slot] = (int)bc;
    const int live = tile_live(tile);
    const bool sp = (uint32_t)live <= V.switch_point;
    V.sparse[slot] = sp ? 1 : 0;
    atomicAdd(row_used + br, (unsigned long long)tile_len(live, sp));
}
void launch_b4_load_dense(const uint8_t* wc, const uint8_t* ic, int64_t n_in, int64_t n_out, const B4View& V,
                          int64_t* row_used, cudaStream_t s) {
    const int64_t n = V.BR * V.BC;
    if (n == 0) return;
    k_b4_load_dense<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(wc, ic, n_in, n_out, V,
                                                               reinterpret_cast<unsigned long long*>(row_used));
    count_launch();
}

// per block-row: packed tile bytes in use, ULEB128 bytes of the block-column
// deltas, live slots (for the allocation bookkeeping and Block4View)
__global__ void k_b4_row_used(B4View V, int64_t* __restrict__ out) {
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (br >= V.BR) return;
    long long u = 0, ib = 0, lv = 0;
    for (int e = lane; e < V.nt[br]; e += 32) {
        const int64_t ti = V.es[br] + e;
        const int live = tile_live(V.tile[ti]);
        u += tile_len(live, V.sparse[ti] != 0);
        lv += live;
        const uint32_t prev = e > 0 ? (uint32_t)V.bc[ti - 1] : 0u;
        uint32_t d = (uint32_t)V.bc[ti] - prev;
        int n = 0;
        do { d >>= 7; ++n; } while (d);
        ib += n;
    }
    u = warp_sum(u); ib = warp_sum(ib); lv = warp_sum(lv);
    if (lane == 0) { out[br] = u; out[V.BR + br] = ib; out[2 * V.BR + br] = lv; }
}
void launch_b4_row_used(const B4View& V, int64_t* out, cudaStream_t s) {
    if (V.BR == 0) return;
    k_b4_row_used<<<(unsigned)((V.BR + 7) / 8), 256, 0, s>>>(V, out);
    count_launch();
}

// ── forward ─────────────────────────────────────────────────────────────────
// One warp per block-column, lanes over batch samples.  Per tile, in
// ascending block-row (the reference's single-thread tile order), each of
// the 4 columns gets acc = fma(w0, x0, w1*x1) + fma(w2, x2, w3*x3) -- the
// reference build's evaluation of `acc += w4[li] * x` -- summed into a
// per-column total that is added to the scattered result at the end
// (linear_disldo.hpp:235-335).  Rows past n_in contribute 0 * x[b, 0].
__global__ void __launch_bounds__(128) k_b4_forward(LayerView L, B4View V, const float* __restrict__ xT, int B,
                                                    float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bcol = (int64_t)blockIdx.x * 4 + warp;
    const int b = blockIdx.y * 32 + lane;
    if (bcol >= V.BC) return;
    const bool bok = b < B;
    float mo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int64_t col0 = bcol * 4;
    // The slot weights w = fp4(code) * S(row, col) are the same for every
    // sample, so each is computed once per warp: lane l holds slot l & 15
    // (li = l & 3, lj = (l >> 2) & 3) of one of two tiles (l >> 4), and the
    // sums fetch them by shuffle.  S is scale_of's fused chain from 0.
    const int q = lane & 15, qli = q & 3, qlj = q >> 2;
    const bool qcol = col0 + qlj < L.n_out;
    float osq[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) osq[k] = (qcol && k < L.rank) ? L.os[(col0 + qlj) * L.rank + k] : 0.0f;
    const int t0 = V.cptr[bcol], t1 = V.cptr[bcol + 1];
    // four tiles at a time: their indices, bytes, x values and weights are
    // all in flight before the first tile's sums, which run in tile order
    constexpr int G = 4;
    for (int t = t0; t < t1; t += G) {
        int64_t br[G];
        int ct[G];
#pragma unroll
        for (int u = 0; u < G; ++u) {
            const bool ok = t + u < t1;
            ct[u] = ok ? V.ctile[t + u] : -1;
            br[u] = ok ? V.cbr[t + u] : 0;
        }
        float x[G][4], wl[G / 2];
#pragma unroll
        for (int u = 0; u < G; ++u)
#pragma unroll
            for (int li = 0; li < 4; ++li) {
                const int64_t row = br[u] * 4 + li;
                x[u][li] = (bok && ct[u] >= 0 && row < L.n_in) ? xT[row * B + b] : 0.0f;
            }
#pragma unroll
        for (int pr = 0; pr < G / 2; ++pr) {
            const int u = 2 * pr + (lane >> 4);
            const int cu = (lane >> 4) ? ct[2 * pr + 1] : ct[2 * pr];
            const int64_t bru = (lane >> 4) ? br[2 * pr + 1] : br[2 * pr];
            const int64_t row = bru * 4 + qli;
            float w = 0.0f;
            if (cu >= 0 && row < L.n_in) {
                const uint4 tw = V.tile[cu];
                float sc = 0.0f;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (k < L.rank) sc = __fmaf_rn(L.vs[row * L.rank + k], osq[k], sc);
                w = __fmul_rn(fp4_decode(tile_byte(tw, q) & 0xFu), sc);
            }
            wl[pr] = w;
            (void)u;
        }
#pragma unroll
        for (int u = 0; u < G; ++u) {
            if (ct[u] < 0) break;
            const int src = (u & 1) << 4;
#pragma unroll
            for (int lj = 0; lj < 4; ++lj) {
                float w[4];
#pragma unroll
                for (int li = 0; li < 4; ++li) w[li] = __shfl_sync(0xffffffffu, wl[u >> 1], src | (lj * 4 + li));
                if (col0 + lj >= L.n_out) continue;
                const float acc = __fadd_rn(__fmaf_rn(w[0], x[u][0], __fmul_rn(w[1], x[u][1])),
                                            __fmaf_rn(w[2], x[u][2], __fmul_rn(w[3], x[u][3])));
                mo[lj] = __fadd_rn(mo[lj], acc);
            }
        }
    }
    if (!bok) return;
#pragma unroll
    for (int lj = 0; lj < 4; ++lj) {
        const int64_t col = col0 + lj;
        if (col < L.n_out) {
            float* o = y + (int64_t)b * L.n_out + col;
            *o = __fadd_rn(*o, mo[lj]);
        }
    }
}
void launch_b4_forward(const LayerView& L, const B4View& V, const float* xT, int B, float* y, cudaStream_t s) {
    if (V.BC == 0 || B == 0) return;
    dim3 g((unsigned)((V.BC + 3) / 4), (unsigned)((B + 31) / 32));
    k_b4_forward<<<g, 128, 0, s>>>(L, V, xT, B, y);
    count_launch();
}

// ── dx at lr == 0 ───────────────────────────────────────────────────────────
// One warp per block-row, lanes over samples.  Per tile in stored order, row
// li adds quant*(S*dy) over its 4 columns: pairwise (p0+p1)+(p2+p3) for a
// tile of full width (Block4Vec path), a fused chain over the valid columns
// at the matrix edge (scalar path) -- linear_disldo.hpp:1512-1703.
__global__ void __launch_bounds__(128) k_b4_dx(LayerView L, B4View V, const float* __restrict__ dyT, int B,
                                               float* __restrict__ dx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t br = (int64_t)blockIdx.x * 4 + warp;
    const int b = blockIdx.y * 32 + lane;
    if (br >= V.BR) return;
    const bool bok = b < B;
    const int nt = V.nt[br];
    if (nt == 0) return;
    // each slot's weight code and scale S are the same for every sample:
    // lane l computes them for slot l & 15 of one of two tiles (l >> 4) and
    // the sample lanes fetch them by shuffle
    const int q = lane & 15, qli = q & 3, qlj = q >> 2;
    const int64_t es = V.es[br];
    float d[4];
#pragma unroll
    for (int li = 0; li < 4; ++li) {
        const int64_t row = br * 4 + li;
        d[li] = (bok && row < L.n_in) ? dx[(int64_t)b * L.n_in + row] : 0.0f;
    }
    for (int e = 0; e < nt; e += 2) {
        float qv = 0.0f, sv = 0.0f;
        {
            const int eu = e + (lane >> 4);
            if (eu < nt) {
                const int64_t tu = es + eu;
                const int64_t row = br * 4 + qli, col = (int64_t)V.bc[tu] * 4 + qlj;
                if (row < L.n_in && col < L.n_out) {
                    qv = fp4_decode(tile_byte(V.tile[tu], q) & 0xFu);
                    sv = scale_of(L, row, col);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (e + u >= nt) break;
            const int64_t ti = es + e + u;
            const int64_t col0 = (int64_t)V.bc[ti] * 4;
            const bool full = col0 + 4 <= L.n_out;
            const int src = u << 4;
            float dyv[4];
#pragma unroll
            for (int lj = 0; lj < 4; ++lj) dyv[lj] = (bok && col0 + lj < L.n_out) ? dyT[(col0 + lj) * B + b] : 0.0f;
#pragma unroll
            for (int li = 0; li < 4; ++li) {
                const int64_t row = br * 4 + li;
                if (row >= L.n_in) continue;
                if (full) {
                    float p[4];
#pragma unroll
                    for (int lj = 0; lj < 4; ++lj) {
                        const float qq = __shfl_sync(0xffffffffu, qv, src | (lj * 4 + li));
                        const float ss = __shfl_sync(0xffffffffu, sv, src | (lj * 4 + li));
                        p[lj] = __fmul_rn(qq, __fmul_rn(ss, dyv[lj]));
                    }
                    d[li] = __fadd_rn(d[li], __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])));
                } else {
                    for (int lj = 0; lj < 4; ++lj) {
                        if (col0 + lj >= L.n_out) continue;
                        const float qq = __shfl_sync(0xffffffffu, qv, src | (lj * 4 + li));
                        const float ss = __shfl_sync(0xffffffffu, sv, src | (lj * 4 + li));
                        d[li] = __fmaf_rn(qq, __fmul_rn(ss, dyv[lj]), d[li]);
                    }
                }
            }
        }
    }
    if (!bok) return;
#pragma unroll
    for (int li = 0; li < 4; ++li) {
        const int64_t row = br * 4 + li;
        if (row < L.n_in) dx[(int64_t)b * L.n_in + row] = d[li];
    }
}
void launch_b4_dx(const LayerView& L, const B4View& V, const float* dyT, int B, float* dx, cudaStream_t s) {
    if (V.BR == 0 || B == 0) return;
    dim3 g((unsigned)((V.BR + 3) / 4), (unsigned)((B + 31) / 32));
    k_b4_dx<<<g, 128, 0, s>>>(L, V, dyT, B, dx);
    count_launch();
}

// Block4Store::merge_row_workspace (block4.hpp:1368-1465) for one block-row,
// run by its half-warp.  The reference, while the packed bytes exceed the
// row's tile allocation, scans the row in (tile, li, lj) order for the live
// slot of smallest a = |importance * importance_scale * output_importance_
// scale| (the first live slot, replaced only by a strictly smaller a), zeroes
// it and repacks that tile.  Zeroing a slot changes no other slot's a, so
// without NaN importances the evictions are the live slots in ascending
// (a, tile, li, lj) order, stopped as soon as the row fits: here they are
// taken a level (one value of a) at a time, one tile per lane per step with a prefix
// sum of the tiles' byte savings, which gives the same slots, repacking and
// counters in O(levels x tiles) instead of O(evictions x tiles).  A NaN
// importance changes the reference's scan (a NaN first live slot is taken,
// later ones never are), so a row holding one is evicted one slot at a time
// exactly as the reference does.  Then tiles that still do not fit are
// counted.
__device__ __forceinline__ double b4_abs_imp(const LayerView& L, uint32_t byte, int64_t r, int64_t c) {
    return fabs((double)fp4_decode(byte >> 4) * (double)L.is[r] * (double)L.ois[c]);
}

template <int W>   // lanes per block-row: 16 (a half-warp) or 32
__device__ void b4_evict_row(const LayerView& L, const B4View& V, int64_t br, int64_t base, int nt, int s,
                             unsigned hmask) {
    const int64_t cap = V.alloc[V.BR + br];
    long long used = 0;
    for (int e = s; e < nt; e += W) used += tile_len(tile_live(V.tile[base + e]), V.sparse[base + e] != 0);
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) used += __shfl_xor_sync(hmask, used, o);
    if (used > cap) {
        bool nan_here = false;
        for (int e = s; e < nt && !nan_here; e += W) {
            const uint4 tw = V.tile[base + e];
            const int64_t c0 = (int64_t)V.bc[base + e] * 4;
            for (int q = 0; q < 16; ++q) {
                const uint32_t byte = tile_byte(tw, q);
                if (byte != 0 && isnan(b4_abs_imp(L, byte, br * 4 + (q & 3), c0 + (q >> 2)))) nan_here = true;
            }
        }
        if (__any_sync(hmask, nan_here)) {
            // the reference's scan, one eviction at a time (lane 0)
            if (s == 0) {
                while (used > cap) {
                    double best = -1.0;
                    int be = -1, bq = 0;
                    for (int e = 0; e < nt; ++e) {
                        const uint4 tw = V.tile[base + e];
                        const int64_t c0 = (int64_t)V.bc[base + e] * 4;
                        for (int l_i = 0; l_i < 4; ++l_i)
                            for (int l_j = 0; l_j < 4; ++l_j) {
                                const uint32_t byte = tile_byte(tw, l_j * 4 + l_i);
                                if (byte == 0) continue;
                                const double av = b4_abs_imp(L, byte, br * 4 + l_i, c0 + l_j);
                                if (best < 0.0 || av < best) { best = av; be = e; bq = l_j * 4 + l_i; }
                            }
                    }
                    if (be < 0) break;   // nothing live left
                    uint4 tw = V.tile[base + be];
                    const int old_len = tile_len(tile_live(tw), V.sparse[base + be] != 0);
                    set_tile_byte(tw, bq, 0u);
                    const int live = tile_live(tw);
                    const bool sp = (uint32_t)live <= V.switch_point;
                    used -= old_len - tile_len(live, sp);
                    V.tile[base + be] = tw;
                    V.sparse[base + be] = sp ? 1 : 0;
                }
            }
            used = __shfl_sync(hmask, used, W == 32 ? 0 : (int)(threadIdx.x & 16));
            __syncwarp(hmask);
        } else {
            while (used > cap) {
                // the smallest a among the live slots
                double amin = -1.0;
                for (int e = s; e < nt; e += W) {
                    const uint4 tw = V.tile[base + e];
                    const int64_t c0 = (int64_t)V.bc[base + e] * 4;
                    for (int q = 0; q < 16; ++q) {
                        const uint32_t byte = tile_byte(tw, q);
                        if (byte == 0) continue;
                        const double av = b4_abs_imp(L, byte, br * 4 + (q & 3), c0 + (q >> 2));
                        if (amin < 0.0 || av < amin) amin = av;
                    }
                }
#pragma unroll
                for (int o = W / 2; o > 0; o >>= 1) {
                    const double ob = __shfl_xor_sync(hmask, amin, o);
                    if (ob >= 0.0 && (amin < 0.0 || ob < amin)) amin = ob;
                }
                if (amin < 0.0) break;   // nothing live left
                // its slots in (tile, li, lj) order, W tiles per step, while the row does not fit
                for (int e0 = 0; e0 < nt && used > cap; e0 += W) {
                    const int e = e0 + s;
                    uint4 tw = make_uint4(0u, 0u, 0u, 0u);
                    int live = 0, k = 0, old_len = 0;
                    int64_t c0 = 0;
                    if (e < nt) {
                        tw = V.tile[base + e];
                        c0 = (int64_t)V.bc[base + e] * 4;
                        live = tile_live(tw);
                        old_len = tile_len(live, V.sparse[base + e] != 0);
                        for (int q = 0; q < 16; ++q) {
                            const uint32_t byte = tile_byte(tw, q);
                            if (byte != 0 && b4_abs_imp(L, byte, br * 4 + (q & 3), c0 + (q >> 2)) == amin) ++k;
                        }
                    }
                    auto saving = [&](int j) {   // bytes saved by evicting j of this tile's level slots
                        const int lv = live - j;
                        return (long long)(old_len - tile_len(lv, (uint32_t)lv <= V.switch_point));
                    };
                    const long long d = k > 0 ? saving(k) : 0;
                    long long incl = d;
#pragma unroll
                    for (int o = 1; o < W; o <<= 1) {
                        const long long t = __shfl_up_sync(hmask, incl, o, W);
                        if (s >= o) incl += t;
                    }
                    const long long excl = incl - d, need = used - cap;
                    int take = 0;
                    if (k > 0 && excl < need) {
                        take = k;
                        for (int j = 1; j < k; ++j)
                            if (excl + saving(j) >= need) { take = j; break; }
                    }
                    long long applied = 0;
                    if (take > 0) {
                        int left = take;
                        for (int l_i = 0; l_i < 4 && left > 0; ++l_i)
                            for (int l_j = 0; l_j < 4 && left > 0; ++l_j) {
                                const int q = l_j * 4 + l_i;
                                const uint32_t byte = tile_byte(tw, q);
                                if (byte != 0 && b4_abs_imp(L, byte, br * 4 + l_i, c0 + l_j) == amin) {
                                    set_tile_byte(tw, q, 0u);
                                    --left;
                                }
                            }
                        const int lv = tile_live(tw);
                        V.tile[base + e] = tw;
                        V.sparse[base + e] = (uint32_t)lv <= V.switch_point ? 1 : 0;
                        applied = saving(take);
                    }
#pragma unroll
                    for (int o = W / 2; o > 0; o >>= 1) applied += __shfl_xor_sync(hmask, applied, o);
                    used -= applied;
                }
            }
        }
        __syncwarp(hmask);
    }
    if (s == 0) {
        // tiles that do not fit even after eviction (the reference counts them)
        long long fit = 0;
        int fitted = 0;
        for (int e = 0; e < nt; ++e) {
            const int tl = tile_len(tile_live(V.tile[base + e]), V.sparse[base + e] != 0);
            if (fit + tl > cap) break;
            fit += tl;
            ++fitted;
        }
        if (fitted < nt) {
            atomicAdd(V.counters + 1, 1ull);
            atomicAdd(V.counters + 2, (unsigned long long)(used - fit));
        }
    }
}

// ── backward with update (lr != 0) ─────────────────────────────────────────
// One half-warp per block-row; lane s (0..15) owns slot s of the current
// tile (li = s & 3, lj = s >> 2).  Tiles are processed in stored order; for
// each, every slot runs its per-sample recurrence (the scattered path's
// bounded RMSprop step, here over the tile's 4 columns as the reference's
// Block4Vec code does, linear_disldo.hpp:1497-1703) and the row's dx terms
// are combined with half-warp shuffles in the reference build's order:
//   dx   += (p0 + p1) + (p2 + p3),  p = quant * (S * dy)      (full width)
//   mrow += (double)((q0 + q2) + (q1 + q3)),  q = (qf * os) * g
// or sequential fused chains over the valid columns at the matrix edge.
// dx partial sums live in dbuf (shared memory when it fits, else dxT).
// After all tiles: canonical repacking, the row's eviction down to its tile
// byte allocation (merge_row_workspace) and the block4 value_scale step
// (linear_disldo.hpp:1882-1950).
template <int RANK, bool STOCH>
__global__ void __launch_bounds__(128) k_b4_update(LayerView L, B4View V, const float* __restrict__ xT,
                                                   const float* __restrict__ dyT, int B, UpdateParams P,
                                                   float* __restrict__ dxT, int use_smem) {
    extern __shared__ float sh_d[];
    const int lane = threadIdx.x & 31, half = lane >> 4, s = lane & 15;
    const int hw = (threadIdx.x >> 4);                     // half-warp within the block
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 4) + hw;
    const unsigned hmask = half ? 0xFFFF0000u : 0x0000FFFFu;
    if (br >= V.BR) return;
    const int nt = V.nt[br];
    if (nt == 0) return;
    const int li = s & 3, lj = s >> 2;
    const int64_t row = br * 4 + li;
    const bool row_ok = row < L.n_in;
    const bool leader = lj == 0;                           // lanes s = 0..3 own row li's sums
    float* dbuf = use_smem ? sh_d + (size_t)hw * 4 * B + (size_t)li * B : dxT + (row_ok ? row : 0) * B;
    if (use_smem && leader && row_ok)
        for (int b = 0; b < B; ++b) dbuf[b] = dxT[row * B + b];
    __syncwarp(hmask);
    const uint32_t nnz_row = (uint32_t)nt * 4u;
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)nnz_row) : P.lr;
    const float onem = __fsub_rn(1.0f, P.beta2);
    float vsk[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) vsk[k] = row_ok ? L.vs[row * RANK + k] : 0.0f;
    const float isr = row_ok ? L.is[row] : 0.0f;
    double trg[RANK], trc[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) { trg[k] = 0.0; trc[k] = 0.0; }
    const int64_t base = V.es[br];
    for (int e = 0; e < nt; ++e) {
        const int64_t ti = base + e;
        uint4 tw = V.tile[ti];
        const int64_t col0 = (int64_t)V.bc[ti] * 4, col = col0 + lj;
        const bool col_ok = col < L.n_out;
        const bool act = row_ok && col_ok;
        const bool full = col0 + 4 <= L.n_out;
        const uint32_t byte = tile_byte(tw, s);
        float osk[RANK];
        float S = 0.0f;
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            osk[k] = col_ok ? L.os[col * RANK + k] : 0.0f;
            S = __fmaf_rn(vsk[k], osk[k], S);
        }
        if (!act) S = 0.0f;
        const float cis = act ? __fmul_rn(isr, L.ois[col]) : 0.0f;
        const float qorig = act ? fp4_decode(byte & 0xFu) : 0.0f;
        float quant = qorig;
        float ci = act ? __fmul_rn(fp4_decode(byte >> 4), cis) : 0.0f;
        float mcol[RANK], mcolc[RANK];
        double mrow[RANK], mrowc[RANK];
#pragma unroll
        for (int k = 0; k < RANK; ++k) { mcol[k] = mcolc[k] = 0.0f; mrow[k] = mrowc[k] = 0.0; }
        for (int b = 0; b < B; ++b) {
            const float x = row_ok ? xT[row * B + b] : 0.0f;
            const float dy = col_ok ? dyT[col * B + b] : 0.0f;
            const float g = __fmul_rn(dy, x);
            float cb = 0.0f, qf = 0.0f;
            if (act) {
                cb = __fmul_rn(qorig, x);
                ci = bounded_ci(ci, g, cb, P.beta2, onem);
                const float ngS = __fmul_rn(-g, S);
                float raw = P.damp ? __fdiv_rn(ngS, __fadd_rn(__fsqrt_rn(ci), P.eps)) : ngS;
                if (raw > 2.0f) raw = 2.0f;
                if (raw < -2.0f) raw = -2.0f;
                quant = __fmaf_rn(eff_lr, raw, quant);
                qf = (quant == 0.0f) ? 0.1f : quant;
            }
            const float sdy = __fmul_rn(S, dy);
            if (full) {
#pragma unroll
                for (int k = 0; k < RANK; ++k) {
                    const float qo = __fmul_rn(qf, osk[k]);
                    const float pg = __fmul_rn(qo, g), pc = __fmul_rn(qo, cb);
                    const float ag = __fadd_rn(pg, __shfl_xor_sync(hmask, pg, 8));
                    const float ac = __fadd_rn(pc, __shfl_xor_sync(hmask, pc, 8));
                    const float hg = __fadd_rn(ag, __shfl_xor_sync(hmask, ag, 4));
                    const float hc = __fadd_rn(ac, __shfl_xor_sync(hmask, ac, 4));
                    mrow[k] = __dadd_rn(mrow[k], (double)hg);
                    mrowc[k] = __dadd_rn(mrowc[k], (double)hc);
                    mcol[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), g, mcol[k]);
                    mcolc[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), cb, mcolc[k]);
                }
                const float p = __fmul_rn(quant, sdy);
                const float a = __fadd_rn(p, __shfl_xor_sync(hmask, p, 4));
                const float hs = __fadd_rn(a, __shfl_xor_sync(hmask, a, 8));
                if (leader && row_ok) dbuf[b] = __fadd_rn(dbuf[b], hs);
            } else {
                // matrix-edge tile: sequential fused chains over the valid columns
                const int src0 = (lane & 16) | li;
                float dsum = leader && row_ok ? dbuf[b] : 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int src = src0 + 4 * j;
                    const float qj = __shfl_sync(hmask, quant, src);
                    const float tj = __shfl_sync(hmask, sdy, src);
                    const float qfj = __shfl_sync(hmask, qf, src);
                    const float gj = __shfl_sync(hmask, g, src);
                    const float cj = __shfl_sync(hmask, cb, src);
                    const int okj = __shfl_sync(hmask, (int)col_ok, src);
                    if (okj) {
#pragma unroll
                        for (int k = 0; k < RANK; ++k) {
                            const float osj = __shfl_sync(hmask, osk[k], src);
                            const double qo = (double)qfj * (double)osj;
                            mrow[k] = __fma_rn(qo, (double)gj, mrow[k]);
                            mrowc[k] = __fma_rn(qo, (double)cj, mrowc[k]);
                        }
                        dsum = __fmaf_rn(qj, tj, dsum);
                    } else {
#pragma unroll
                        for (int k = 0; k < RANK; ++k) (void)__shfl_sync(hmask, osk[k], src);
                    }
                }
#pragma unroll
                for (int k = 0; k < RANK; ++k) {
                    mcol[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), g, mcol[k]);
                    mcolc[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), cb, mcolc[k]);
                }
                if (leader && row_ok) dbuf[b] = dsum;
            }
        }
        __syncwarp(hmask);
        // per-tile sums into the row's totals (t_row_grad), in tile order
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            trg[k] = __dadd_rn(trg[k], mrow[k]);
            trc[k] = __dadd_rn(trc[k], mrowc[k]);
        }
        if (act && P.os_trainable) {
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                atomicAdd(P.colg + col * RANK + k, mcol[k]);
                atomicAdd(P.colc + col * RANK + k, mcolc[k]);
            }
        }
        // re-quantize the slot (deterministic set or stochastic draw)
        if (act) {
            const float imp_ratio = __fdiv_rn(ci, cis);
            uint32_t wq, iq;
            if (STOCH) {
                const uint64_t el = (1ULL << 61) | ((uint64_t)row * (uint64_t)L.n_out + (uint64_t)col);
                wq = fp4_quantize_stochastic(quant, rng_draw(P.call_key, el, 0));
                iq = fp4_quantize_stochastic(imp_ratio, rng_draw(P.call_key, el, 1));
            } else {
                wq = fp4_encode(quant);
                iq = fp4_encode(imp_ratio);
            }
            set_tile_byte(tw, s, (iq << 4) | wq);
        }
        // gather the 16 bytes back into one tile word (lane s holds slot s)
        const uint32_t mine = tile_byte(tw, s);
        uint32_t words[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) w |= __shfl_sync(hmask, mine, (lane & 16) | (q * 4 + k)) << (8 * k);
            words[q] = w;
        }
        if (s == 0) {
            const uint4 nw = make_uint4(words[0], words[1], words[2], words[3]);
            V.tile[ti] = nw;
            V.sparse[ti] = (uint32_t)tile_live(nw) <= V.switch_point ? 1 : 0;
        }
        __syncwarp(hmask);
    }
    b4_evict_row<16>(L, V, br, base, nt, s, hmask);
    // ── block4 value_scale step and dx write-back (leader lane of each row) ──
    if (leader && row_ok) {
        const float scale_eff_lr = __fdiv_rn(P.lr, (float)nnz_row);
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            if (trg[k] == 0.0 && trc[k] == 0.0) continue;
            const int64_t i = row * RANK + k;
            rmsprop_scale(L.vs + i, L.vsi + i, (float)trg[k], scale_eff_lr, (float)trc[k], L.vstep + i, P);
        }
        if (use_smem)
            for (int b = 0; b < B; ++b) dxT[row * B + b] = dbuf[b];
    }
}

// ── the same update with tiles in parallel (every tile full: n_out % 4 == 0) ─
// Within a block-row only two things chain the tiles: the row's dx, an
// ordered fadd over its tiles' per-sample sums hs = (p0 + p1) + (p2 + p3),
// and the row's value_scale sums, an ordered dadd over the tiles' per-tile
// double sums.  Each tile's own recurrence (its 16 slots over the samples)
// depends on nothing outside it.  So the update runs as
//   k_b4_update_tiles: a half-warp per tile, 8 per block-row at a time,
//     writing the tile's new bytes, its hs[4 rows][B] and its per-row
//     double sums to scratch;
//   k_b4_rows_chain: a warp per row, the ordered chains over the tiles
//     (dx in place, then the value_scale step from the totals);
//   k_b4_evict_rows: a warp per block-row, the eviction.
// Same values, same order of every sum as k_b4_update, with all tiles of
// the layer's block-rows in flight instead of one half-warp per block-row.
constexpr int kB4Group = 64;   // tiles per block of k_b4_update_tiles
// OST: the output scale trains (per-slot column sums are kept)
template <int RANK, bool STOCH, bool OST>
__global__ void __launch_bounds__(128) k_b4_update_tiles(LayerView L, B4View V, const float* __restrict__ xT,
                                                         const float* __restrict__ dyT, int B, UpdateParams P,
                                                         int64_t br0, int64_t part_base, float* __restrict__ hsb,
                                                         double* __restrict__ mrb, float* __restrict__ mcb) {
    const int lane = threadIdx.x & 31, half = lane >> 4, s = lane & 15;
    const int hw = threadIdx.x >> 4;                     // 8 half-warps per block
    const int64_t br = br0 + blockIdx.y;                 // blockIdx.x: a group of kB4Group tiles
    const unsigned hmask = half ? 0xFFFF0000u : 0x0000FFFFu;
    if (br >= V.BR) return;
    const int nt = min(V.nt[br], (int)(blockIdx.x + 1) * kB4Group);
    const int li = s & 3, lj = s >> 2;
    const int64_t row = br * 4 + li;
    const bool row_ok = row < L.n_in;
    const bool leader = lj == 0;
    const uint32_t nnz_row = (uint32_t)V.nt[br] * 4u;
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)nnz_row) : P.lr;
    const float onem = __fsub_rn(1.0f, P.beta2);
    float vsk[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) vsk[k] = row_ok ? L.vs[row * RANK + k] : 0.0f;
    const float isr = row_ok ? L.is[row] : 0.0f;
    const int64_t base = V.es[br];
    for (int e = (int)blockIdx.x * kB4Group + hw; e < nt; e += 8) {
        const int64_t ti = base + e;
        const int64_t loc = ti - part_base;
        uint4 tw = V.tile[ti];
        const int64_t col = (int64_t)V.bc[ti] * 4 + lj;
        const bool act = row_ok;                         // every column of a full tile exists
        const uint32_t byte = tile_byte(tw, s);
        float osk[RANK];
        float S = 0.0f;
#pragma unroll
        for (int k = 0; k < RANK; ++k) {
            osk[k] = L.os[col * RANK + k];
            S = __fmaf_rn(vsk[k], osk[k], S);
        }
        if (!act) S = 0.0f;
        const float cis = act ? __fmul_rn(isr, L.ois[col]) : 0.0f;
        const float qorig = act ? fp4_decode(byte & 0xFu) : 0.0f;
        float quant = qorig;
        float ci = act ? __fmul_rn(fp4_decode(byte >> 4), cis) : 0.0f;
        float mcol[RANK], mcolc[RANK];
        double mrow[RANK], mrowc[RANK];
#pragma unroll
        for (int k = 0; k < RANK; ++k) { mcol[k] = mcolc[k] = 0.0f; mrow[k] = mrowc[k] = 0.0; }
        float* hrow = hsb + (loc * 4 + li) * (int64_t)B;
#pragma unroll 4
        for (int b = 0; b < B; ++b) {
            const float x = row_ok ? xT[row * B + b] : 0.0f;
            const float dy = dyT[col * B + b];
            const float g = __fmul_rn(dy, x);
            float cb = 0.0f, qf = 0.0f;
            if (act) {
                cb = __fmul_rn(qorig, x);
                ci = bounded_ci(ci, g, cb, P.beta2, onem);
                const float ngS = __fmul_rn(-g, S);
                float raw = P.damp ? __fdiv_rn(ngS, __fadd_rn(__fsqrt_rn(ci), P.eps)) : ngS;
                if (raw > 2.0f) raw = 2.0f;
                if (raw < -2.0f) raw = -2.0f;
                quant = __fmaf_rn(eff_lr, raw, quant);
                qf = (quant == 0.0f) ? 0.1f : quant;
            }
            const float sdy = __fmul_rn(S, dy);
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                const float qo = __fmul_rn(qf, osk[k]);
                const float pg = __fmul_rn(qo, g), pc = __fmul_rn(qo, cb);
                const float ag = __fadd_rn(pg, __shfl_xor_sync(hmask, pg, 8));
                const float ac = __fadd_rn(pc, __shfl_xor_sync(hmask, pc, 8));
                const float hg = __fadd_rn(ag, __shfl_xor_sync(hmask, ag, 4));
                const float hc = __fadd_rn(ac, __shfl_xor_sync(hmask, ac, 4));
                mrow[k] = __dadd_rn(mrow[k], (double)hg);
                mrowc[k] = __dadd_rn(mrowc[k], (double)hc);
                if (OST) {
                    mcol[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), g, mcol[k]);
                    mcolc[k] = __fmaf_rn(__fmul_rn(qf, vsk[k]), cb, mcolc[k]);
                }
            }
            const float p = __fmul_rn(quant, sdy);
            const float a = __fadd_rn(p, __shfl_xor_sync(hmask, p, 4));
            const float hs = __fadd_rn(a, __shfl_xor_sync(hmask, a, 8));
            if (leader) hrow[b] = hs;
        }
        if (leader) {
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                mrb[((loc * 4 + li) * RANK + k) * 2] = mrow[k];
                mrb[((loc * 4 + li) * RANK + k) * 2 + 1] = mrowc[k];
            }
        }
        if (OST) {   // the slot's column sums, added in order by k_b4_col_sums
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                mcb[((loc * 16 + s) * RANK + k) * 2] = act ? mcol[k] : 0.0f;
                mcb[((loc * 16 + s) * RANK + k) * 2 + 1] = act ? mcolc[k] : 0.0f;
            }
        }
        if (act) {
            const float imp_ratio = __fdiv_rn(ci, cis);
            uint32_t wq, iq;
            if (STOCH) {
                const uint64_t el = (1ULL << 61) | ((uint64_t)row * (uint64_t)L.n_out + (uint64_t)col);
                wq = fp4_quantize_stochastic(quant, rng_draw(P.call_key, el, 0));
                iq = fp4_quantize_stochastic(imp_ratio, rng_draw(P.call_key, el, 1));
            } else {
                wq = fp4_encode(quant);
                iq = fp4_encode(imp_ratio);
            }
            set_tile_byte(tw, s, (iq << 4) | wq);
        }
        const uint32_t mine = tile_byte(tw, s);
        uint32_t words[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) w |= __shfl_sync(hmask, mine, (lane & 16) | (q * 4 + k)) << (8 * k);
            words[q] = w;
        }
        if (s == 0) {
            const uint4 nw = make_uint4(words[0], words[1], words[2], words[3]);
            V.tile[ti] = nw;
            V.sparse[ti] = (uint32_t)tile_live(nw) <= V.switch_point ? 1 : 0;
        }
    }
}

// output_scale gradient sums of the chunk's tiles, one thread per column, in
// the reference's order: block-rows ascending (the tile column index lists
// each block-column's tiles so), rows li ascending within a tile
template <int RANK>
__global__ void k_b4_col_sums(LayerView L, B4View V, int64_t br0, int64_t br1, int64_t part_base,
                              const float* __restrict__ mcb, float* __restrict__ colg, float* __restrict__ colc) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= L.n_out) return;
    const int64_t bcol = c >> 2;
    const int lj = (int)(c & 3);
    float g[RANK], h[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) { g[k] = colg[c * RANK + k]; h[k] = colc[c * RANK + k]; }
    for (int t = V.cptr[bcol]; t < V.cptr[bcol + 1]; ++t) {
        const int64_t br = V.cbr[t];
        if (br < br0) continue;
        if (br >= br1) break;
        const int64_t loc = (int64_t)V.ctile[t] - part_base;
        for (int li = 0; li < 4; ++li) {
            if (br * 4 + li >= L.n_in) break;
            const float* m = mcb + ((loc * 16 + lj * 4 + li) * RANK) * 2;
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                g[k] = __fadd_rn(g[k], m[2 * k]);
                h[k] = __fadd_rn(h[k], m[2 * k + 1]);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < RANK; ++k) { colg[c * RANK + k] = g[k]; colc[c * RANK + k] = h[k]; }
}

// the ordered chains of one row over its block-row's tiles (a warp per row):
// dx[b] = ((dx[b] + hs_0[b]) + hs_1[b]) + ..., the value_scale totals
// likewise in double, then the block4 value_scale step (linear_disldo.hpp:1882-1950)
template <int RANK>
__global__ void __launch_bounds__(128) k_b4_rows_chain(LayerView L, B4View V, int B, UpdateParams P, int64_t br0,
                                                       int64_t br1, int64_t part_base,
                                                       const float* __restrict__ hsb, const double* __restrict__ mrb,
                                                       float* __restrict__ dxT) {
    const int lane = threadIdx.x & 31;
    const int64_t row = br0 * 4 + (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int64_t br = row >> 2;
    const int li = (int)(row & 3);
    if (br >= br1 || row >= L.n_in) return;
    const int nt = V.nt[br];
    if (nt == 0) return;
    const int64_t loc0 = V.es[br] - part_base;
    const int64_t stride = (int64_t)4 * B;
    for (int b = lane; b < B; b += 32) {
        float acc = dxT[row * B + b];
        const float* h = hsb + (loc0 * 4 + li) * (int64_t)B + b;
        int e = 0;
        for (; e + 8 <= nt; e += 8) {   // eight loads in flight, then the ordered adds
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = h[(int64_t)(e + u) * stride];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
        }
        for (; e < nt; ++e) acc = __fadd_rn(acc, h[(int64_t)e * stride]);
        dxT[row * B + b] = acc;
    }
    if (lane < RANK) {
        const int k = lane;
        double trg = 0.0, trc = 0.0;
        const double* m = mrb + ((loc0 * 4 + li) * RANK + k) * 2;
        for (int e = 0; e < nt; ++e) {
            trg = __dadd_rn(trg, m[(int64_t)e * 4 * RANK * 2]);
            trc = __dadd_rn(trc, m[(int64_t)e * 4 * RANK * 2 + 1]);
        }
        if (trg != 0.0 || trc != 0.0) {
            const float scale_eff_lr = __fdiv_rn(P.lr, (float)((uint32_t)nt * 4u));
            const int64_t i = row * RANK + k;
            rmsprop_scale(L.vs + i, L.vsi + i, (float)trg, scale_eff_lr, (float)trc, L.vstep + i, P);
        }
    }
}

// The importance magnitudes a of a tile's 16 slots, indexed li * 4 + lj (the
// eviction's scan order), -1 for empty slots.  a = |dec(imp)| * m[li][lj]
// with m = |is[r]| * |ois[c]| in double: every factor has at most 24
// significant bits (dec at most 2), so each product is exact and equals
// b4_abs_imp's, which multiplies in another order; it is NaN exactly when
// b4_abs_imp's is (a NaN factor, or 0 times infinity in either order).
__device__ __forceinline__ void b4_tile_levels(const uint4& tw, const double isd[4], const double oisd[4],
                                               double a[16]) {
    const uint32_t wd[4] = {tw.x, tw.y, tw.z, tw.w};
#pragma unroll
    for (int li = 0; li < 4; ++li)
#pragma unroll
        for (int lj = 0; lj < 4; ++lj) {
            const uint32_t byte = (wd[lj] >> (8 * li)) & 0xFFu;
            const double mag = (double)fabsf(fp4_decode(byte >> 4));
            a[li * 4 + lj] = byte ? mag * (isd[li] * oisd[lj]) : -1.0;
        }
}
// the smaller of two levels, -1 meaning none
__device__ __forceinline__ double b4_lvl_min(double m, double a) { return (a >= 0.0 && (m < 0.0 || a < m)) ? a : m; }

// The eviction of one block-row by a full warp: the same evictions, repacking
// and counters as b4_evict_row, organised for rows of many tiles:
//   * the packed flags are first refreshed from the tiles' live counts (the
//     warp-per-row update writes slot bytes only; for tiles whose flags are
//     current this rewrites the same values);
//   * each slot's a is computed from registers (b4_tile_levels) instead of
//     two global loads per slot;
//   * one walk per importance level, which also finds the next level (the
//     smallest a above the current one; every slot at the current level has
//     been evicted when a walk ends with the row still too long);
//   * the fit count at the end by a warp prefix sum over the tiles.
// A row holding a NaN importance takes b4_evict_row's one-at-a-time path.
__device__ void b4_evict_row_warp(const LayerView& L, const B4View& V, int64_t br, int64_t base, int nt, int lane) {
    const unsigned full = 0xFFFFFFFFu;
    const int64_t cap = V.alloc[V.BR + br];
    double isd[4];
#pragma unroll
    for (int li = 0; li < 4; ++li) {
        const int64_t r = br * 4 + li;
        isd[li] = r < L.n_in ? fabs((double)L.is[r]) : 0.0;
    }
    auto ois_of = [&](int64_t c0, double oisd[4]) {
#pragma unroll
        for (int lj = 0; lj < 4; ++lj) oisd[lj] = c0 + lj < L.n_out ? fabs((double)L.ois[c0 + lj]) : 0.0;
    };
    long long used = 0;
    bool nan_here = false;
    double amin = -1.0;
    for (int e = lane; e < nt; e += 32) {
        const uint4 tw = V.tile[base + e];
        const int live = tile_live(tw);
        const bool sp = (uint32_t)live <= V.switch_point;
        V.sparse[base + e] = sp ? 1 : 0;
        used += tile_len(live, sp);
        double oisd[4], a[16];
        ois_of((int64_t)V.bc[base + e] * 4, oisd);
        b4_tile_levels(tw, isd, oisd, a);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            if (isnan(a[q])) nan_here = true;
            amin = b4_lvl_min(amin, a[q]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) used += __shfl_xor_sync(full, used, o);
    if (used <= cap) return;   // every tile fits
    if (__any_sync(full, nan_here)) {
        b4_evict_row<32>(L, V, br, base, nt, lane, full);
        return;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amin = b4_lvl_min(amin, __shfl_xor_sync(full, amin, o));
    while (used > cap && amin >= 0.0) {
        double nxt = -1.0;
        for (int e0 = 0; e0 < nt && used > cap; e0 += 32) {
            const int e = e0 + lane;
            uint4 tw = make_uint4(0u, 0u, 0u, 0u);
            int live = 0, k = 0, old_len = 0;
            uint32_t lvl = 0;   // this level's slots, bit li * 4 + lj
            if (e < nt) {
                tw = V.tile[base + e];
                double oisd[4], a[16];
                ois_of((int64_t)V.bc[base + e] * 4, oisd);
                b4_tile_levels(tw, isd, oisd, a);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    if (a[q] == amin) lvl |= 1u << q;
                    else if (a[q] > amin) nxt = b4_lvl_min(nxt, a[q]);
                }
                live = tile_live(tw);
                old_len = tile_len(live, V.sparse[base + e] != 0);
                k = __popc(lvl);
            }
            auto saving = [&](int j) {   // bytes saved by evicting j of this tile's level slots
                const int lv = live - j;
                return (long long)(old_len - tile_len(lv, (uint32_t)lv <= V.switch_point));
            };
            const long long d = k > 0 ? saving(k) : 0;
            long long incl = d;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long t = __shfl_up_sync(full, incl, o);
                if (lane >= o) incl += t;
            }
            const long long excl = incl - d, need = used - cap;
            int take = 0;
            if (k > 0 && excl < need) {
                take = k;
                for (int j = 1; j < k; ++j)
                    if (excl + saving(j) >= need) { take = j; break; }
            }
            long long applied = 0;
            if (take > 0) {
                uint32_t m = lvl;
                for (int j = 0; j < take; ++j) {
                    const int bit = __ffs(m) - 1;
                    m &= m - 1u;
                    set_tile_byte(tw, (bit & 3) * 4 + (bit >> 2), 0u);   // slot lj * 4 + li
                }
                const int lv = tile_live(tw);
                V.tile[base + e] = tw;
                V.sparse[base + e] = (uint32_t)lv <= V.switch_point ? 1 : 0;
                applied = saving(take);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) applied += __shfl_xor_sync(full, applied, o);
            used -= applied;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) nxt = b4_lvl_min(nxt, __shfl_xor_sync(full, nxt, o));
        amin = nxt;
    }
    // tiles that do not fit even after eviction (the reference counts them):
    // the first tile whose running length passes the allocation
    long long fit = 0;
    int fitted = nt;
    for (int e0 = 0; e0 < nt; e0 += 32) {
        const int e = e0 + lane;
        const long long tl = e < nt ? tile_len(tile_live(V.tile[base + e]), V.sparse[base + e] != 0) : 0;
        long long incl = tl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long t = __shfl_up_sync(full, incl, o);
            if (lane >= o) incl += t;
        }
        const unsigned over = __ballot_sync(full, e < nt && fit + incl > cap);
        if (over) {
            const int first = __ffs(over) - 1;
            fit += __shfl_sync(full, incl - tl, first);
            fitted = e0 + first;
            break;
        }
        fit += __shfl_sync(full, incl, 31);
    }
    if (lane == 0 && fitted < nt) {
        atomicAdd(V.counters + 1, 1ull);
        atomicAdd(V.counters + 2, (unsigned long long)(used - fit));
    }
}

// a warp per block-row (the update kernel's own eviction uses its half-warp)
__global__ void __launch_bounds__(128) k_b4_evict_rows(LayerView L, B4View V, int64_t br0, int64_t br1) {
    const int lane = threadIdx.x & 31;
    const int64_t br = br0 + (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (br >= br1) return;
    const int nt = V.nt[br];
    if (nt == 0) return;
    b4_evict_row_warp(L, V, br, V.es[br], nt, lane);
}

// ── the same update, a warp per row (every tile full, B % 4 == 0, B <= 128) ─
// The row's dx chain ((dx + hs_0) + hs_1) + ... runs in tile order for every
// sample, and each slot's recurrence runs in sample order; a warp that owns
// one row and walks its tiles 32 at a time (lane = tile, the thread holding
// the tile's 4 slots of that row) keeps both chains in registers, so the
// per-(tile, row, sample) sums hs never leave the SM and the tile passes need
// no scratch.  Per sample, with x[row, b] the same for the whole warp:
//   * x == 0 (and every slot of the warp in the range where the step reduces
//     to it -- finite scale, weight and importance state, ci in [0, 100],
//     dy finite, eps > 0): the step leaves quant and the value_scale sums
//     unchanged and ci = fma(beta2, ci, (1 - beta2) * 0), exactly as the
//     full step evaluates it (the same closed form as the scattered update);
//   * otherwise the full step, as k_b4_update_tiles;
//   * hs = (p0 + p1) + (p2 + p3), p = quant * (S * dy), goes to shared
//     memory, and after 32 samples the lanes (= samples) add the 32 tiles'
//     hs in tile order to the row's dx.
// The 4 warps of a CTA are the 4 rows of one block-row: they share a dy panel
// (the chunk's 128 columns x 32 samples) staged in shared memory by cp.async.
// The tile bytes are written a byte per slot; the packed flags are refreshed
// by k_b4_evict_rows.  Same values and the same order of every sum as
// k_b4_update_tiles + k_b4_rows_chain.
constexpr int kB4RowsPitch = 4 * 32 + 4;   // panel floats per tile (16-byte bank stagger)

__device__ __forceinline__ void b4_cp_async16(void* smem, const void* gmem) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem) : "memory");
}

// 6 blocks per SM at scale rank 1 (80 registers), 4 above (the per-slot
// state grows with the rank)
template <int RANK, bool STOCH, bool OST, int NB>
__global__ void __launch_bounds__(128, RANK == 1 ? 6 : 4) k_b4_update_rows(LayerView L, B4View V, const float* __restrict__ xT,
                                                           const float* __restrict__ dyT, int B, UpdateParams P,
                                                           int64_t br0, int64_t part_base, float* __restrict__ mcb,
                                                           float* __restrict__ dxT) {
    __shared__ __align__(16) float dyp[32 * kB4RowsPitch];   // [tile][column j][sample]
    __shared__ float hs_s[4][32][33];                          // [row][tile][sample]
    __shared__ __align__(16) float xs_s[4][NB * 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t br = br0 + blockIdx.x;
    const int li = warp;
    const int64_t row = br * 4 + li;
    const bool row_ok = row < L.n_in;   // warp-uniform; such warps only help stage the panels
    const int nt = V.nt[br];
    if (nt == 0) return;                // the whole block
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)((uint32_t)nt * 4u)) : P.lr;
    const float beta2 = P.beta2;
    const float onem = __fsub_rn(1.0f, beta2);
    const float zterm = __fmul_rn(onem, 0.0f);
    const bool fast_ok = (!P.damp || P.eps > 0.0f) && isfinite(eff_lr) && beta2 >= 0.0f && beta2 <= 1.0f &&
                         P.dy_flag != nullptr && *P.dy_flag != P.dy_tag;
    float vsk[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) vsk[k] = row_ok ? L.vs[row * RANK + k] : 0.0f;
    const float isr = row_ok ? L.is[row] : 0.0f;
    float* xs = xs_s[warp];
    for (int t = lane; t < NB * 32; t += 32) xs[t] = (row_ok && t < B) ? xT[row * B + t] : 0.0f;
    float acc[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int b = k * 32 + lane;
        acc[k] = (row_ok && b < B) ? dxT[row * B + b] : 0.0f;
    }
    double tg[RANK], tc[RANK];
#pragma unroll
    for (int k = 0; k < RANK; ++k) { tg[k] = 0.0; tc[k] = 0.0; }
    const int64_t base = V.es[br];
    const int nblk = (B + 31) >> 5;
    for (int e0 = 0; e0 < nt; e0 += 32) {
        const int n = min(32, nt - e0);
        const bool have = lane < n;
        const int64_t ti = base + e0 + (have ? lane : 0);
        const uint4 tw = V.tile[ti];
        const int64_t col0 = (int64_t)V.bc[ti] * 4;
        const uint32_t wd[4] = {tw.x, tw.y, tw.z, tw.w};   // word j: column j, byte li: row li
        float quant[4], ci[4], qo0[4], S[4], osk[4][RANK];
        float mc[4][RANK], mcc[4][RANK];
        bool fin0 = true;   // finite S and weight: the part of the fast condition fixed per chunk
        bool fin = true;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t byte = (wd[j] >> (8 * li)) & 0xFFu;
            const int64_t col = col0 + j;
            float sc = 0.0f;
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                osk[j][k] = L.os[col * RANK + k];
                sc = __fmaf_rn(vsk[k], osk[j][k], sc);
                mc[j][k] = 0.0f;
                mcc[j][k] = 0.0f;
            }
            S[j] = sc;
            const float cis = __fmul_rn(isr, L.ois[col]);
            qo0[j] = fp4_decode(byte & 0xFu);
            quant[j] = qo0[j];
            ci[j] = __fmul_rn(fp4_decode(byte >> 4), cis);
            fin0 = fin0 && isfinite(sc) && isfinite(qo0[j]);
            const float qf = (quant[j] == 0.0f) ? 0.1f : quant[j];
            fin = fin && ci[j] >= 0.0f && ci[j] <= 100.0f;
#pragma unroll
            for (int k = 0; k < RANK; ++k) {
                fin = fin && isfinite(__fmul_rn(qf, osk[j][k]));
                if (OST) fin = fin && isfinite(__fmul_rn(qf, vsk[k]));
            }
        }
        double mr[RANK], mrc[RANK];
#pragma unroll
        for (int k = 0; k < RANK; ++k) { mr[k] = 0.0; mrc[k] = 0.0; }
        bool wfast = fast_ok && __all_sync(0xffffffffu, !have || (fin0 && fin));
        for (int sb = 0; sb < nblk; ++sb) {
            const int t0 = sb * 32, nb = min(32, B - t0);
            __syncthreads();   // the previous panel's readers are done
            for (int q = threadIdx.x; q < 32 * 4 * 8; q += 128) {
                const int t = q >> 5, j = (q >> 3) & 3, g = q & 7;
                if (t < n && g * 4 < nb) {
                    const int64_t c = (int64_t)V.bc[base + e0 + t] * 4 + j;
                    b4_cp_async16(&dyp[t * kB4RowsPitch + j * 32 + g * 4], dyT + c * B + t0 + g * 4);
                }
            }
            asm volatile("cp.async.wait_all;\n" ::: "memory");
            __syncthreads();
            if (!row_ok) continue;
            float a = acc[0];
#pragma unroll
            for (int k = 1; k < NB; ++k)
                if (sb == k) a = acc[k];
            const float* dp = dyp + lane * kB4RowsPitch;
            float* hrow = hs_s[warp][lane];
            for (int u0 = 0; u0 < nb; u0 += 4) {
                const float4 x4 = *reinterpret_cast<const float4*>(xs + t0 + u0);
                float4 d4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) d4[j] = *reinterpret_cast<const float4*>(dp + j * 32 + u0);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float x = u == 0 ? x4.x : u == 1 ? x4.y : u == 2 ? x4.z : x4.w;
                    float dy[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) dy[j] = u == 0 ? d4[j].x : u == 1 ? d4[j].y : u == 2 ? d4[j].z : d4[j].w;
                    if (x == 0.0f && wfast) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) ci[j] = __fmaf_rn(beta2, ci[j], zterm);
                    } else {
                        float pg[4][RANK], pc[4][RANK];
                        bool f = fin0;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float g = __fmul_rn(dy[j], x);
                            const float cb = __fmul_rn(qo0[j], x);
                            ci[j] = bounded_ci(ci[j], g, cb, beta2, onem);
                            const float ngS = __fmul_rn(-g, S[j]);
                            float raw = P.damp ? __fdiv_rn(ngS, __fadd_rn(__fsqrt_rn(ci[j]), P.eps)) : ngS;
                            if (raw > 2.0f) raw = 2.0f;
                            if (raw < -2.0f) raw = -2.0f;
                            quant[j] = __fmaf_rn(eff_lr, raw, quant[j]);
                            const float qf = (quant[j] == 0.0f) ? 0.1f : quant[j];
                            f = f && ci[j] >= 0.0f && ci[j] <= 100.0f;
#pragma unroll
                            for (int k = 0; k < RANK; ++k) {
                                const float qo = __fmul_rn(qf, osk[j][k]);
                                pg[j][k] = __fmul_rn(qo, g);
                                pc[j][k] = __fmul_rn(qo, cb);
                                f = f && isfinite(qo);
                                if (OST) {
                                    const float qv = __fmul_rn(qf, vsk[k]);
                                    mc[j][k] = __fmaf_rn(qv, g, mc[j][k]);
                                    mcc[j][k] = __fmaf_rn(qv, cb, mcc[j][k]);
                                    f = f && isfinite(qv);
                                }
                            }
                        }
#pragma unroll
                        for (int k = 0; k < RANK; ++k) {
                            const float hg = __fadd_rn(__fadd_rn(pg[0][k], pg[2][k]), __fadd_rn(pg[1][k], pg[3][k]));
                            const float hc = __fadd_rn(__fadd_rn(pc[0][k], pc[2][k]), __fadd_rn(pc[1][k], pc[3][k]));
                            mr[k] = __dadd_rn(mr[k], (double)hg);
                            mrc[k] = __dadd_rn(mrc[k], (double)hc);
                        }
                        wfast = fast_ok && __all_sync(0xffffffffu, !have || f);
                    }
                    float p[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) p[j] = __fmul_rn(quant[j], __fmul_rn(S[j], dy[j]));
                    hrow[u0 + u] = __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3]));
                }
            }
            __syncwarp();
            // dx: lanes = samples, the chunk's tiles in stored order
            if (lane < nb)
                for (int l = 0; l < n; ++l) a = __fadd_rn(a, hs_s[warp][l][lane]);
#pragma unroll
            for (int k = 0; k < NB; ++k)
                if (sb == k) acc[k] = a;
            __syncwarp();
        }
        if (!row_ok) continue;
        if (have) {
            uint8_t* tb = reinterpret_cast<uint8_t*>(V.tile + ti);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t col = col0 + j;
                const float imp_ratio = __fdiv_rn(ci[j], __fmul_rn(isr, L.ois[col]));
                uint32_t wq, iq;
                if (STOCH) {
                    const uint64_t el = (1ULL << 61) | ((uint64_t)row * (uint64_t)L.n_out + (uint64_t)col);
                    wq = fp4_quantize_stochastic(quant[j], rng_draw(P.call_key, el, 0));
                    iq = fp4_quantize_stochastic(imp_ratio, rng_draw(P.call_key, el, 1));
                } else {
                    wq = fp4_encode(quant[j]);
                    iq = fp4_encode(imp_ratio);
                }
                tb[j * 4 + li] = (uint8_t)((iq << 4) | wq);
                if (OST) {
                    const int64_t loc = ti - part_base;
#pragma unroll
                    for (int k = 0; k < RANK; ++k) {
                        mcb[((loc * 16 + j * 4 + li) * RANK + k) * 2] = mc[j][k];
                        mcb[((loc * 16 + j * 4 + li) * RANK + k) * 2 + 1] = mcc[j][k];
                    }
                }
            }
        }
        // the row's value_scale totals: the tiles' double sums in stored order
#pragma unroll
        for (int k = 0; k < RANK; ++k)
            for (int l = 0; l < n; ++l) {
                tg[k] = __dadd_rn(tg[k], __shfl_sync(0xffffffffu, mr[k], l));
                tc[k] = __dadd_rn(tc[k], __shfl_sync(0xffffffffu, mrc[k], l));
            }
    }
    if (!row_ok) return;
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        const int b = k * 32 + lane;
        if (b < B) dxT[row * B + b] = acc[k];
    }
    if (lane == 0) {
        const float scale_eff_lr = __fdiv_rn(P.lr, (float)((uint32_t)nt * 4u));
#pragma unroll
        for (int k = 0; k < RANK; ++k)
            if (tg[k] != 0.0 || tc[k] != 0.0) {
                const int64_t i = row * RANK + k;
                rmsprop_scale(L.vs + i, L.vsi + i, (float)tg[k], scale_eff_lr, (float)tc[k], L.vstep + i, P);
            }
    }
}

bool b4_update_split_applies(const LayerView& L) { return L.n_out % 4 == 0; }

void launch_b4_update_split(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                            const UpdateParams& P, float* dxT, int64_t br0, int64_t br1, int64_t part_base,
                            float* hsb, double* mrb, float* mcb, cudaStream_t s) {
    if (br1 <= br0 || B == 0) return;
    const unsigned nbr = (unsigned)(br1 - br0);
    const dim3 tg((unsigned)((V.BC + kB4Group - 1) / kB4Group), nbr);   // a row holds at most BC tiles
#define SILI_B4S(R, ST)                                                                                     \
    do {                                                                                                   \
        if (P.os_trainable)                                                                                \
            k_b4_update_tiles<R, ST, true><<<tg, 128, 0, s>>>(L, V, xT, dyT, B, P, br0, part_base, hsb, mrb, mcb); \
        else                                                                                               \
            k_b4_update_tiles<R, ST, false><<<tg, 128, 0, s>>>(L, V, xT, dyT, B, P, br0, part_base, hsb, mrb, mcb); \
    } while (0)
    switch (L.rank * 2 + (P.stochastic ? 1 : 0)) {
        case 2: SILI_B4S(1, false); break;
        case 3: SILI_B4S(1, true); break;
        case 4: SILI_B4S(2, false); break;
        case 5: SILI_B4S(2, true); break;
        case 6: SILI_B4S(3, false); break;
        case 7: SILI_B4S(3, true); break;
        case 8: SILI_B4S(4, false); break;
        default: SILI_B4S(4, true); break;
    }
#undef SILI_B4S
    count_launch();
    if (P.os_trainable) {
        const unsigned cg = (unsigned)((L.n_out + 255) / 256);
        switch (L.rank) {
            case 1: k_b4_col_sums<1><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            case 2: k_b4_col_sums<2><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            case 3: k_b4_col_sums<3><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            default: k_b4_col_sums<4><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
        }
        count_launch();
    }
    switch (L.rank) {
        case 1: k_b4_rows_chain<1><<<nbr, 128, 0, s>>>(L, V, B, P, br0, br1, part_base, hsb, mrb, dxT); break;
        case 2: k_b4_rows_chain<2><<<nbr, 128, 0, s>>>(L, V, B, P, br0, br1, part_base, hsb, mrb, dxT); break;
        case 3: k_b4_rows_chain<3><<<nbr, 128, 0, s>>>(L, V, B, P, br0, br1, part_base, hsb, mrb, dxT); break;
        default: k_b4_rows_chain<4><<<nbr, 128, 0, s>>>(L, V, B, P, br0, br1, part_base, hsb, mrb, dxT); break;
    }
    count_launch();
}
// b4_relayout's move: block-row br's nt[br] tiles from old_es[br] to
// new_es[br] in the new arrays (a warp per block-row)
__global__ void k_b4_move(int64_t BR, const int64_t* __restrict__ old_es, const int64_t* __restrict__ new_es,
                          const int* __restrict__ nt, const int* __restrict__ bc, const uint4* __restrict__ tile,
                          const uint8_t* __restrict__ sp, int* __restrict__ nbc, uint4* __restrict__ ntile,
                          uint8_t* __restrict__ nsp) {
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (br >= BR) return;
    const int64_t o = old_es[br], d = new_es[br];
    for (int e = threadIdx.x & 31; e < nt[br]; e += 32) {
        nbc[d + e] = bc[o + e];
        ntile[d + e] = tile[o + e];
        nsp[d + e] = sp[o + e];
    }
}
void launch_b4_move(int64_t BR, const int64_t* old_es, const int64_t* new_es, const int* nt, const int* bc,
                    const uint4* tile, const uint8_t* sp, int* nbc, uint4* ntile, uint8_t* nsp, cudaStream_t s) {
    if (BR <= 0) return;
    k_b4_move<<<(unsigned)((BR + 7) / 8), 256, 0, s>>>(BR, old_es, new_es, nt, bc, tile, sp, nbc, ntile, nsp);
    count_launch();
}

bool b4_update_rows_applies(const LayerView& L, int B) { return L.n_out % 4 == 0 && B > 0 && B <= 128 && B % 4 == 0; }

void launch_b4_update_rows(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                           const UpdateParams& P, float* dxT, int64_t br0, int64_t br1, int64_t part_base,
                           float* mcb, cudaStream_t s) {
    if (br1 <= br0 || B == 0) return;
    const unsigned nbr = (unsigned)(br1 - br0);
#define SILI_B4R(R, ST, NBV)                                                                                \
    do {                                                                                                   \
        if (P.os_trainable)                                                                                \
            k_b4_update_rows<R, ST, true, NBV><<<nbr, 128, 0, s>>>(L, V, xT, dyT, B, P, br0, part_base, mcb, dxT); \
        else                                                                                               \
            k_b4_update_rows<R, ST, false, NBV><<<nbr, 128, 0, s>>>(L, V, xT, dyT, B, P, br0, part_base, mcb, dxT); \
    } while (0)
#define SILI_B4R_NB(R, ST)              \
    do {                                \
        if (B <= 64) SILI_B4R(R, ST, 2); \
        else SILI_B4R(R, ST, 4);         \
    } while (0)
    switch (L.rank * 2 + (P.stochastic ? 1 : 0)) {
        case 2: SILI_B4R_NB(1, false); break;
        case 3: SILI_B4R_NB(1, true); break;
        case 4: SILI_B4R_NB(2, false); break;
        case 5: SILI_B4R_NB(2, true); break;
        case 6: SILI_B4R_NB(3, false); break;
        case 7: SILI_B4R_NB(3, true); break;
        case 8: SILI_B4R_NB(4, false); break;
        default: SILI_B4R_NB(4, true); break;
    }
#undef SILI_B4R_NB
#undef SILI_B4R
    count_launch();
    if (P.os_trainable) {
        const unsigned cg = (unsigned)((L.n_out + 255) / 256);
        switch (L.rank) {
            case 1: k_b4_col_sums<1><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            case 2: k_b4_col_sums<2><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            case 3: k_b4_col_sums<3><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
            default: k_b4_col_sums<4><<<cg, 256, 0, s>>>(L, V, br0, br1, part_base, mcb, P.colg, P.colc); break;
        }
        count_launch();
    }
}

void launch_b4_evict_rows(const LayerView& L, const B4View& V, cudaStream_t s) {
    if (V.BR == 0) return;
    k_b4_evict_rows<<<(unsigned)((V.BR + 3) / 4), 128, 0, s>>>(L, V, 0, V.BR);
    count_launch();
}

void launch_b4_update(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                      const UpdateParams& P, float* dxT, cudaStream_t s) {
    if (V.BR == 0 || B == 0) return;
    // 8 half-warps (block-rows) per 128-thread block; dx partials in shared
    // memory when 8 * 4 * B floats fit
    const size_t smem = (size_t)8 * 4 * B * sizeof(float);
    const int use_smem = smem <= 96 * 1024 ? 1 : 0;
    const unsigned grid = (unsigned)((V.BR + 7) / 8);
#define SILI_B4(R, ST)                                                                                       \
    do {                                                                                                     \
        if (use_smem && smem > 48 * 1024)                                                                    \
            cudaFuncSetAttribute(k_b4_update<R, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        k_b4_update<R, ST><<<grid, 128, use_smem ? smem : 0, s>>>(L, V, xT, dyT, B, P, dxT, use_smem);       \
    } while (0)
    switch (L.rank * 2 + (P.stochastic ? 1 : 0)) {
        case 2: SILI_B4(1, false); break;
        case 3: SILI_B4(1, true); break;
        case 4: SILI_B4(2, false); break;
        case 5: SILI_B4(2, true); break;
        case 6: SILI_B4(3, false); break;
        case 7: SILI_B4(3, true); break;
        case 8: SILI_B4(4, false); break;
        default: SILI_B4(4, true); break;
    }
#undef SILI_B4
    count_launch();
}

// ── sparse-input forward: sisldo_forward's block4 windows ─────────────────
// sisldo_ops.hpp:379-549.  For sample b, a block-row forms a window when any
// of its 4 input rows has an entry in the sparse input; each column of each
// tile of that block-row adds, over its live slots in li order,
// fma(os * vs, x * w, acc) -- the reference build's evaluation of
// acc += (w * vs * os) * x.  Windows are taken in ascending block-row.
__global__ void __launch_bounds__(128) k_b4_forward_sparse(LayerView L, B4View V, const float* __restrict__ xT,
                                                           const uint8_t* __restrict__ presT, int B,
                                                           float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bcol = (int64_t)blockIdx.x * 4 + warp;
    const int b = blockIdx.y * 32 + lane;
    if (bcol >= V.BC) return;
    const bool bok = b < B;
    float mo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int64_t col0 = bcol * 4;
    float osc[4];
#pragma unroll
    for (int lj = 0; lj < 4; ++lj) osc[lj] = col0 + lj < L.n_out ? L.os[(col0 + lj) * L.rank] : 0.0f;
    for (int t = V.cptr[bcol]; t < V.cptr[bcol + 1]; ++t) {
        const int64_t br = V.cbr[t];
        bool win = false;
        float x[4], vsr[4];
#pragma unroll
        for (int li = 0; li < 4; ++li) {
            const int64_t row = br * 4 + li;
            const bool ok = bok && row < L.n_in;
            win = win || (ok && presT[row * B + b] != 0);
            x[li] = ok ? xT[row * B + b] : 0.0f;
            vsr[li] = row < L.n_in ? L.vs[row * L.rank] : 0.0f;
        }
        if (!win) continue;
        const uint4 tw = V.tile[V.ctile[t]];
#pragma unroll
        for (int lj = 0; lj < 4; ++lj) {
            if (col0 + lj >= L.n_out) continue;
            float acc = 0.0f;
#pragma unroll
            for (int li = 0; li < 4; ++li) {
                if (br * 4 + li >= L.n_in) continue;
                const uint32_t byte = tile_byte(tw, lj * 4 + li);
                if (byte == 0) continue;
                acc = __fmaf_rn(__fmul_rn(osc[lj], vsr[li]), __fmul_rn(x[li], fp4_decode(byte & 0xFu)), acc);
            }
            mo[lj] = __fadd_rn(mo[lj], acc);
        }
    }
    if (!bok) return;
#pragma unroll
    for (int lj = 0; lj < 4; ++lj) {
        const int64_t col = col0 + lj;
        if (col < L.n_out) {
            float* o = y + (int64_t)b * L.n_out + col;
            *o = __fadd_rn(*o, mo[lj]);
        }
    }
}
void launch_b4_forward_sparse(const LayerView& L, const B4View& V, const float* xT, const uint8_t* presT, int B,
                              float* y, cudaStream_t s) {
    if (V.BC == 0 || B == 0) return;
    dim3 g((unsigned)((V.BC + 3) / 4), (unsigned)((B + 31) / 32));
    k_b4_forward_sparse<<<g, 128, 0, s>>>(L, V, xT, presT, B, y);
    count_launch();
}

// ── sparse-gradient backward: disldo_backward_sparse_grad's block4 part ────
// sisldo_ops.hpp:835-1104.  One half-warp per block-row, samples in order;
// lane s owns slot s (li = s & 3, lj = s >> 2) of the current tile.  A tile
// takes part for sample b when its 4-column window holds gradient entries;
// slots whose dy is non-zero add to dx (fused chains over the window's
// columns, li's chain carried by lane li) and, at lr != 0, get the plain
// RMSprop step with a stochastic requantize.  After each sample the row's
// workspace merge evicts down to its allocation; after all samples the
// rank-1 value_scale step (no finite checks, as the reference).
__global__ void __launch_bounds__(128) k_b4_backward_sparse(LayerView L, B4View V, const float* __restrict__ xT,
                                                            const float* __restrict__ dyT,
                                                            const uint8_t* __restrict__ presT, int B,
                                                            UpdateParams P, float* __restrict__ dxT) {
    const int lane = threadIdx.x & 31, s = lane & 15;
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4);
    const unsigned hmask = (lane >> 4) ? 0xFFFF0000u : 0x0000FFFFu;
    if (br >= V.BR) return;
    const int nt = V.nt[br];
    if (nt == 0) return;
    const int li = s & 3, lj = s >> 2;
    const int64_t row = br * 4 + li;
    const bool row_ok = row < L.n_in, leader = lj == 0;
    const int64_t base = V.es[br];
    const int64_t nnz_row = (int64_t)nt * 4;
    const bool training = P.lr != 0.0f;
    const float eff_lr = P.lr_per_row_nnz ? __fdiv_rn(P.lr, (float)nnz_row) : P.lr;
    const float onem = __fsub_rn(1.0f, P.beta2);
    const float vs = row_ok ? L.vs[row * L.rank] : 0.0f;
    const float isr = row_ok ? L.is[row] : 0.0f;
    double rgs = 0.0, rgc = 0.0;                  // row sums (leader lanes)
    double an = 0.0, ao = 0.0, sn = 0.0, so = 0.0;
    float mx = 0.0f;
    const int src0 = (lane & 16) | li;
    for (int b = 0; b < B; ++b) {
        const float in_val = row_ok ? xT[row * B + b] : 0.0f;
        float dxa = 0.0f;
        double rgl = 0.0, rglc = 0.0;              // this sample's row sums, added per sample
        for (int e = 0; e < nt; ++e) {
            const int64_t ti = base + e;
            const int64_t col = (int64_t)V.bc[ti] * 4 + lj;
            const bool col_ok = col < L.n_out;
            const bool pres = col_ok && presT[col * B + b] != 0;
            if (!__any_sync(hmask, pres)) continue;   // no gradient entry in the window
            const float dyv = pres ? dyT[col * B + b] : 0.0f;
            const bool act = row_ok && col_ok && dyv != 0.0f;
            uint4 tw = V.tile[ti];
            const uint32_t byte = tile_byte(tw, s);
            const float wd = fp4_decode(byte & 0xFu);
            const float osv = col_ok ? L.os[col * L.rank] : 0.0f;
            const float cs = __fmul_rn(vs, osv);
            const float w = __fmul_rn(wd, cs);
            // dx terms a*b, chained by the row's leader in column order
            const float ta = training ? w : __fmul_rn(osv, vs);
            const float tb = training ? dyv : __fmul_rn(dyv, wd);
            double qg = 0.0, qc = 0.0;
            uint32_t nb = byte;
            if (act && training) {
                const float cis = __fmul_rn(isr, L.ois[col]);
                const float imp_dec = fp4_decode(byte >> 4);
                const float grad = __fmul_rn(dyv, in_val);
                const float contrib = __fmul_rn(in_val, w);
                float imp = __fmul_rn(imp_dec, cis);
                imp = __fmaf_rn(P.beta2, imp, __fmul_rn(onem, __fmaf_rn(grad, grad, __fmul_rn(contrib, contrib))));
                const float ng = __fmul_rn(-eff_lr, grad);
                const float step = P.damp ? __fdiv_rn(ng, __fadd_rn(__fsqrt_rn(imp), P.eps)) : ng;
                const float new_w = __fadd_rn(w, step);
                const uint64_t el = (1ULL << 61) | (((uint64_t)b * (uint64_t)L.n_in + (uint64_t)row) * (uint64_t)L.n_out +
                                                    (uint64_t)col);
                const uint32_t wq = fp4_quantize_stochastic(__fdiv_rn(new_w, cs), rng_draw(P.call_key, el, 0));
                const uint32_t iq = fp4_quantize_stochastic(__fdiv_rn(imp, cis), rng_draw(P.call_key, el, 1));
                nb = (iq << 4) | wq;
                const float actual = __fmul_rn(fp4_decode(iq), cis), stored = __fmul_rn(imp_dec, cis);
                an += fabs((double)actual); ao += fabs((double)stored);
                sn += (double)actual * (double)actual; so += (double)stored * (double)stored;
                mx = fmaxf(mx, fabsf(actual));
                const double wo = __dmul_rn((double)wd, (double)osv);
                qg = __dmul_rn(wo, (double)__fmul_rn(dyv, in_val));
                qc = __dmul_rn(wo, (double)contrib);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int src = src0 + 4 * j;
                const float aj = __shfl_sync(hmask, ta, src);
                const float bj = __shfl_sync(hmask, tb, src);
                const int okj = __shfl_sync(hmask, (int)act, src);
                const double gj = __shfl_sync(hmask, qg, src);
                const double cj = __shfl_sync(hmask, qc, src);
                if (okj) {
                    dxa = __fmaf_rn(aj, bj, dxa);
                    if (training) { rgl = __dadd_rn(rgl, gj); rglc = __dadd_rn(rglc, cj); }
                }
            }
            if (training) {
                const bool dirty = __any_sync(hmask, act);
                set_tile_byte(tw, s, nb);
                uint32_t words[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t wv = 0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) wv |= __shfl_sync(hmask, nb, (lane & 16) | (q * 4 + k)) << (8 * k);
                    words[q] = wv;
                }
                if (dirty && s == 0) {
                    const uint4 nw = make_uint4(words[0], words[1], words[2], words[3]);
                    V.tile[ti] = nw;
                    V.sparse[ti] = (uint32_t)tile_live(nw) <= V.switch_point ? 1 : 0;
                }
                __syncwarp(hmask);
            }
        }
        if (training) b4_evict_row<16>(L, V, br, base, nt, s, hmask);
        if (leader && row_ok) {
            float* d = dxT + row * B + b;
            *d = __fadd_rn(*d, dxa);
            rgs = __dadd_rn(rgs, rgl);
            rgc = __dadd_rn(rgc, rglc);
        }
        __syncwarp(hmask);
    }
    if (!training) return;
    if (an != 0.0 || ao != 0.0 || sn != 0.0 || so != 0.0) {
        atomicAdd(P.stats + 0, an - ao);
        atomicAdd(P.stats + 1, sn - so);
    }
    atomicMax(reinterpret_cast<unsigned int*>(P.stat_max), __float_as_uint(mx));
    if (leader && row_ok && !(rgs == 0.0 && rgc == 0.0)) {
        // the rank-1 value_scale step of sisldo_ops.hpp:1080-1101
        const float se = __fdiv_rn(P.lr, (float)nnz_row);
        const float g = (float)rgs, c = (float)rgc;
        float* vsi = L.vsi + row * L.rank;
        const float nv = __fmaf_rn(P.beta2, *vsi, __fmul_rn(onem, __fmaf_rn(g, g, __fmul_rn(c, c))));
        uint32_t* st = L.vstep + row * L.rank;
        const uint32_t step = *st + 1u;
        *st = step;
        const float bc = __fsub_rn(1.0f, bias_pow(P, step));
        const float hat = bc > 0.0f ? __fdiv_rn(nv, bc) : nv;
        *vsi = nv;
        L.vs[row * L.rank] = __fsub_rn(L.vs[row * L.rank], __fdiv_rn(__fmul_rn(se, g), __fadd_rn(__fsqrt_rn(hat), P.eps)));
    }
}
void launch_b4_backward_sparse(const LayerView& L, const B4View& V, const float* xT, const float* dyT,
                               const uint8_t* presT, int B, const UpdateParams& P, float* dxT, cudaStream_t s) {
    if (V.BR == 0 || B == 0) return;
    k_b4_backward_sparse<<<(unsigned)((V.BR + 7) / 8), 128, 0, s>>>(L, V, xT, dyT, presT, B, P, dxT);
    count_launch();
}

// ── tile column index ───────────────────────────────────────────────────────
__global__ void k_b4_list(B4View V, const int* __restrict__ tile_off, int* __restrict__ keys,
                          int* __restrict__ slots, int* __restrict__ brs) {
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (br >= V.BR) return;
    for (int e = lane; e < V.nt[br]; e += 32) {
        const int o = tile_off[br] + e;
        const int64_t ti = V.es[br] + e;
        keys[o] = V.bc[ti];
        slots[o] = (int)ti;
        brs[o] = (int)br;
    }
}
void launch_b4_list(const B4View& V, const int* tile_off, int* keys, int* slots, int* brs, cudaStream_t s) {
    if (V.BR == 0) return;
    k_b4_list<<<(unsigned)((V.BR + 7) / 8), 256, 0, s>>>(V, tile_off, keys, slots, brs);
    count_launch();
}

// column pointers from the sorted keys (lower bound of each block-column) and
// the (slot, block-row) pairs gathered in sorted order
__global__ void k_b4_index(const int* __restrict__ sorted_keys, const int* __restrict__ perm, int n, int64_t BC,
                           const int* __restrict__ slots, const int* __restrict__ brs, int* __restrict__ cptr,
                           int* __restrict__ ctile, int* __restrict__ cbr) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { ctile[i] = slots[perm[i]]; cbr[i] = brs[perm[i]]; }
    if (i <= BC) {
        int lo = 0, hi = n;
        while (lo < hi) { const int mid = (lo + hi) >> 1; if (sorted_keys[mid] < (int)i) lo = mid + 1; else hi = mid; }
        cptr[i] = lo;
    }
}
void launch_b4_index(const int* sorted_keys, const int* perm, int n, int64_t BC, const int* slots, const int* brs,
                     int* cptr, int* ctile, int* cbr, cudaStream_t s) {
    const int64_t m = std::max<int64_t>(n, BC + 1);
    k_b4_index<<<(unsigned)((m + 255) / 256), 256, 0, s>>>(sorted_keys, perm, n, BC, slots, brs, cptr, ctile, cbr);
    count_launch();
}

}  // namespace sili
