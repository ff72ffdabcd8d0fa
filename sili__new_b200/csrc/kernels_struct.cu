// Structural kernels: warp-parallel ULEB128 row decoding into the derived
// row/column index, state export, headroom re-layout, activation
// sparsifiers and synaptogenesis probe generation.
#include "common.cuh"
#include "kernels.cuh"

namespace sili {

__global__ void k_row_nnz(const int64_t* __restrict__ es, const int64_t* __restrict__ ee, int64_t n_in,
                          int* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n_in) out[r] = (int)(ee[r] - es[r]);
}
void launch_row_nnz(const int64_t* es, const int64_t* ee, int64_t n_in, int* out, cudaStream_t s) {
    if (n_in == 0) return;
    k_row_nnz<<<(unsigned)((n_in + 255) / 256), 256, 0, s>>>(es, ee, n_in, out); count_launch();
}

// One warp per row: decodes the row's ULEB128 deltas (delta_csr_types.hpp:
// 229-241, DeltaCSRRowCursor :801-832) 32 bytes at a time with a ballot over
// terminator bytes and a warp prefix sum over the deltas, and writes every
// synapse's absolute column, row and value position.
__global__ void __launch_bounds__(256) k_decode_rows(LayerView L, int* __restrict__ abs_cols, int* __restrict__ frow,
                                                     int* __restrict__ fvpos, int* __restrict__ colcount) {
    __shared__ uint32_t stage[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + warp;
    if (r >= L.n_in) return;
    RowDecoder d{L.bs[r], L.be[r], 0u};
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    int f = L.rowptr[r];
    int e = 0;
    while (e < nnz && d.pos < d.end) {
        uint32_t col;
        const int cnt = warp_decode_window(L.idx, d, stage[warp], col);
        if (cnt == 0) break;
        if (lane < cnt && e + lane < nnz) {
            abs_cols[f + lane] = (int)col;
            if (frow) frow[f + lane] = (int)r;
            if (fvpos) fvpos[f + lane] = (int)(es + e + lane);
            if (colcount) atomicAdd(colcount + col, 1);
        }
        f += cnt;
        e += cnt;
    }
}
void launch_decode_rows(const LayerView& L, int* abs_cols, int* frow, int* fvpos, int* colcount, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_decode_rows<<<(unsigned)((L.n_in + 7) / 8), 256, 0, s>>>(L, abs_cols, frow, fvpos, colcount); count_launch();
}

// CSC shadow with every column padded to a multiple of 8 entries: entry k of
// the column-sorted order goes to pcolptr[col] + (k - colptr[col]); the
// padding entries are (row n_in, value position -1), i.e. the zero input row
// with weight 0, so the forward kernels need no per-element bounds tests.
__global__ void k_gather_csc(const int* __restrict__ sorted_f, const int* __restrict__ sorted_col,
                             const int* __restrict__ frow, const int* __restrict__ fvpos,
                             const int* __restrict__ colptr, const int* __restrict__ pcolptr, int64_t nnz,
                             int* __restrict__ crow, int* __restrict__ cvpos, int* __restrict__ fcpos) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= nnz) return;
    const int f = sorted_f[k], c = sorted_col[k];
    const int64_t o = pcolptr[c] + (k - colptr[c]);
    crow[o] = frow[f];
    cvpos[o] = fvpos[f];
    fcpos[f] = (int)o;   // where synapse f (row-major order) sits in the padded CSC
}
__global__ void k_pad_csc(const int* __restrict__ colcount, const int* __restrict__ pcolptr, int64_t n_cols,
                          int n_in, int* __restrict__ crow, int* __restrict__ cvpos) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n_cols) return;
    for (int o = pcolptr[c] + colcount[c]; o < pcolptr[c + 1]; ++o) { crow[o] = n_in; cvpos[o] = -1; }
}
// padded column counts: (count + 7) & ~7
__global__ void k_pad_counts(const int* __restrict__ colcount, int64_t n, int* __restrict__ out) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n) out[c] = (colcount[c] + 7) & ~7;
}
void launch_gather_csc(const int* sorted_f, const int* sorted_col, const int* frow, const int* fvpos,
                       const int* colptr, const int* pcolptr, int64_t nnz, int* crow, int* cvpos, int* fcpos,
                       cudaStream_t s) {
    if (nnz == 0) return;
    k_gather_csc<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(sorted_f, sorted_col, frow, fvpos, colptr, pcolptr, nnz,
                                                               crow, cvpos, fcpos);
    count_launch();
}
void launch_pad_csc(const int* colcount, const int* pcolptr, int64_t n_cols, int n_in, int* crow, int* cvpos,
                    cudaStream_t s) {
    if (n_cols == 0) return;
    k_pad_csc<<<(unsigned)((n_cols + 255) / 256), 256, 0, s>>>(colcount, pcolptr, n_cols, n_in, crow, cvpos);
    count_launch();
}
void launch_pad_counts(const int* colcount, int64_t n, int* out, cudaStream_t s) {
    if (n == 0) return;
    k_pad_counts<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(colcount, n, out);
    count_launch();
}

__global__ void k_fill_f32(float* p, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}
void launch_fill_f32(float* p, int64_t n, float v, cudaStream_t s) {
    if (n <= 0) return;
    k_fill_f32<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p, n, v); count_launch();
}
// Default read value of an unset scale slot: component 0 reads 1, the others
// 0 (get_value_scale_k / get_output_scale_k, delta_csr_types.hpp:1100-1104).
__global__ void k_fill_scale_default(float* p, int64_t begin, int64_t end, int rank) {
    const int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < end) p[i] = (i % rank) == 0 ? 1.0f : 0.0f;
}
void launch_fill_scale_default(float* p, int64_t begin, int64_t end, int rank, cudaStream_t s) {
    if (end <= begin) return;
    k_fill_scale_default<<<(unsigned)((end - begin + 255) / 256), 256, 0, s>>>(p, begin, end, rank); count_launch();
}

// decode -> deterministic encode of both nibbles (ValueAccessor get/set round
// trip used by compact/expand, sisldo_ops.hpp:79-82): identity except NaN
// code 8, which re-encodes to 0.
__global__ void k_recode(uint8_t* v, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t b = v[i];
    v[i] = (uint8_t)((fp4_encode(fp4_decode(b >> 4)) << 4) | fp4_encode(fp4_decode(b & 15u)));
}
void launch_recode_values(uint8_t* v, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    k_recode<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(v, n); count_launch();
}

// recompute_stats (delta_csr_types.hpp:1350-1364): sums of |w|, w^2, |imp|, imp^2
// over live synapses (double, atomics -> order-free within double rounding) and maxima.
__global__ void k_stats(LayerView L, double* __restrict__ sums, float* __restrict__ maxes) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + warp;
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    float m0 = 0.f, m1 = 0.f;
    if (r < L.n_in) {
        for (int64_t vb = L.es[r] + lane; vb < L.ee[r]; vb += 32) {
            const uint8_t b = L.val[vb];
            const float w = fp4_decode(b >> 4), im = fp4_decode(b & 15u);
            s0 += fabs((double)w); s1 += (double)w * w; s2 += fabs((double)im); s3 += (double)im * im;
            m0 = fmaxf(m0, fabsf(w)); m1 = fmaxf(m1, fabsf(im));
        }
    }
    s0 = warp_sum(s0); s1 = warp_sum(s1); s2 = warp_sum(s2); s3 = warp_sum(s3);
    for (int o = 16; o > 0; o >>= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (lane == 0 && r < L.n_in) {
        atomicAdd(sums + 0, s0); atomicAdd(sums + 1, s1); atomicAdd(sums + 2, s2); atomicAdd(sums + 3, s3);
        atomicMax(reinterpret_cast<unsigned int*>(maxes + 0), __float_as_uint(m0));
        atomicMax(reinterpret_cast<unsigned int*>(maxes + 1), __float_as_uint(m1));
    }
}
void launch_stats(const LayerView& L, double* sums, float* maxes, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_stats<<<(unsigned)((L.n_in + 7) / 8), 256, 0, s>>>(L, sums, maxes); count_launch();
}

// delta_csr_to_absolute (delta_csr_memory.hpp:95-123): flat columns come from
// the decoded index; weights/importance are the decoded stored codes.
__global__ void k_export(LayerView L, int* __restrict__ idx, float* __restrict__ w, float* __restrict__ imp) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
    if (r >= L.n_in) return;
    const int64_t es = L.es[r];
    const int nnz = (int)(L.ee[r] - es);
    const int f0 = L.rowptr[r];
    for (int e = threadIdx.x; e < nnz; e += 32) {
        const uint8_t b = L.val[es + e];
        if (idx) idx[f0 + e] = L.abs_cols[f0 + e];
        if (w) w[f0 + e] = fp4_decode(b >> 4);
        if (imp) imp[f0 + e] = fp4_decode(b & 15u);
    }
}
void launch_export(const LayerView& L, int* idx, float* w, float* imp, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_export<<<(unsigned)((L.n_in + 7) / 8), dim3(32, 8), 0, s>>>(L, idx, w, imp); count_launch();
}

// Copies every row's allocation (live bytes and blank tail up to the
// smaller of the old and new allocation) to its new offsets; new buffers are
// zero-filled by the caller, so grown headroom reads as zeros.
__global__ void k_copy_rows(LayerView L, const int64_t* __restrict__ nbs, const int64_t* __restrict__ nes,
                            uint8_t* __restrict__ nidx, uint8_t* __restrict__ nval, bool recode) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
    if (r >= L.n_in) return;
    const int64_t blive = L.be[r] - L.bs[r];
    for (int64_t i = threadIdx.x; i < blive; i += 32) nidx[nbs[r] + i] = L.idx[L.bs[r] + i];
    const int64_t elive = L.ee[r] - L.es[r];
    for (int64_t i = threadIdx.x; i < elive; i += 32) {
        uint8_t b = L.val[L.es[r] + i];
        if (recode) b = (uint8_t)((fp4_encode(fp4_decode(b >> 4)) << 4) | fp4_encode(fp4_decode(b & 15u)));
        nval[nes[r] + i] = b;
    }
}
void launch_copy_rows(const LayerView& L, const int64_t* nbs, const int64_t* nes, uint8_t* nidx, uint8_t* nval,
                      bool recode, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_copy_rows<<<(unsigned)((L.n_in + 7) / 8), dim3(32, 8), 0, s>>>(L, nbs, nes, nidx, nval, recode); count_launch();
}

__global__ void k_add_offset(int64_t* p, int64_t begin, int64_t end, int64_t delta) {
    const int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < end) p[i] += delta;
}
void launch_add_offset(int64_t* p, int64_t begin, int64_t end, int64_t delta, cudaStream_t s) {
    if (end <= begin || delta == 0) return;
    k_add_offset<<<(unsigned)((end - begin + 255) / 256), 256, 0, s>>>(p, begin, end, delta); count_launch();
}

// rescale_value_row / rescale_importance_row (delta_csr_types.hpp:1389-1431):
// re-encode one nibble of every synapse of the row at a new scale.
__global__ void k_rescale_row(LayerView L, int row, float old_scale, float new_scale, bool weight) {
    const int64_t es = L.es[row], ee = L.ee[row];
    for (int64_t vb = es + threadIdx.x; vb < ee; vb += blockDim.x) {
        const uint8_t b = L.val[vb];
        float w = fp4_decode(b >> 4), im = fp4_decode(b & 15u);
        if (weight) w = __fdiv_rn(__fmul_rn(w, old_scale), new_scale);
        else im = __fdiv_rn(__fmul_rn(im, old_scale), new_scale);
        L.val[vb] = (uint8_t)((fp4_encode(w) << 4) | fp4_encode(im));
    }
}
void launch_rescale_row(const LayerView& L, int row, float old_scale, float new_scale, bool weight,
                        cudaStream_t s) {
    k_rescale_row<<<1, 256, 0, s>>>(L, row, old_scale, new_scale, weight); count_launch();
}

__global__ void k_set_bytes(uint8_t* d, const uint8_t* s, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) d[i] = s[i];
}
void launch_set_bytes(uint8_t* d, const uint8_t* src, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    k_set_bytes<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d, src, n); count_launch();
}

__global__ void k_fp4_quantize(const float* v, uint8_t* out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = (uint8_t)fp4_encode(v[i]);
}
void launch_fp4_quantize(const float* v, uint8_t* out, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    k_fp4_quantize<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(v, out, n); count_launch();
}

// dense_to_csr (cpu_backend.cpp:3075-3116): count then ordered fill, one warp per row.
__global__ void k_d2c_count(const float* __restrict__ x, int rows, int cols, float thr, int* __restrict__ counts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    if (b >= rows) return;
    int n = 0;
    for (int c = lane; c < cols; c += 32) {
        const float v = x[(int64_t)b * cols + c];
        n += (v > thr || v < -thr) ? 1 : 0;
    }
    n = warp_sum(n);
    if (lane == 0) counts[b] = n;
}
__global__ void k_d2c_fill(const float* __restrict__ x, int rows, int cols, float thr, const int* __restrict__ ptrs,
                           int* __restrict__ idx, float* __restrict__ vals) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + warp;
    if (b >= rows) return;
    int o = ptrs[b];
    for (int c0 = 0; c0 < cols; c0 += 32) {
        const int c = c0 + lane;
        const float v = c < cols ? x[(int64_t)b * cols + c] : 0.0f;
        const bool keep = c < cols && (v > thr || v < -thr);
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const int p = o + __popc(m & ((1u << lane) - 1u));
            idx[p] = c;
            vals[p] = v;
        }
        o += __popc(m);
    }
}
void launch_dense_to_csr_count(const float* x, int rows, int cols, float thr, int* counts, cudaStream_t s) {
    if (rows == 0) return;
    k_d2c_count<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(x, rows, cols, thr, counts); count_launch();
}
void launch_dense_to_csr_fill(const float* x, int rows, int cols, float thr, const int* ptrs, int* idx,
                              float* vals, cudaStream_t s) {
    if (rows == 0) return;
    k_d2c_fill<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(x, rows, cols, thr, ptrs, idx, vals); count_launch();
}

// Keys for a descending sort by |v|: |v| bits (NaN above inf, as a bit
// pattern); a stable radix sort keeps ties in ascending flat index.
__global__ void k_abs_keys(const float* __restrict__ x, int64_t n, uint32_t* __restrict__ keys,
                           int* __restrict__ ids) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    keys[i] = __float_as_uint(x[i]) & 0x7FFFFFFFu;
    ids[i] = (int)i;
}
void launch_abs_keys(const float* x, int64_t n, uint32_t* keys, int* ids, cudaStream_t s) {
    if (n <= 0) return;
    k_abs_keys<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, keys, ids); count_launch();
}
__global__ void k_topk_emit(const float* __restrict__ x, const int* __restrict__ flat, int64_t k, int cols,
                            int* __restrict__ rowcount, int* __restrict__ idx, float* __restrict__ vals) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= k) return;
    const int f = flat[i];
    idx[i] = f % cols;
    vals[i] = x[f];
    atomicAdd(rowcount + f / cols, 1);
}
void launch_topk_emit(const float* x, const int* flat_sorted, int64_t k, int cols, int* rowcount, int* idx,
                      float* vals, cudaStream_t s) {
    if (k <= 0) return;
    k_topk_emit<<<(unsigned)((k + 255) / 256), 256, 0, s>>>(x, flat_sorted, k, cols, rowcount, idx, vals); count_launch();
}

__global__ void k_iota(int* p, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = (int)i;
}
void launch_iota(int* p, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    k_iota<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p, n); count_launch();
}

// ── probes (delta_csr_build_probes, delta_csr_memory.hpp:1308-1427) ────────
__device__ __forceinline__ bool row_has_col(const LayerView& L, int64_t r, int c) {
    int lo = L.rowptr[r], hi = L.rowptr[r + 1];
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const int v = L.abs_cols[mid];
        if (v < c) lo = mid + 1;
        else hi = mid;
    }
    return lo < L.rowptr[r + 1] && L.abs_cols[lo] == c;
}
// global mode: flag (a, b) of the kin x kout outer product if column
// out_sorted[b] does not exist in row in_sorted[a]
__global__ void k_probe_flags(LayerView L, const int* __restrict__ in_sorted, int kin,
                              const int* __restrict__ out_sorted, int kout, int* __restrict__ flags) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)kin * kout) return;
    const int a = (int)(i / kout), b = (int)(i % kout);
    flags[i] = row_has_col(L, in_sorted[a], out_sorted[b]) ? 0 : 1;
}
void launch_probe_flags(const LayerView& L, const int* in_sorted, int kin, const int* out_sorted, int kout, int* flags,
                        cudaStream_t s) {
    const int64_t n = (int64_t)kin * kout;
    if (n <= 0) return;
    k_probe_flags<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(L, in_sorted, kin, out_sorted, kout, flags); count_launch();
}
__global__ void k_probe_emit(const int* __restrict__ in_sorted, int kin, const int* __restrict__ out_sorted, int kout,
                             const int* __restrict__ flags, const int* __restrict__ pos,
                             const float* __restrict__ in_acc, const float* __restrict__ grad_acc,
                             int* __restrict__ prow, int* __restrict__ pcol, float* __restrict__ pval) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)kin * kout || !flags[i]) return;
    const int r = in_sorted[i / kout], c = out_sorted[i % kout];
    const int p = pos[i];
    prow[p] = r;
    pcol[p] = c;
    pval[p] = __fmul_rn(in_acc[r], grad_acc[c]);
}
void launch_probe_emit(const int* in_sorted, int kin, const int* out_sorted, int kout, const int* flags, const int* pos,
                       const float* in_acc, const float* grad_acc, int* prow, int* pcol, float* pval, cudaStream_t s) {
    const int64_t n = (int64_t)kin * kout;
    if (n <= 0) return;
    k_probe_emit<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in_sorted, kin, out_sorted, kout, flags, pos, in_acc,
                                                               grad_acc, prow, pcol, pval); count_launch();
}
// per-row mode: for candidate row a, the first k columns of the global
// descending order that the row does not already hold; written to slots
// [a*k, a*k+count) (compacted by the host afterwards).
__global__ void k_probe_per_row(LayerView L, const int* __restrict__ in_sorted, int kin,
                                const int* __restrict__ out_sorted, int64_t n_out, int k,
                                const float* __restrict__ in_acc, const float* __restrict__ grad_acc,
                                int* __restrict__ prow, int* __restrict__ pcol, float* __restrict__ pval,
                                int* __restrict__ counts) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int a = blockIdx.x * 8 + warp;
    if (a >= kin) return;
    const int r = in_sorted[a];
    int got = 0;
    for (int64_t b0 = 0; b0 < n_out && got < k; b0 += 32) {
        const int64_t b = b0 + lane;
        const int c = b < n_out ? out_sorted[b] : -1;
        const bool ok = c >= 0 && !row_has_col(L, r, c);
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int p = got + __popc(m & ((1u << lane) - 1u));
            if (p < k) {
                const int64_t o = (int64_t)a * k + p;
                prow[o] = r;
                pcol[o] = c;
                pval[o] = __fmul_rn(in_acc[r], grad_acc[c]);
            }
        }
        got += __popc(m);
    }
    if (lane == 0) counts[a] = got < k ? got : k;
}
void launch_probe_per_row(const LayerView& L, const int* in_sorted, int kin, const int* out_sorted, int64_t n_out,
                          int k, const float* in_acc, const float* grad_acc, int* prow, int* pcol, float* pval,
                          int* counts, cudaStream_t s) {
    if (kin <= 0) return;
    k_probe_per_row<<<(unsigned)((kin + 7) / 8), 256, 0, s>>>(L, in_sorted, kin, out_sorted, n_out, k, in_acc,
                                                               grad_acc, prow, pcol, pval, counts); count_launch();
}

// ── load_weights import (delta_csr_from_absolute, delta_csr_memory.hpp:16-93) ──
__device__ __forceinline__ int uleb_len(uint32_t v) { int n = 1; while (v >>= 7) ++n; return n; }

__global__ void k_import_lengths(const int* __restrict__ ptrs, const int* __restrict__ idx, int n_in,
                                 int* __restrict__ len) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= n_in) return;
    for (int f = ptrs[r] + lane; f < ptrs[r + 1]; f += 32) {
        const uint32_t prev = f > ptrs[r] ? (uint32_t)idx[f - 1] : 0u;
        len[f] = uleb_len((uint32_t)idx[f] - prev);
    }
}
void launch_import_lengths(const int* ptrs, const int* idx, int n_in, int* len, cudaStream_t s) {
    if (n_in == 0) return;
    k_import_lengths<<<(unsigned)((n_in + 7) / 8), 256, 0, s>>>(ptrs, idx, n_in, len); count_launch();
}
__global__ void k_import_rows(const int* __restrict__ ptrs, const int* __restrict__ boff, int n_in,
                              int64_t* __restrict__ row_bytes, int64_t* __restrict__ row_n) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_in) return;
    row_bytes[r] = (int64_t)boff[ptrs[r + 1]] - boff[ptrs[r]];
    row_n[r] = ptrs[r + 1] - ptrs[r];
}
void launch_import_rows(const int* ptrs, const int* boff, int n_in, int64_t* row_bytes, int64_t* row_n,
                        cudaStream_t s) {
    if (n_in == 0) return;
    k_import_rows<<<(unsigned)((n_in + 255) / 256), 256, 0, s>>>(ptrs, boff, n_in, row_bytes, row_n); count_launch();
}
// Writes each synapse's ULEB128 delta at its row's byte offset and its value
// byte (deterministic FP4 of the weight, importance code 0) at its element slot.
__global__ void k_import_write(const int* __restrict__ ptrs, const int* __restrict__ idx,
                               const float* __restrict__ vals, const float* __restrict__ imps,
                               const int* __restrict__ boff, int n_in,
                               const int64_t* __restrict__ bs, const int64_t* __restrict__ es,
                               uint8_t* __restrict__ ibuf, uint8_t* __restrict__ vbuf) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= n_in) return;
    const int p0 = ptrs[r];
    for (int f = p0 + lane; f < ptrs[r + 1]; f += 32) {
        uint32_t v = (uint32_t)idx[f] - (f > p0 ? (uint32_t)idx[f - 1] : 0u);
        int64_t o = bs[r] + (boff[f] - boff[p0]);
        do {
            uint8_t b = (uint8_t)(v & 0x7Fu);
            v >>= 7;
            if (v) b |= 0x80u;
            ibuf[o++] = b;
        } while (v);
        vbuf[es[r] + (f - p0)] = (uint8_t)((fp4_encode(vals[f]) << 4) | (imps ? fp4_encode(imps[f]) : 0u));
    }
}
void launch_import_write(const int* ptrs, const int* idx, const float* vals, const float* imps, const int* boff,
                         int n_in, const int64_t* bs, const int64_t* es, uint8_t* ibuf, uint8_t* vbuf, cudaStream_t s) {
    if (n_in == 0) return;
    k_import_write<<<(unsigned)((n_in + 7) / 8), 256, 0, s>>>(ptrs, idx, vals, imps, boff, n_in, bs, es, ibuf, vbuf);
    count_launch();
}

}  // namespace sili

namespace sili {
// FoldedLayer's fold sum (sili/sparse_rnn.py:1120-1125): y[b, j] = sum over
// folds f (ascending) of raw[b, f * out_dim + j], raw of width n_folds * out_dim
__global__ void k_fold_sum(const float* __restrict__ raw, int B, int n_folds, int64_t out_dim, float* __restrict__ y) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)B * out_dim) return;
    const int64_t b = t / out_dim, j = t % out_dim;
    const float* r = raw + b * (int64_t)n_folds * out_dim + j;
    float acc = 0.0f;
    for (int f = 0; f < n_folds; ++f) acc = __fadd_rn(acc, r[(int64_t)f * out_dim]);
    y[t] = acc;
}
void launch_fold_sum(const float* raw, int B, int n_folds, int64_t out_dim, float* y, cudaStream_t s) {
    const int64_t n = (int64_t)B * out_dim;
    if (n == 0) return;
    k_fold_sum<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(raw, B, n_folds, out_dim, y);
    count_launch();
}
// FoldedLayer's suffix sum (Python's sum over the suffix outputs,
// sili/sparse_rnn.py:1120-1122): y = 0 + raw_0 + raw_1 + ..., elementwise
struct RawPtrs { const float* p[kFoldedMaxSuffixes]; };
__global__ void k_suffix_sum(RawPtrs R, int n, int64_t count, float* __restrict__ y) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float a = 0.0f;
    for (int k = 0; k < n; ++k) a = __fadd_rn(a, R.p[k][i]);
    y[i] = a;
}
void launch_suffix_sum(const float* const* raws, int n, int64_t count, float* y, cudaStream_t s) {
    if (count == 0 || n <= 0) return;
    RawPtrs R{};
    for (int k = 0; k < n && k < kFoldedMaxSuffixes; ++k) R.p[k] = raws[k];
    k_suffix_sum<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(R, n < kFoldedMaxSuffixes ? n : kFoldedMaxSuffixes,
                                                                 count, y);
    count_launch();
}
// its backward for one column slice: raw[b, f * w + j] = dy[b, j0 + j]
// (the np.tile of sili/sparse_rnn.py:1144-1148), one thread per output float
__global__ void k_fold_broadcast(const float* __restrict__ dy, int B, int64_t out_dim, int64_t j0, int64_t w,
                                 int n_folds, float* __restrict__ raw) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t row = (int64_t)n_folds * w;
    if (t >= (int64_t)B * row) return;
    const int64_t b = t / row, j = (t % row) % w;
    raw[t] = dy[b * out_dim + j0 + j];
}
void launch_fold_broadcast(const float* dy, int B, int64_t out_dim, int64_t j0, int64_t w, int n_folds, float* raw,
                           cudaStream_t s) {
    const int64_t n = (int64_t)B * n_folds * w;
    if (n == 0) return;
    k_fold_broadcast<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dy, B, out_dim, j0, w, n_folds, raw);
    count_launch();
}
}  // namespace sili
