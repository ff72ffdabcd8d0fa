// Construction-time CSR operations on the device -- what the reference's
// conversion path (sili/conversion, FoldedLayer.from_descriptor) does in
// torch / numpy on the host, with the same results:
//   csr_union             cpu_backend.cpp:3200-3238 over csr.hpp:505-580
//   prune_to_csr          sparse_prune.py:466-482 (to_sparse_csr: keep |w| >= min_abs)
//   csr_transpose         the csr.t().to_sparse_csr() of sparse_rnn.py:1002
//   stack_csr_vertical    rnn_fold.py:259-320
//   fit_rank1_envelope    sparse_rnn.py:854-882 (fit_rank1_scale_envelope)
//   fp4_row_rescale       sparse_rnn.py:1021-1037 (per-row max-abs / 6 scales)
// csr_union: each output row is the two-pointer merge of the two input rows'
// column lists, exactly as the reference walks them (so unsorted input gives
// the reference's result too): a thread per row counts, a scan places the
// rows, a thread per row writes.
#include <cuda_runtime.h>
#include <cub/cub.cuh>

#include <string>
#include <vector>

#include "kernels.cuh"
#include "sili_b200.h"

namespace sili {
int set_error(int code, const std::string& msg);
}

namespace {

#define CKU(x)                                                                                          \
    do {                                                                                                \
        cudaError_t e_ = (x);                                                                           \
        if (e_ != cudaSuccess) return sili::set_error(SILI_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

__global__ void k_union_count(const int* __restrict__ pa, const int* __restrict__ ia, const int* __restrict__ pb,
                              const int* __restrict__ ib, int n_rows, int* __restrict__ len) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    int a = pa[r], ae = pa[r + 1], b = pb[r], be = pb[r + 1], n = 0;
    while (a < ae && b < be) {
        const int ca = ia[a], cb = ib[b];
        if (ca < cb) ++a;
        else if (cb < ca) ++b;
        else { ++a; ++b; }
        ++n;
    }
    len[r] = n + (ae - a) + (be - b);
}

__global__ void k_union_fill(const int* __restrict__ pa, const int* __restrict__ ia, const float* __restrict__ va,
                             const int* __restrict__ pb, const int* __restrict__ ib, const float* __restrict__ vb,
                             int n_rows, int prefer, const int* __restrict__ op, int* __restrict__ oi,
                             float* __restrict__ ov) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    int a = pa[r], ae = pa[r + 1], b = pb[r], be = pb[r + 1], w = op[r];
    while (a < ae && b < be) {
        const int ca = ia[a], cb = ib[b];
        if (ca < cb) { oi[w] = ca; ov[w] = va[a]; ++a; }
        else if (cb < ca) { oi[w] = cb; ov[w] = vb[b]; ++b; }
        else {
            oi[w] = ca;
            ov[w] = prefer == 0 ? va[a] : prefer == 1 ? vb[b] : __fadd_rn(va[a], vb[b]);
            ++a; ++b;
        }
        ++w;
    }
    for (; a < ae; ++a, ++w) { oi[w] = ia[a]; ov[w] = va[a]; }
    for (; b < be; ++b, ++w) { oi[w] = ib[b]; ov[w] = vb[b]; }
}

// A device copy of a host-or-device array (cudaMemcpyDefault tells them apart).
template <typename T>
struct Staged {
    T* p = nullptr;
    ~Staged() { if (p) cudaFree(p); }
    int load(const T* src, size_t n, cudaStream_t s) {
        CKU(cudaMalloc((void**)&p, (n + 1) * sizeof(T)));
        if (n) CKU(cudaMemcpyAsync(p, src, n * sizeof(T), cudaMemcpyDefault, s));
        return SILI_OK;
    }
};

int check_ptrs(const std::vector<int>& p, const char* which) {
    if (p[0] < 0) return sili::set_error(SILI_EINVAL, std::string("csr_union: ") + which + " ptrs[0] < 0");
    for (size_t r = 1; r < p.size(); ++r)
        if (p[r] < p[r - 1]) return sili::set_error(SILI_EINVAL, std::string("csr_union: ") + which + " ptrs decrease");
    return SILI_OK;
}

// ── prune_to_csr: |w| >= min_abs and w != 0 (to_sparse drops zeros), a warp
// per row, columns ascending (ballot compaction in column order)
__global__ void k_prune_count(const float* __restrict__ w, int64_t rows, int64_t cols, float min_abs,
                              int* __restrict__ cnt) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    int n = 0;
    for (int64_t c = lane; c < cols; c += 32) {
        const float v = w[r * cols + c];
        n += (fabsf(v) >= min_abs && v != 0.0f) ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xFFFFFFFFu, n, o);
    if (lane == 0) cnt[r] = n;
}
__global__ void k_prune_fill(const float* __restrict__ w, int64_t rows, int64_t cols, float min_abs,
                             const int* __restrict__ ptrs, int* __restrict__ idx, float* __restrict__ vals) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    int o = ptrs[r];
    for (int64_t c0 = 0; c0 < cols; c0 += 32) {
        const int64_t c = c0 + lane;
        const float v = c < cols ? w[r * cols + c] : 0.0f;
        const bool keep = c < cols && fabsf(v) >= min_abs && v != 0.0f;
        const unsigned b = __ballot_sync(0xFFFFFFFFu, keep);
        if (keep) {
            const int at = o + __popc(b & ((1u << lane) - 1u));
            idx[at] = (int)c;
            vals[at] = v;
        }
        o += __popc(b);
    }
}

// ── transpose: entries keyed by column, stably sorted (rows stay ascending
// within each new row), gathered
__global__ void k_rows_of(const int* __restrict__ ptrs, int n_rows, int* __restrict__ row_of) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    for (int f = ptrs[r]; f < ptrs[r + 1]; ++f) row_of[f] = r;
}
__global__ void k_iota_int(int* __restrict__ a, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = i;
}
__global__ void k_count_cols(const int* __restrict__ idx, int nnz, int* __restrict__ cnt) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nnz) atomicAdd(&cnt[idx[i]], 1);
}
__global__ void k_gather_t(const int* __restrict__ perm, const int* __restrict__ row_of, const float* __restrict__ vals,
                           int nnz, int* __restrict__ oidx, float* __restrict__ ovals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nnz) return;
    const int f = perm[i];
    oidx[i] = row_of[f];
    ovals[i] = vals[f];
}

// ── stack_csr_vertical: part p's row pointers shifted by the nonzeros before it
__global__ void k_shift_ptrs(const int* __restrict__ src, int n, int add, int* __restrict__ dst) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[i] + add;
}

// ── fit_rank1_scale_envelope: alternating max-fits.  The values are >= 0
// (|M| over a positive scale), so their float bit patterns order like the
// values and an integer atomicMax is the float max, order-independent.
__global__ void k_fill_f(float* __restrict__ a, int64_t n, float v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = v;
}
__global__ void k_env_rows(const int* __restrict__ ptrs, const int* __restrict__ idx, const float* __restrict__ vals,
                           int n_rows, const float* __restrict__ col_scale, float* __restrict__ row_scale) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    float m = row_scale[r];
    for (int f = ptrs[r]; f < ptrs[r + 1]; ++f) m = fmaxf(m, __fdiv_rn(fabsf(vals[f]), col_scale[idx[f]]));
    row_scale[r] = m;
}
__global__ void k_env_cols(const int* __restrict__ ptrs, const int* __restrict__ idx, const float* __restrict__ vals,
                           int n_rows, const float* __restrict__ row_scale, float* __restrict__ col_scale) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    const float rs = row_scale[r];
    for (int f = ptrs[r]; f < ptrs[r + 1]; ++f)
        atomicMax((int*)&col_scale[idx[f]], __float_as_int(__fdiv_rn(fabsf(vals[f]), rs)));
}

// ── FoldedLayer.from_descriptor's FP4 preparation: mode 0 (per_row) -- each
// row's scale = (float)(max|w| / 6.0 in double) when that max is > 0 (else
// 1), values divided by it; mode 1 (rank1) -- row_scale = row_env / 6 in
// float, combined = row_scale * col_scale, values divided where combined > 0
__global__ void k_fp4_rescale(const int* __restrict__ ptrs, const int* __restrict__ idx, float* __restrict__ vals,
                              int n_rows, int mode, const float* __restrict__ col_scale,
                              float* __restrict__ row_scale) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    if (mode == 0) {
        float m = 0.0f;
        for (int f = ptrs[r]; f < ptrs[r + 1]; ++f) m = fmaxf(m, fabsf(vals[f]));
        float s = 1.0f;
        if (ptrs[r + 1] > ptrs[r] && m > 0.0f) {
            s = __double2float_rn(__ddiv_rn((double)m, 6.0));
            for (int f = ptrs[r]; f < ptrs[r + 1]; ++f) vals[f] = __fdiv_rn(vals[f], s);
        }
        row_scale[r] = s;
    } else {
        const float rs = __fdiv_rn(row_scale[r], 6.0f);
        for (int f = ptrs[r]; f < ptrs[r + 1]; ++f) {
            const float comb = __fmul_rn(rs, col_scale[idx[f]]);
            if (comb > 0.0f) vals[f] = __fdiv_rn(vals[f], comb);
        }
        row_scale[r] = rs;
    }
}

bool is_dev_ptr(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

namespace {
int need_dev(const void* p, const char* who) {
    if (p && !is_dev_ptr(p)) return sili::set_error(SILI_EINVAL, std::string(who) + ": arrays must be device memory");
    return SILI_OK;
}
}  // namespace

extern "C" int sili_prune_to_csr(const float* w, int64_t rows, int64_t cols, float min_abs, int* ptrs, int* idx,
                                 float* vals, int64_t* nnz_out, void* stream) {
    if (rows < 0 || cols < 0 || !w || !ptrs) return sili::set_error(SILI_EINVAL, "prune_to_csr: bad arguments");
    int rc;
    if ((rc = need_dev(w, "prune_to_csr")) || (rc = need_dev(ptrs, "prune_to_csr")) ||
        (rc = need_dev(idx, "prune_to_csr")) || (rc = need_dev(vals, "prune_to_csr")))
        return rc;
    cudaStream_t s = (cudaStream_t)stream;
    Staged<int> cnt;
    Staged<unsigned char> tmp;
    CKU(cudaMalloc((void**)&cnt.p, (size_t)(rows + 1) * 4));
    CKU(cudaMemsetAsync(cnt.p, 0, (size_t)(rows + 1) * 4, s));
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (rows > 0) {
        k_prune_count<<<grid, 256, 0, s>>>(w, rows, cols, min_abs, cnt.p);
        sili::count_launch();
    }
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, cnt.p, ptrs, (int)(rows + 1), s);
    CKU(cudaMalloc((void**)&tmp.p, bytes + 1));
    CKU(cub::DeviceScan::ExclusiveSum(tmp.p, bytes, cnt.p, ptrs, (int)(rows + 1), s));
    int total = 0;
    CKU(cudaMemcpyAsync(&total, ptrs + rows, 4, cudaMemcpyDeviceToHost, s));
    CKU(cudaStreamSynchronize(s));
    if (nnz_out) *nnz_out = total;
    if (idx && vals && rows > 0) {
        k_prune_fill<<<grid, 256, 0, s>>>(w, rows, cols, min_abs, ptrs, idx, vals);
        sili::count_launch();
    }
    CKU(cudaGetLastError());
    return SILI_OK;
}

extern "C" int sili_csr_transpose(const int* ptrs, const int* idx, const float* vals, int n_rows, int n_cols,
                                  int* out_ptrs, int* out_idx, float* out_vals, void* stream) {
    if (n_rows < 0 || n_cols < 0 || !ptrs || !out_ptrs) return sili::set_error(SILI_EINVAL, "csr_transpose: bad arguments");
    int rc;
    for (const void* p : {(const void*)ptrs, (const void*)idx, (const void*)vals, (const void*)out_ptrs,
                          (const void*)out_idx, (const void*)out_vals})
        if ((rc = need_dev(p, "csr_transpose"))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    int nnz = 0;
    CKU(cudaMemcpyAsync(&nnz, ptrs + n_rows, 4, cudaMemcpyDeviceToHost, s));
    CKU(cudaStreamSynchronize(s));
    Staged<int> row_of, perm, perm_o, keys_o, cnt;
    Staged<unsigned char> tmp;
    CKU(cudaMalloc((void**)&cnt.p, (size_t)(n_cols + 1) * 4));
    CKU(cudaMemsetAsync(cnt.p, 0, (size_t)(n_cols + 1) * 4, s));
    if (nnz > 0) {
        CKU(cudaMalloc((void**)&row_of.p, (size_t)nnz * 4));
        CKU(cudaMalloc((void**)&perm.p, (size_t)nnz * 4));
        CKU(cudaMalloc((void**)&perm_o.p, (size_t)nnz * 4));
        CKU(cudaMalloc((void**)&keys_o.p, (size_t)nnz * 4));
        k_rows_of<<<(unsigned)((n_rows + 255) / 256), 256, 0, s>>>(ptrs, n_rows, row_of.p);
        k_iota_int<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(perm.p, nnz);
        k_count_cols<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(idx, nnz, cnt.p);
        sili::count_launch(3);
        int bits = 1;
        while ((int64_t(1) << bits) < n_cols) ++bits;
        size_t bytes = 0;
        cub::DeviceRadixSort::SortPairs(nullptr, bytes, idx, keys_o.p, perm.p, perm_o.p, nnz, 0, bits, s);
        CKU(cudaMalloc((void**)&tmp.p, bytes + 1));
        CKU(cub::DeviceRadixSort::SortPairs(tmp.p, bytes, idx, keys_o.p, perm.p, perm_o.p, nnz, 0, bits, s));
        k_gather_t<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(perm_o.p, row_of.p, vals, nnz, out_idx, out_vals);
        sili::count_launch();
    }
    Staged<unsigned char> tmp2;
    size_t b2 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, b2, cnt.p, out_ptrs, n_cols + 1, s);
    CKU(cudaMalloc((void**)&tmp2.p, b2 + 1));
    CKU(cub::DeviceScan::ExclusiveSum(tmp2.p, b2, cnt.p, out_ptrs, n_cols + 1, s));
    CKU(cudaGetLastError());
    CKU(cudaStreamSynchronize(s));
    return SILI_OK;
}

extern "C" int sili_csr_stack_vertical(int n_parts, const int* const* ptrs, const int* const* idx,
                                       const float* const* vals, const int* rows, int* out_ptrs, int* out_idx,
                                       float* out_vals, void* stream) {
    if (n_parts < 1 || !ptrs || !idx || !vals || !rows) return sili::set_error(SILI_EINVAL, "stack_csr_vertical: bad arguments");
    cudaStream_t s = (cudaStream_t)stream;
    int rc;
    int64_t row0 = 0, nnz0 = 0;
    CKU(cudaMemsetAsync(out_ptrs, 0, 4, s));
    for (int p = 0; p < n_parts; ++p) {
        if ((rc = need_dev(ptrs[p], "stack_csr_vertical")) || (rc = need_dev(out_ptrs, "stack_csr_vertical"))) return rc;
        int n = 0;
        CKU(cudaMemcpyAsync(&n, ptrs[p] + rows[p], 4, cudaMemcpyDeviceToHost, s));
        CKU(cudaStreamSynchronize(s));
        if (rows[p] > 0) {
            k_shift_ptrs<<<(unsigned)((rows[p] + 255) / 256), 256, 0, s>>>(ptrs[p] + 1, rows[p], (int)nnz0,
                                                                          out_ptrs + row0 + 1);
            sili::count_launch();
        }
        if (n > 0) {
            CKU(cudaMemcpyAsync(out_idx + nnz0, idx[p], (size_t)n * 4, cudaMemcpyDeviceToDevice, s));
            CKU(cudaMemcpyAsync(out_vals + nnz0, vals[p], (size_t)n * 4, cudaMemcpyDeviceToDevice, s));
        }
        row0 += rows[p];
        nnz0 += n;
    }
    CKU(cudaGetLastError());
    CKU(cudaStreamSynchronize(s));
    return SILI_OK;
}

extern "C" int sili_fit_rank1_envelope(const int* ptrs, const int* idx, const float* vals, int n_rows, int n_cols,
                                       int n_iters, float* row_scale, float* col_scale, void* stream) {
    if (n_rows < 0 || n_cols < 0 || n_iters < 0) return sili::set_error(SILI_EINVAL, "fit_rank1_envelope: bad arguments");
    int rc;
    for (const void* p : {(const void*)ptrs, (const void*)idx, (const void*)vals, (const void*)row_scale,
                          (const void*)col_scale})
        if ((rc = need_dev(p, "fit_rank1_envelope"))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned gr = (unsigned)((n_rows + 255) / 256), gc = (unsigned)((n_cols + 255) / 256);
    if (n_cols) k_fill_f<<<gc, 256, 0, s>>>(col_scale, n_cols, 1.0f);
    if (n_rows) k_fill_f<<<gr, 256, 0, s>>>(row_scale, n_rows, 1.0f);
    sili::count_launch(2);
    for (int it = 0; it < n_iters; ++it) {
        if (n_rows) {
            k_fill_f<<<gr, 256, 0, s>>>(row_scale, n_rows, 1e-12f);
            k_env_rows<<<gr, 256, 0, s>>>(ptrs, idx, vals, n_rows, col_scale, row_scale);
        }
        if (n_cols) k_fill_f<<<gc, 256, 0, s>>>(col_scale, n_cols, 1e-12f);
        if (n_rows) k_env_cols<<<gr, 256, 0, s>>>(ptrs, idx, vals, n_rows, row_scale, col_scale);
        sili::count_launch(4);
    }
    CKU(cudaGetLastError());
    return SILI_OK;
}

extern "C" int sili_fp4_row_rescale(const int* ptrs, const int* idx, float* vals, int n_rows, int mode,
                                    const float* col_scale, float* row_scale, void* stream) {
    if (n_rows < 0 || (mode != 0 && mode != 1)) return sili::set_error(SILI_EINVAL, "fp4_row_rescale: bad arguments");
    int rc;
    for (const void* p : {(const void*)ptrs, (const void*)idx, (const void*)vals, (const void*)row_scale})
        if ((rc = need_dev(p, "fp4_row_rescale"))) return rc;
    if (mode == 1 && (rc = need_dev(col_scale, "fp4_row_rescale"))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    if (n_rows) {
        k_fp4_rescale<<<(unsigned)((n_rows + 255) / 256), 256, 0, s>>>(ptrs, idx, vals, n_rows, mode, col_scale,
                                                                       row_scale);
        sili::count_launch();
    }
    CKU(cudaGetLastError());
    return SILI_OK;
}

extern "C" int sili_csr_union(const int* pa, const int* ia, const float* va, const int* pb, const int* ib,
                              const float* vb, int n_rows, int prefer, int* out_ptrs, int* out_idx, float* out_vals,
                              int64_t* nnz_out, void* stream) {
    if (n_rows < 0 || !pa || !pb || !out_ptrs) return sili::set_error(SILI_EINVAL, "csr_union: bad arguments");
    if (prefer < 0 || prefer > 2) return sili::set_error(SILI_EINVAL, "prefer must be 'a', 'b', or 'sum'");
    cudaStream_t s = (cudaStream_t)stream;
    std::vector<int> hpa((size_t)n_rows + 1), hpb((size_t)n_rows + 1);
    CKU(cudaMemcpyAsync(hpa.data(), pa, hpa.size() * 4, cudaMemcpyDefault, s));
    CKU(cudaMemcpyAsync(hpb.data(), pb, hpb.size() * 4, cudaMemcpyDefault, s));
    CKU(cudaStreamSynchronize(s));
    int rc = check_ptrs(hpa, "A");
    if (!rc) rc = check_ptrs(hpb, "B");
    if (rc) return rc;
    const size_t na = (size_t)hpa[n_rows], nb = (size_t)hpb[n_rows];
    Staged<int> dpa, dpb, dia, dib, dlen, dop, doi;
    Staged<float> dva, dvb, dov;
    Staged<unsigned char> tmp;
    if ((rc = dpa.load(pa, hpa.size(), s)) || (rc = dpb.load(pb, hpb.size(), s)) || (rc = dia.load(ia, na, s)) ||
        (rc = dib.load(ib, nb, s)))
        return rc;
    CKU(cudaMalloc((void**)&dlen.p, ((size_t)n_rows + 1) * 4));
    CKU(cudaMalloc((void**)&dop.p, ((size_t)n_rows + 1) * 4));
    CKU(cudaMemsetAsync(dlen.p, 0, ((size_t)n_rows + 1) * 4, s));
    const unsigned grid = (unsigned)((n_rows + 255) / 256);
    if (n_rows > 0) {
        k_union_count<<<grid, 256, 0, s>>>(dpa.p, dia.p, dpb.p, dib.p, n_rows, dlen.p);
        sili::count_launch();
    }
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, dlen.p, dop.p, n_rows + 1, s);
    CKU(cudaMalloc((void**)&tmp.p, bytes + 1));
    CKU(cub::DeviceScan::ExclusiveSum(tmp.p, bytes, dlen.p, dop.p, n_rows + 1, s));
    int total = 0;
    CKU(cudaMemcpyAsync(&total, dop.p + n_rows, 4, cudaMemcpyDeviceToHost, s));
    CKU(cudaMemcpyAsync(out_ptrs, dop.p, ((size_t)n_rows + 1) * 4, cudaMemcpyDefault, s));
    CKU(cudaStreamSynchronize(s));
    if (nnz_out) *nnz_out = total;
    if (out_idx && out_vals) {
        if ((rc = dva.load(va, na, s)) || (rc = dvb.load(vb, nb, s))) return rc;
        CKU(cudaMalloc((void**)&doi.p, (size_t)total * 4 + 4));
        CKU(cudaMalloc((void**)&dov.p, (size_t)total * 4 + 4));
        if (n_rows > 0) {
            k_union_fill<<<grid, 256, 0, s>>>(dpa.p, dia.p, dva.p, dpb.p, dib.p, dvb.p, n_rows, prefer, dop.p, doi.p,
                                              dov.p);
            sili::count_launch();
        }
        CKU(cudaGetLastError());
        if (total) {
            CKU(cudaMemcpyAsync(out_idx, doi.p, (size_t)total * 4, cudaMemcpyDefault, s));
            CKU(cudaMemcpyAsync(out_vals, dov.p, (size_t)total * 4, cudaMemcpyDefault, s));
        }
    }
    CKU(cudaStreamSynchronize(s));
    return SILI_OK;
}
