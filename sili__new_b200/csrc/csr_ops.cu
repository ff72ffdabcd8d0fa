// Construction-time CSR operations on the device: csr_union (the module
// function of sili/cpu_backend.cpp:3200-3238 over csr.hpp:505-580).  Each
// output row is the two-pointer merge of the two input rows' column lists,
// exactly as the reference walks them (so unsorted input gives the
// reference's result too): a thread per row counts, a scan places the rows,
// a thread per row writes.
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

}  // namespace

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
