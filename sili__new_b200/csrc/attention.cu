// Banded and sparse attention on the device: the three attention kernels
// of the folded stack (sili/lib/headers/attention.hpp) --
//   banded_attention_forward        :39-96   dense within a geometric band
//   sparse_banded_attention_forward :121-197 top-k keys by L2 norm in the band
//   sparse_attention_forward        :228-333 global top-k queries and keys
//   banded_attention_backward       :354-442
// -- over groups (heads x sequences) of row-major [T, d] / [K, d] fp32
// matrices.  Query group g reads key/value group g / (G / Gk), so grouped-
// query attention (32 query heads over 8 KV heads) runs in one launch.
//
// One warp per query.  The warp walks its keys (the band, or its list of
// selected keys) 32 at a time: the K and V rows of a chunk are staged in the
// warp's shared-memory slice (K rows padded to d + 1 floats so the lane-per-
// key dot products never share a bank), lane j scores key j against the
// query held in shared memory, and the output (lanes over d) accumulates by
// the online-softmax recurrence (running max, rescaled sum), divided by the
// sum at the end.  The reference normalises after a full max pass instead;
// both are the same softmax, equal to fp32 rounding.
//
// The band of query t is centred on the geometric diagonal
// ck = (t (K-1) + (T-1)/2) / (T-1) (integer division), keys
// [max(ck - hbw, 0), min(ck + hbw, K - 1)], clamped to <= t when causal --
// the reference's index arithmetic, so every query sees the same keys.
#include <cuda_runtime.h>
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <string>

#include "kernels.cuh"
#include "sili_b200.h"

namespace sili {
int set_error(int code, const std::string& msg);
}

namespace {

#define CKA(x)                                                                                          \
    do {                                                                                                \
        cudaError_t e_ = (x);                                                                           \
        if (e_ != cudaSuccess) return sili::set_error(SILI_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

constexpr int kMaxD = 256;        // head dimension limit (8 values per lane)
constexpr int kWarpsFwd = 4;

struct AttnShape {
    int64_t G, Gk, T, K, d;
    int64_t hbw;
    int causal;
};

__device__ __forceinline__ void band_of(const AttnShape& S, int64_t t, int64_t& lo, int64_t& hi) {
    const int64_t ck = (S.T <= 1 || S.K <= 1) ? 0 : (t * (S.K - 1) + (S.T - 1) / 2) / (S.T - 1);
    lo = ck > S.hbw ? ck - S.hbw : 0;
    hi = ck + S.hbw < S.K - 1 ? ck + S.hbw : S.K - 1;
    if (S.causal && hi > t) hi = t;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Keys of one query: a contiguous band [lo, hi] (list == nullptr) or n keys
// from a list.  Returns the output row (already divided by the softmax sum)
// in acc[] (lane holds d-indices lane + 32 j).
template <int NJ>
__device__ void attend(const float* __restrict__ qrow, const float* __restrict__ Kg, const float* __restrict__ Vg,
                       int64_t d, float scale, int64_t lo, int64_t n, const int* __restrict__ list,
                       int64_t causal_t, float* sq, float* sk, float* sv, float acc[NJ]) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = lane; i < d; i += 32) sq[i] = qrow[i];
    float m = -INFINITY, l = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j] = 0.f;
    const int64_t dp = d + 1;
    for (int64_t c0 = 0; c0 < n; c0 += 32) {
        const int cnt = (int)(n - c0 < 32 ? n - c0 : 32);
        __syncwarp();
        // stage the chunk's K and V rows (row by row, lanes over d)
        for (int r = 0; r < cnt; ++r) {
            const int64_t key = list ? (int64_t)list[c0 + r] : lo + c0 + r;
            const float* kr = Kg + key * d;
            const float* vr = Vg + key * d;
            for (int64_t i = lane; i < d; i += 32) {
                sk[r * dp + i] = kr[i];
                sv[r * d + i] = vr[i];
            }
        }
        __syncwarp();
        float s = -INFINITY;
        if (lane < cnt) {
            const int64_t key = list ? (int64_t)list[c0 + lane] : lo + c0 + lane;
            if (causal_t < 0 || key <= causal_t) {
                float dot = 0.f;
                const float* kr = sk + lane * dp;
                for (int64_t i = 0; i < d; ++i) dot = fmaf(sq[i], kr[i], dot);
                s = dot * scale;
            }
        }
        const float cm = warp_max(s);
        if (cm == -INFINITY) continue;        // no valid key in this chunk
        const float mn = fmaxf(m, cm);
        const float corr = m == -INFINITY ? 0.f : expf(m - mn);
        const float p = s == -INFINITY ? 0.f : expf(s - mn);
        l = l * corr + warp_sum(p);
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[j] *= corr;
        for (int r = 0; r < cnt; ++r) {
            const float pr = __shfl_sync(0xFFFFFFFFu, p, r);
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int64_t i = lane + 32 * j;
                if (i < d) acc[j] = fmaf(pr, sv[r * d + i], acc[j]);
            }
        }
        m = mn;
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j] *= inv;
}

// banded (list == nullptr) / sparse-banded (per-query lists sel[g][t][0..cnt[g][t]))
template <int NJ>
__global__ void __launch_bounds__(kWarpsFwd * 32) k_attn_band(AttnShape S, const float* __restrict__ q,
                                                             const float* __restrict__ k, const float* __restrict__ v,
                                                             const int* __restrict__ sel, const int* __restrict__ selcnt,
                                                             int64_t sel_stride, float* __restrict__ out) {
    extern __shared__ float smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gq = (int64_t)blockIdx.x * kWarpsFwd + warp;   // flat (group, query)
    if (gq >= S.G * S.T) return;
    const int64_t g = gq / S.T, t = gq % S.T;
    const int64_t gk = g / (S.G / S.Gk);
    const int64_t d = S.d;
    float* sq = smem + (int64_t)warp * (d + 32 * (d + 1) + 32 * d);
    float* sk = sq + d;
    float* sv = sk + 32 * (d + 1);
    int64_t lo, hi;
    band_of(S, t, lo, hi);
    const float scale = 1.0f / sqrtf((float)d);
    float acc[NJ];
    const float* Kg = k + gk * S.K * d;
    const float* Vg = v + gk * S.K * d;
    if (sel) {
        attend<NJ>(q + gq * d, Kg, Vg, d, scale, 0, selcnt[gq], sel + gq * sel_stride, -1, sq, sk, sv, acc);
    } else {
        attend<NJ>(q + gq * d, Kg, Vg, d, scale, lo, hi - lo + 1, nullptr, -1, sq, sk, sv, acc);
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int64_t i = lane + 32 * j;
        if (i < d) out[gq * d + i] = acc[j];
    }
}

// Global top-k attention (one group): the kk selected queries (q_idx) each
// attend the kk selected keys (k_idx, in selection order); causal masks key
// positions after the query's.
template <int NJ>
__global__ void __launch_bounds__(kWarpsFwd * 32) k_attn_sparse(int64_t d, int64_t kk, int causal,
                                                               const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, const int* __restrict__ qidx,
                                                               const int* __restrict__ kidx, float* __restrict__ out) {
    extern __shared__ float smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t qi = (int64_t)blockIdx.x * kWarpsFwd + warp;
    if (qi >= kk) return;
    float* sq = smem + (int64_t)warp * (d + 32 * (d + 1) + 32 * d);
    float* sk = sq + d;
    float* sv = sk + 32 * (d + 1);
    const int64_t t = qidx[qi];
    float acc[NJ];
    attend<NJ>(q + t * d, k, v, d, 1.0f / sqrtf((float)d), 0, kk, kidx, causal ? t : -1, sq, sk, sv, acc);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int64_t i = lane + 32 * j;
        if (i < d) out[t * d + i] = acc[j];
    }
}

__global__ void k_iota_i32(int* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = (int)i;
}

// Squared L2 norm of every row (fixed ascending order per row).
__global__ void k_row_sqnorm(const float* __restrict__ x, int64_t rows, int64_t d, float* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float s = 0.f;
    for (int64_t i = 0; i < d; ++i) s = fmaf(x[r * d + i], x[r * d + i], s);
    out[r] = s;
}

// sparse_banded's selection: per (group, query), the kk keys of the band
// with the largest squared norms (ties toward the lower key), in ascending
// key order.  Key j is selected when fewer than kk band keys rank above it.
__global__ void __launch_bounds__(128) k_band_select(AttnShape S, int64_t inner_k, const float* __restrict__ knorm,
                                                     int* __restrict__ sel, int* __restrict__ cnt, int64_t stride) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gq = (int64_t)blockIdx.x * 4 + warp;
    if (gq >= S.G * S.T) return;
    const int64_t g = gq / S.T, t = gq % S.T;
    const float* nr = knorm + (g / (S.G / S.Gk)) * S.K;
    int64_t lo, hi;
    band_of(S, t, lo, hi);
    const int64_t w = hi - lo + 1;
    const int64_t kk = (inner_k == 0 || inner_k >= w) ? w : inner_k;
    int64_t out = 0;
    for (int64_t c0 = 0; c0 < w; c0 += 32) {
        const int64_t j = lo + c0 + lane;
        bool take = false;
        if (c0 + lane < w) {
            if (kk == w) {
                take = true;
            } else {
                const float nj = nr[j];
                int64_t rank = 0;
                for (int64_t m = lo; m <= hi && rank < kk; ++m) {
                    const float nm = nr[m];
                    rank += (nm > nj || (nm == nj && m < j)) ? 1 : 0;
                }
                take = rank < kk;
            }
        }
        const unsigned b = __ballot_sync(0xFFFFFFFFu, take);
        if (take) sel[gq * stride + out + __popc(b & ((1u << lane) - 1u))] = (int)j;
        out += __popc(b);
    }
    if (lane == 0) cnt[gq] = (int)out;
}

// banded_attention_backward, pass 1 (warp per query): the band's softmax
// weights recomputed as the forward (max pass, exp, normalise),
// g = sum attn (dO . V_k), ds = attn (dO . V_k - g) stored per band slot, and
// dQ[t] = sum ds * scale * K[k].
__global__ void __launch_bounds__(128) k_band_bwd_q(AttnShape S, const float* __restrict__ q,
                                                    const float* __restrict__ k, const float* __restrict__ v,
                                                    const float* __restrict__ dO, int64_t W, float* __restrict__ attn,
                                                    float* __restrict__ dsb, float* __restrict__ dQ) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gq = (int64_t)blockIdx.x * 4 + warp;
    if (gq >= S.G * S.T) return;
    const int64_t g = gq / S.T, t = gq % S.T, d = S.d;
    const int64_t gk = g / (S.G / S.Gk);
    const float* Kg = k + gk * S.K * d;
    const float* Vg = v + gk * S.K * d;
    const float* qr = q + gq * d;
    const float* dor = dO + gq * d;
    int64_t lo, hi;
    band_of(S, t, lo, hi);
    const int64_t w = hi - lo + 1;
    const float scale = 1.0f / sqrtf((float)d);
    float* a = attn + gq * W;
    float* ds = dsb + gq * W;
    // scores (lane per key), max
    float mx = -INFINITY;
    for (int64_t b0 = 0; b0 < w; b0 += 32) {
        const int64_t bi = b0 + lane;
        if (bi < w) {
            const float* kr = Kg + (lo + bi) * d;
            float dot = 0.f;
            for (int64_t i = 0; i < d; ++i) dot = fmaf(qr[i], kr[i], dot);
            a[bi] = dot * scale;
            mx = fmaxf(mx, a[bi]);
        }
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int64_t bi = lane; bi < w; bi += 32) {
        const float e = expf(a[bi] - mx);
        a[bi] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    const float inv = sum > 0.f ? 1.0f / sum : 0.f;
    float gsum = 0.f;
    for (int64_t bi = lane; bi < w; bi += 32) {
        a[bi] *= inv;
        const float* vr = Vg + (lo + bi) * d;
        float dot = 0.f;
        for (int64_t i = 0; i < d; ++i) dot = fmaf(dor[i], vr[i], dot);
        ds[bi] = dot;                 // dO . V_k for now
        gsum = fmaf(a[bi], dot, gsum);
    }
    gsum = warp_sum(gsum);
    for (int64_t bi = lane; bi < w; bi += 32) ds[bi] = a[bi] * (ds[bi] - gsum);
    __syncwarp();
    // dQ[t] (lanes over d), keys in band order
    for (int64_t i = lane; i < d; i += 32) {
        float acc = 0.f;
        for (int64_t bi = 0; bi < w; ++bi) acc = fmaf(ds[bi] * scale, Kg[(lo + bi) * d + i], acc);
        dQ[gq * d + i] = acc;
    }
}

// pass 2 (warp per key of a key group): the queries whose band holds key k
// form one contiguous range (band ends never decrease with t); over them,
// in ascending t and over every query group reading this key group,
// dV[k] = sum attn dO and dK[k] = sum ds * scale * Q.
__global__ void __launch_bounds__(128) k_band_bwd_kv(AttnShape S, const float* __restrict__ q,
                                                     const float* __restrict__ dO, int64_t W,
                                                     const float* __restrict__ attn, const float* __restrict__ dsb,
                                                     float* __restrict__ dK, float* __restrict__ dV) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t gkk = (int64_t)blockIdx.x * 4 + warp;
    if (gkk >= S.Gk * S.K) return;
    const int64_t gk = gkk / S.K, key = gkk % S.K, d = S.d;
    const int64_t ratio = S.G / S.Gk;
    const float scale = 1.0f / sqrtf((float)d);
    // first query whose band reaches key (hi(t) >= key), last with lo(t) <= key
    int64_t a0 = 0, a1 = S.T;
    while (a0 < a1) {
        const int64_t mid = (a0 + a1) / 2;
        int64_t lo, hi;
        band_of(S, mid, lo, hi);
        if (hi >= key) a1 = mid; else a0 = mid + 1;
    }
    int64_t b0 = a0, b1 = S.T;
    while (b0 < b1) {
        const int64_t mid = (b0 + b1) / 2;
        int64_t lo, hi;
        band_of(S, mid, lo, hi);
        if (lo <= key) b0 = mid + 1; else b1 = mid;
    }
    for (int64_t i = lane; i < d; i += 32) {
        float av = 0.f, ak = 0.f;
        for (int64_t r = 0; r < ratio; ++r) {
            const int64_t g = gk * ratio + r;
            for (int64_t t = a0; t < b0; ++t) {
                int64_t lo, hi;
                band_of(S, t, lo, hi);
                if (key < lo || key > hi) continue;
                const int64_t gq = g * S.T + t;
                const float at = attn[gq * W + (key - lo)];
                const float ds = dsb[gq * W + (key - lo)];
                av = fmaf(at, dO[gq * d + i], av);
                ak = fmaf(ds * scale, q[gq * d + i], ak);
            }
        }
        dV[gkk * d + i] = av;
        dK[gkk * d + i] = ak;
    }
}

template <typename T>
struct DevArr {
    T* p = nullptr;
    bool owned = false;
    ~DevArr() { if (owned && p) cudaFree(p); }
};

bool is_dev(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// a device view of a host-or-device input array of n floats
int stage_in(const float* src, int64_t n, DevArr<float>& out, cudaStream_t s) {
    if (is_dev(src)) { out.p = const_cast<float*>(src); return SILI_OK; }
    CKA(cudaMalloc((void**)&out.p, (size_t)(n + 1) * 4));
    out.owned = true;
    if (n) CKA(cudaMemcpyAsync(out.p, src, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    return SILI_OK;
}
int stage_out(float* dst, int64_t n, DevArr<float>& out) {
    if (is_dev(dst)) { out.p = dst; return SILI_OK; }
    CKA(cudaMalloc((void**)&out.p, (size_t)(n + 1) * 4));
    out.owned = true;
    return SILI_OK;
}
int finish_out(float* dst, int64_t n, DevArr<float>& out, cudaStream_t s) {
    if (out.owned && n) CKA(cudaMemcpyAsync(dst, out.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    return SILI_OK;
}

int check_shape(const AttnShape& S, const char* who) {
    if (S.G < 1 || S.Gk < 1 || S.T < 0 || S.K < 0 || S.d < 0 || S.G % S.Gk || S.hbw < 0)
        return sili::set_error(SILI_EINVAL, std::string(who) + ": bad shape (groups must divide, sizes >= 0)");
    if (S.d > kMaxD) return sili::set_error(SILI_EINVAL, std::string(who) + ": head dimension above 256");
    return SILI_OK;
}

size_t fwd_smem(int64_t d) { return (size_t)kWarpsFwd * (d + 32 * (d + 1) + 32 * d) * sizeof(float); }

template <int NJ>
int launch_band(const AttnShape& S, const float* q, const float* k, const float* v, const int* sel, const int* cnt,
                int64_t stride, float* out, cudaStream_t s) {
    const size_t sm = fwd_smem(S.d);
    CKA(cudaFuncSetAttribute(k_attn_band<NJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    const int64_t nq = S.G * S.T;
    k_attn_band<NJ><<<(unsigned)((nq + kWarpsFwd - 1) / kWarpsFwd), kWarpsFwd * 32, sm, s>>>(S, q, k, v, sel, cnt,
                                                                                               stride, out);
    sili::count_launch();
    return SILI_OK;
}
int dispatch_band(const AttnShape& S, const float* q, const float* k, const float* v, const int* sel,
                  const int* cnt, int64_t stride, float* out, cudaStream_t s) {
    const int64_t nj = (S.d + 31) / 32;
    if (nj <= 1) return launch_band<1>(S, q, k, v, sel, cnt, stride, out, s);
    if (nj <= 2) return launch_band<2>(S, q, k, v, sel, cnt, stride, out, s);
    if (nj <= 4) return launch_band<4>(S, q, k, v, sel, cnt, stride, out, s);
    return launch_band<8>(S, q, k, v, sel, cnt, stride, out, s);
}

template <int NJ>
int launch_sparse(int64_t d, int64_t kk, int causal, const float* q, const float* k, const float* v, const int* qi,
                  const int* ki, float* out, cudaStream_t s) {
    const size_t sm = fwd_smem(d);
    CKA(cudaFuncSetAttribute(k_attn_sparse<NJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    k_attn_sparse<NJ><<<(unsigned)((kk + kWarpsFwd - 1) / kWarpsFwd), kWarpsFwd * 32, sm, s>>>(d, kk, causal, q, k,
                                                                                                v, qi, ki, out);
    sili::count_launch();
    return SILI_OK;
}

}  // namespace

extern "C" {

int sili_banded_attention(const float* q, const float* k, const float* v, float* out, int64_t groups,
                          int64_t kv_groups, int64_t T, int64_t K, int64_t d, int64_t half_bandwidth,
                          int64_t inner_k, int causal, void* stream) {
    AttnShape S{groups, kv_groups, T, K, d, half_bandwidth, causal ? 1 : 0};
    int rc = check_shape(S, "banded_attention");
    if (rc) return rc;
    if (inner_k < 0) return sili::set_error(SILI_EINVAL, "banded_attention: inner_k < 0");
    if (!q || !k || !v || !out) return sili::set_error(SILI_EINVAL, "banded_attention: null array");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t nq = S.G * S.T * S.d, nk = S.Gk * S.K * S.d;
    DevArr<float> dq, dk, dv, dout;
    if ((rc = stage_in(q, nq, dq, s)) || (rc = stage_in(k, nk, dk, s)) || (rc = stage_in(v, nk, dv, s)) ||
        (rc = stage_out(out, nq, dout)))
        return rc;
    if (nq > 0) {
        if (S.K == 0) {
            CKA(cudaMemsetAsync(dout.p, 0, (size_t)nq * 4, s));
        } else if (inner_k == 0) {
            if ((rc = dispatch_band(S, dq.p, dk.p, dv.p, nullptr, nullptr, 0, dout.p, s))) return rc;
        } else {
            // sparse_banded_attention_forward: select each query's top-inner_k band keys by norm
            const int64_t W = std::min<int64_t>(2 * S.hbw + 1, S.K);
            const int64_t stride = std::min<int64_t>(inner_k, W);
            float* knorm = nullptr;
            int *sel = nullptr, *cnt = nullptr;
            CKA(cudaMallocAsync((void**)&knorm, (size_t)(S.Gk * S.K + 1) * 4, s));
            CKA(cudaMallocAsync((void**)&sel, (size_t)(S.G * S.T * stride + 1) * 4, s));
            CKA(cudaMallocAsync((void**)&cnt, (size_t)(S.G * S.T + 1) * 4, s));
            k_row_sqnorm<<<(unsigned)((S.Gk * S.K + 255) / 256), 256, 0, s>>>(dk.p, S.Gk * S.K, S.d, knorm);
            k_band_select<<<(unsigned)((S.G * S.T + 3) / 4), 128, 0, s>>>(S, inner_k, knorm, sel, cnt, stride);
            sili::count_launch(2);
            rc = dispatch_band(S, dq.p, dk.p, dv.p, sel, cnt, stride, dout.p, s);
            cudaFreeAsync(knorm, s);
            cudaFreeAsync(sel, s);
            cudaFreeAsync(cnt, s);
            if (rc) return rc;
        }
    }
    CKA(cudaGetLastError());
    if ((rc = finish_out(out, nq, dout, s))) return rc;
    if (dq.owned || dout.owned || dk.owned || dv.owned) CKA(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_sparse_attention(const float* q, const float* k, const float* v, float* out, int64_t T, int64_t d,
                          int64_t top_k, int causal, void* stream) {
    if (T < 0 || d < 0 || top_k < 0 || !q || !k || !v || !out)
        return sili::set_error(SILI_EINVAL, "sparse_attention: bad arguments");
    if (d > kMaxD) return sili::set_error(SILI_EINVAL, "sparse_attention: head dimension above 256");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t n = T * d;
    DevArr<float> dq, dk, dv, dout;
    int rc;
    if ((rc = stage_in(q, n, dq, s)) || (rc = stage_in(k, n, dk, s)) || (rc = stage_in(v, n, dv, s)) ||
        (rc = stage_out(out, n, dout)))
        return rc;
    if (n > 0) CKA(cudaMemsetAsync(dout.p, 0, (size_t)n * 4, s));   // rows not selected stay zero
    if (T > 0 && d > 0) {
        // kk = top_k, or floor(sqrt(T)) (at least 1) when 0 -- attention.hpp:246-248
        const int64_t kk = top_k == 0 ? std::max<int64_t>(1, (int64_t)std::sqrt((float)T)) : std::min(top_k, T);
        float *nrm = nullptr, *nrm_o = nullptr;
        int *iota = nullptr, *idx = nullptr;
        void* tmp = nullptr;
        size_t bytes = 0;
        cub::DeviceRadixSort::SortPairsDescending(nullptr, bytes, nrm, nrm_o, iota, idx, (int)T, 0, 32, s);
        CKA(cudaMallocAsync((void**)&nrm, (size_t)T * 8, s));      // query norms, then key norms
        CKA(cudaMallocAsync((void**)&nrm_o, (size_t)T * 4, s));
        CKA(cudaMallocAsync((void**)&iota, (size_t)T * 4, s));
        CKA(cudaMallocAsync((void**)&idx, (size_t)T * 8, s));      // query order, then key order
        CKA(cudaMallocAsync(&tmp, bytes + 1, s));
        k_row_sqnorm<<<(unsigned)((T + 255) / 256), 256, 0, s>>>(dq.p, T, d, nrm);
        k_row_sqnorm<<<(unsigned)((T + 255) / 256), 256, 0, s>>>(dk.p, T, d, nrm + T);
        k_iota_i32<<<(unsigned)((T + 255) / 256), 256, 0, s>>>(iota, T);
        sili::count_launch(3);
        // a stable descending sort: equal norms keep ascending position, so the
        // lower position wins a tie at the k-th norm
        CKA(cub::DeviceRadixSort::SortPairsDescending(tmp, bytes, nrm, nrm_o, iota, idx, (int)T, 0, 32, s));
        CKA(cub::DeviceRadixSort::SortPairsDescending(tmp, bytes, nrm + T, nrm_o, iota, idx + T, (int)T, 0, 32, s));
        if (d <= 32) rc = launch_sparse<1>(d, kk, causal, dq.p, dk.p, dv.p, idx, idx + T, dout.p, s);
        else if (d <= 64) rc = launch_sparse<2>(d, kk, causal, dq.p, dk.p, dv.p, idx, idx + T, dout.p, s);
        else if (d <= 128) rc = launch_sparse<4>(d, kk, causal, dq.p, dk.p, dv.p, idx, idx + T, dout.p, s);
        else rc = launch_sparse<8>(d, kk, causal, dq.p, dk.p, dv.p, idx, idx + T, dout.p, s);
        cudaFreeAsync(tmp, s);
        cudaFreeAsync(nrm, s); cudaFreeAsync(nrm_o, s); cudaFreeAsync(iota, s); cudaFreeAsync(idx, s);
        if (rc) return rc;
    }
    CKA(cudaGetLastError());
    if ((rc = finish_out(out, n, dout, s))) return rc;
    CKA(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_banded_attention_backward(const float* q, const float* k, const float* v, const float* dO, float* dQ,
                                   float* dK, float* dV, int64_t groups, int64_t kv_groups, int64_t T, int64_t K,
                                   int64_t d, int64_t half_bandwidth, int causal, void* stream) {
    AttnShape S{groups, kv_groups, T, K, d, half_bandwidth, causal ? 1 : 0};
    int rc = check_shape(S, "banded_attention_backward");
    if (rc) return rc;
    if (!q || !k || !v || !dO || !dQ || !dK || !dV) return sili::set_error(SILI_EINVAL, "banded_attention_backward: null array");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t nq = S.G * S.T * S.d, nk = S.Gk * S.K * S.d;
    DevArr<float> dq, dk, dv, ddo, odq, odk, odv;
    if ((rc = stage_in(q, nq, dq, s)) || (rc = stage_in(k, nk, dk, s)) || (rc = stage_in(v, nk, dv, s)) ||
        (rc = stage_in(dO, nq, ddo, s)) || (rc = stage_out(dQ, nq, odq)) || (rc = stage_out(dK, nk, odk)) ||
        (rc = stage_out(dV, nk, odv)))
        return rc;
    if (nq > 0) CKA(cudaMemsetAsync(odq.p, 0, (size_t)nq * 4, s));
    if (nk > 0) {
        CKA(cudaMemsetAsync(odk.p, 0, (size_t)nk * 4, s));
        CKA(cudaMemsetAsync(odv.p, 0, (size_t)nk * 4, s));
    }
    if (S.T > 0 && S.K > 0 && S.d > 0) {
        const int64_t W = std::min<int64_t>(2 * S.hbw + 1, S.K);
        float *attn = nullptr, *ds = nullptr;
        CKA(cudaMallocAsync((void**)&attn, (size_t)(S.G * S.T * W) * 4, s));
        CKA(cudaMallocAsync((void**)&ds, (size_t)(S.G * S.T * W) * 4, s));
        k_band_bwd_q<<<(unsigned)((S.G * S.T + 3) / 4), 128, 0, s>>>(S, dq.p, dk.p, dv.p, ddo.p, W, attn, ds, odq.p);
        k_band_bwd_kv<<<(unsigned)((S.Gk * S.K + 3) / 4), 128, 0, s>>>(S, dq.p, ddo.p, W, attn, ds, odk.p, odv.p);
        sili::count_launch(2);
        cudaFreeAsync(attn, s);
        cudaFreeAsync(ds, s);
    }
    CKA(cudaGetLastError());
    if ((rc = finish_out(dQ, nq, odq, s)) || (rc = finish_out(dK, nk, odk, s)) || (rc = finish_out(dV, nk, odv, s)))
        return rc;
    CKA(cudaStreamSynchronize(s));
    return SILI_OK;
}

}  // extern "C"
