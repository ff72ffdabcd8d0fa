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
// One thread per output column, 32 samples per CTA (acc[32] in registers).
// Per tile of RT input rows the CTA stages x[rows][32 samples] into shared
// memory (8 float4 chunks of a 128-byte row); each thread then consumes its
// column's entries whose row lies in the tile, in ascending row order, 32
// fmas per entry, the next entry's packed word loaded ahead.  Lane l reads
// chunk q ^ (l mod 8) at step q (its accumulator 4q + v holds sample
// 4 (q ^ (l mod 8)) + v): the 8 lanes of a quarter-warp then always touch 8
// different bank groups, whatever rows they read, and with the tile 128-byte
// aligned the chunk address is one xor of the row address.  Weight codes are
// decoded through a 16-entry table in shared memory.
constexpr int kFcSg = 32;   // samples per CTA

__device__ __forceinline__ float4 lds128(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

template <bool SPARSE>
__global__ void __launch_bounds__(256, 3) k_forward_cols(LayerView L, const float* __restrict__ xT, int B, int RT,
                                                      float* __restrict__ y) {
    // [pad to 128 B][RT][8] chunks of 4 samples, then vs of the RT rows, then the code table
    extern __shared__ __align__(16) unsigned char fc_smem[];
    const uint32_t raw32 = (uint32_t)__cvta_generic_to_shared(fc_smem);
    const uint32_t pad = (128u - (raw32 & 127u)) & 127u;
    float4* xs4 = reinterpret_cast<float4*>(fc_smem + pad);
    const uint32_t xs32 = raw32 + pad;
    float* vs_t = reinterpret_cast<float*>(xs4 + RT * 8);
    float* ftab = vs_t + RT;
    if (threadIdx.x < 16) ftab[threadIdx.x] = fp4_decode(threadIdx.x);
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int b0 = blockIdx.y * kFcSg;
    const int n_in = (int)L.n_in;
    const uint32_t rot16 = (threadIdx.x & 7) << 4;
    int cur = 0, end = 0;
    float oc = 0.0f;
    if (c < L.n_out) {
        cur = L.colptr[c];
        end = cur + (L.colptr_x[c + 1] - L.colptr_x[c]);
        oc = L.os[c];
    }
    float acc[kFcSg];
#pragma unroll
    for (int v = 0; v < kFcSg; ++v) acc[v] = 0.0f;
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
        for (int t = threadIdx.x; t < nr * 8; t += blockDim.x) {
            const int i = t >> 3, q = t & 7;
            const int b = b0 + 4 * q;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (b < B) v = __ldg(reinterpret_cast<const float4*>(xT + (int64_t)(R0 + i) * B + b));
            xs4[i * 8 + q] = v;
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
            const uint32_t rowa = (xs32 + ((uint32_t)ri << 7)) ^ rot16;
            if (isfinite(w) && (!SPARSE || isfinite(cs))) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
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
                for (int q = 0; q < 8; ++q) {
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
        const int rot = threadIdx.x & 7;
#pragma unroll
        for (int k = 0; k < kFcSg; ++k) {
            const int b = b0 + 4 * ((k >> 2) ^ rot) + (k & 3);
            if (b < B) y[(int64_t)b * L.n_out + c] = acc[k];
        }
    }
}

namespace {
struct ColsPlan {
    int threads = 0, rt = 0;
};
// 256-thread CTAs when that still gives every SM two CTAs, else 128; no plan
// (threads 0) for narrower layers
ColsPlan cols_plan(const LayerView& L, int B) {
    ColsPlan p;
    if (L.rank != 1 || B < 16 || (B & 3) != 0 || L.n_in >= (1 << 27) || L.n_out == 0 || L.n_in == 0) return p;
    const int64_t sgroups = (B + kFcSg - 1) / kFcSg;
    // a CTA re-reads all of x; below 128 columns per CTA that costs more
    // than the per-synapse gathers of k_forward_vec
    int t = 256;
    if (((L.n_out + t - 1) / t) * sgroups < 2 * 148) t = 128;
    if (((L.n_out + t - 1) / t) * sgroups < 2 * 148) return p;
    p.threads = t;
    // x tile: 128 bytes per row, 64 KB (3 CTAs per SM).  Smaller tiles for
    // 128-thread CTAs (more CTAs per SM) measured no faster: the per-tile
    // maximum of the lanes' entry counts grows relative to the mean.
    p.rt = (int)std::min<int64_t>(L.n_in, 512);
    return p;
}
}  // namespace

bool forward_rows_applies(const LayerView& L, int B) { return cols_plan(L, B).threads > 0; }

bool launch_forward_rows(const LayerView& L, const float* xT, int B, float* y, bool sparse, cudaStream_t s) {
    const ColsPlan p = cols_plan(L, B);
    if (p.threads == 0 || !L.cpack || !L.colptr_x) return false;
    const size_t smem = 128 + (size_t)p.rt * (8 * sizeof(float4) + sizeof(float)) + 16 * sizeof(float);
    static unsigned long long attr_devices = 0;   // the attribute is per device and kernel
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(attr_devices & (1ull << dev))) {
        cudaFuncSetAttribute(k_forward_cols<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        cudaFuncSetAttribute(k_forward_cols<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        attr_devices |= 1ull << dev;
    }
    dim3 g((unsigned)((L.n_out + p.threads - 1) / p.threads), (unsigned)((B + kFcSg - 1) / kFcSg));
    if (sparse) k_forward_cols<true><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y);
    else k_forward_cols<false><<<g, p.threads, smem, s>>>(L, xT, B, p.rt, y);
    count_launch();
    return true;
}

}  // namespace sili
