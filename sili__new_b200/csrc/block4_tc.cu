// The block4 forward and the lr = 0 block4 dx on the tensor cores (tcgen05,
// sm_100a).  The text below speaks of the forward; the dx is the same
// product transposed (linear_disldo.hpp:1512-1703 at lr = 0: dx[b, r] +=
// vs[r] * sum_c fp4(w[r, c]) * (dy[b, c] * os[c])): panels over input rows,
// chunks over output columns, the tile rows as the A operand's rows,
// dy * os split into the three bf16 terms.
//
// disldo_forward's block4 part (linear_disldo.hpp:128-339) is, for scale
// rank 1, y[b, c] += os[c] * sum_r (x[b, r] * vs[r]) * fp4(w[r, c]) over the
// 4x4 tiles: a matrix product whose weight operand is exact in bf16 (every
// FP4 value is).  The activations are not, so x' = x * vs is split into three
// bf16 terms hi + mid + lo (each the bf16 rounding of what the previous ones
// left, 24 significant bits together) and all three are multiplied in ONE
// MMA with N = 3 x 64: D[c, p * 64 + b] = sum_r W[r, c] * x'_p[b, r], fp32
// accumulation in tensor memory.  Per product the split loses at most
// 2^-24 |x'|; the result meets the fp32-accumulate tolerance of the north
// star, not the bit-exact order of the CUDA-core path (k_b4_forward), which
// stays the default.
//
// Per CTA: 128 output columns (32 block-columns) x one batch group of 64 x
// one slice of the input rows, walked in chunks of 64 rows (16 block-rows):
//   * B (the split activations, [192 x 64] bf16, 128-byte swizzled K-major)
//     arrives by TMA (cp.async.bulk.tensor) from a [groups * 192, K] buffer
//     that k_b4_xsplit fills once per call;
//   * A (the weights, [128 x 64] bf16 in the same swizzled K-major layout) is
//     written by the threads: thread (warp w, lane l) owns block-column l and
//     block-rows 4w..4w+3 of the chunk, finds their tiles through the panel
//     map (built once per tile layout: each 32-block-column x 16-block-row
//     cell's tile slot or -1), loads the next chunk's tiles while it writes
//     the current ones' codes decoded to bf16 (zeros where no tile exists);
//   * one elected thread issues four tcgen05.mma (K = 16 each) per chunk and
//     commits them to an mbarrier; A and B are double-buffered, so the next
//     chunk's A build and TMA overlap the current chunk's MMAs.
// The epilogue reads D from tensor memory (tcgen05.ld, warp w its lanes
// 32w..32w+31 = columns), adds the three split products and writes the
// slice's partial sums; k_b4_tc_reduce adds the slices in order, scales by
// os[c] and adds to y.  A non-finite result (a NaN weight code, a non-finite
// scale) is recomputed there term by term in the reference's form, so NaN
// and infinity come out where the exact path gives them.
//
// Every wait is bounded: a wait that gives up sets the call's error word,
// waits (bounded again) for the copies and MMAs it started, frees its tensor
// memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.cuh"
#include "sili_b200.h"

namespace sili {
int set_error(int code, const std::string& msg);
}

namespace sili {
namespace {

constexpr int kPanel = 128;            // output columns per CTA (MMA M)
constexpr int kBatch = 64;             // samples per batch group
constexpr int kN = 3 * kBatch;         // MMA N: hi, mid, lo
constexpr int kChunk = 64;             // input rows per chunk (MMA K 4 x 16)
constexpr int kABytes = kPanel * kChunk * 2;   // 16 KB
constexpr int kBBytes = kN * kChunk * 2;       // 24 KB
constexpr int kTmemCols = 256;
constexpr long long kSpin = 1ll << 26;         // mbarrier polls before giving up

struct TcSmem {
    alignas(1024) unsigned char a[2][kABytes];
    alignas(1024) unsigned char b[2][kBBytes];
    alignas(8) unsigned long long tma_bar[2];
    alignas(8) unsigned long long mma_bar[2];
    uint32_t tmem_base;
    uint16_t ftab[16];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// true when the phase with this parity completed; false after kSpin polls
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (long long i = 0; i < kSpin; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// shared-memory matrix descriptor: 128-byte swizzle, K-major, 8-row atoms of
// 1024 bytes (stride byte offset 1024), descriptor version 1
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint64_t start = (smem_u32(p) >> 4) & 0x3FFFu;
    return start | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: D f32, A and B bf16, both K-major
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// byte offset of element (row m, column k) of a [rows x 64] bf16 tile in
// the 128-byte swizzled K-major layout
__device__ __forceinline__ uint32_t sw128_off(int m, int k) {
    const int r = m & 7;
    return (uint32_t)((m >> 3) * 1024 + r * 128 + ((((k >> 3) ^ r) & 7) << 4) + (k & 7) * 2);
}

// The product D[m, n] = sum_k A[m, k] * B'[n, k] in either orientation: the
// forward (m = output column, k = input row) or the lr = 0 dx (m = input row,
// k = output column).
struct TcArgs {
    int64_t M, K;           // output rows (columns of y, or rows of dx) and the summed dimension
    int B, groups;          // batch, batch groups of 64
    int kslices;            // slices of the summed dimension (grid.y)
    int chunks_per_slice;
    const uint4* tile;
    const int* pmap;        // [panels][chunks][16 k-blocks][32 m-blocks] tile slot or -1
    int64_t chunks;         // chunks of the summed dimension in all
    float* part;            // [kslices][B][M] partial sums
    unsigned int* err;      // set when a wait gave up
};

template <bool DX>
__global__ void __launch_bounds__(128, 1) k_b4_tc(const __grid_constant__ CUtensorMap xmap, TcArgs P) {
    extern __shared__ unsigned char tc_raw[];
    TcSmem& S = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int panel = blockIdx.x, slice = blockIdx.y, group = blockIdx.z;
    if (threadIdx.x < 16) {
        const __nv_bfloat16 h = __float2bfloat16_rn(fp4_decode(threadIdx.x));
        S.ftab[threadIdx.x] = *reinterpret_cast<const uint16_t*>(&h);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.tma_bar[i], 1);
            mbar_init(&S.mma_bar[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = S.tmem_base;

    const int chunk0 = slice * P.chunks_per_slice;
    // this thread's four tiles of a chunk: m-block panel * 32 + lane, k-blocks
    // 4 warp .. 4 warp + 3 of the chunk, through the panel map; the next
    // chunk's are loaded while the current one is built
    const int* pm = P.pmap + ((int64_t)panel * P.chunks + chunk0) * 512 + warp * 128 + lane;
    uint4 nt[4];
    auto fetch = [&](int i) {
        int id[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) id[j] = pm[(int64_t)i * 512 + j * 32];
#pragma unroll
        for (int j = 0; j < 4; ++j) nt[j] = id[j] >= 0 ? P.tile[id[j]] : make_uint4(0, 0, 0, 0);
    };
    const int64_t left = (P.K + kChunk - 1) / kChunk - chunk0;
    const int nchunks = (int)(left < P.chunks_per_slice ? left : P.chunks_per_slice);
    constexpr uint32_t idesc = idesc_bf16(kPanel, kN);
    bool ok = true;
    // per buffer s, bit s: the barriers' phase parities and whether MMAs
    // committed to the buffer are not yet waited for (bit masks, not arrays,
    // so that they stay in registers)
    uint32_t tma_phase = 0, mma_phase = 0, issued = 0;
    // Waits on the barriers are thread 0's; the other threads learn the
    // outcome at the next __syncthreads_and, so all threads leave the loop
    // together.
    if (nchunks > 0) fetch(0);
    for (int i = 0; i < nchunks && ok; ++i) {
        const int s = i & 1;
        uint4 ct[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ct[j] = nt[j];
        if (i + 1 < nchunks) fetch(i + 1);
        // the MMAs that read this buffer two chunks ago must be done
        if ((issued >> s) & 1u) {
            if (threadIdx.x == 0 && !mbar_wait(&S.mma_bar[s], (mma_phase >> s) & 1u)) ok = false;
            mma_phase ^= 1u << s;
            issued &= ~(1u << s);
            ok = __syncthreads_and(ok ? 1 : 0) != 0;
            if (!ok) break;
        }
        if (threadIdx.x == 0) {
            mbar_expect_tx(&S.tma_bar[s], kBBytes);
            tma_load_2d(S.b[s], &xmap, (int)((chunk0 + i) * kChunk), group * kN, &S.tma_bar[s]);
        }
        // A: this thread's four tiles (zeros where none exists)
        unsigned char* A = S.a[s];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 t = ct[j];
            const int k0 = 4 * (4 * warp + j);   // the tile's first k within the chunk
            const uint32_t words[4] = {t.x, t.y, t.z, t.w};   // word lj holds slots lj*4 + li (bytes li)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t h[4];
                if (!DX) {
                    // row m = column lj = q of the tile, k = its rows li = 0..3
#pragma unroll
                    for (int li = 0; li < 4; ++li) h[li] = S.ftab[(words[q] >> (8 * li)) & 0xFu];
                } else {
                    // row m = row li = q of the tile, k = its columns lj = 0..3
#pragma unroll
                    for (int lj = 0; lj < 4; ++lj) h[lj] = S.ftab[(words[lj] >> (8 * q)) & 0xFu];
                }
                const uint2 v = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
                *reinterpret_cast<uint2*>(A + sw128_off(lane * 4 + q, k0)) = v;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        bool mma_started = false;
        if (threadIdx.x == 0) {
            if (!mbar_wait(&S.tma_bar[s], (tma_phase >> s) & 1u)) {
                ok = false;
            } else {
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint64_t ad = sw128_desc(S.a[s]), bd = sw128_desc(S.b[s]);
#pragma unroll
                for (int k = 0; k < kChunk / 16; ++k)
                    mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
                mma_commit(&S.mma_bar[s]);
                mma_started = true;
            }
        }
        tma_phase ^= 1u << s;
        if (__syncthreads_or(mma_started ? 1 : 0)) issued |= 1u << s;
        // every thread learns whether thread 0's wait gave up
        ok = __syncthreads_and(ok ? 1 : 0) != 0;
    }
    // the last MMAs complete (a give-up still waits, bounded, for what it started)
    bool fin = true;
    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s)
            if (((issued >> s) & 1u) && !mbar_wait(&S.mma_bar[s], (mma_phase >> s) & 1u)) fin = false;
    }
    ok = __syncthreads_and((ok && fin) ? 1 : 0) != 0;
    if (!ok && threadIdx.x == 0) atomicOr(P.err, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;");
    __syncthreads();
    if (ok && nchunks > 0) {
        // D row m = panel * 128 + 32 warp + lane; columns p * 64 + b
        const int64_t col = (int64_t)panel * kPanel + warp * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        float* out = P.part + (int64_t)slice * P.B * P.M;
        for (int c16 = 0; c16 < kBatch / 16; ++c16) {
            float hi[16], mi[16], lo[16];
            tmem_ld16(lane_addr + c16 * 16, hi);
            tmem_ld16(lane_addr + kBatch + c16 * 16, mi);
            tmem_ld16(lane_addr + 2 * kBatch + c16 * 16, lo);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int v = 0; v < 16; ++v) {
                const int b = group * kBatch + c16 * 16 + v;
                if (b < P.B && col < P.M) out[(int64_t)b * P.M + col] = hi[v] + mi[v] + lo[v];
            }
        }
    } else if (nchunks <= 0) {
        const int64_t col = (int64_t)panel * kPanel + warp * 32 + lane;
        float* out = P.part + (int64_t)slice * P.B * P.M;
        for (int v = 0; v < kBatch; ++v) {
            const int b = group * kBatch + v;
            if (b < P.B && col < P.M) out[(int64_t)b * P.M + col] = 0.0f;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// The panel maps: for every tile (br, bc), its slot at
// [m-block / 32][k-block / 16][k-block % 16][m-block % 32] with m = bc, k = br
// for the forward and m = br, k = bc for the dx (a warp per block-row, lanes
// over its tiles); the map starts all -1.
__global__ void k_b4_panel_map(B4View V, int dx, int64_t chunks, int* __restrict__ pmap) {
    const int lane = threadIdx.x & 31;
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (br >= V.BR) return;
    const int64_t es = V.es[br];
    const int n = V.nt[br];
    for (int k = lane; k < n; k += 32) {
        const int64_t slot = es + k;
        const int64_t bc = V.bc[slot];
        const int64_t mb = dx ? br : bc, kb = dx ? bc : br;
        pmap[((mb >> 5) * chunks + (kb >> 4)) * 512 + (kb & 15) * 32 + (mb & 31)] = (int)slot;
    }
}

// act' = act * kscale split into bf16 hi, mid, lo: row (group * 192 + p * 64
// + b), column k of a [groups * 192, K_pad] array; act is [K (+1), B] (the
// transposed x or dy); samples past B and k past K are 0
__global__ void k_b4_xsplit(const float* __restrict__ actT, const float* __restrict__ kscale, int64_t K, int B,
                            int groups, int64_t kpad, uint16_t* __restrict__ xs) {
    const int64_t total = (int64_t)groups * kBatch * kpad;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t % kpad, gb = t / kpad;
        const int g = (int)(gb / kBatch), bl = (int)(gb % kBatch);
        const int b = g * kBatch + bl;
        const float v = (r < K && b < B) ? __fmul_rn(actT[r * B + b], kscale[r]) : 0.0f;
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        const float r1 = __fsub_rn(v, __bfloat162float(h));
        const __nv_bfloat16 m = __float2bfloat16_rn(r1);
        const float r2 = __fsub_rn(r1, __bfloat162float(m));
        const __nv_bfloat16 l = __float2bfloat16_rn(r2);
        uint16_t* base = xs + ((int64_t)g * kN + bl) * kpad + r;
        base[0] = *reinterpret_cast<const uint16_t*>(&h);
        base[(int64_t)kBatch * kpad] = *reinterpret_cast<const uint16_t*>(&m);
        base[(int64_t)2 * kBatch * kpad] = *reinterpret_cast<const uint16_t*>(&l);
    }
}

// out[b, m] += mscale[m] * (partials summed in slice order).  A non-finite
// result is recomputed term by term over the tiles in the reference's form,
// so that a NaN or an infinity comes out as the exact path gives it:
//   forward (linear_disldo.hpp:128-339, no zero-input skip):
//     y[b, c]  = sum over the column's tiles and rows of x * (fp4(w) * S)
//   dx at lr = 0 (:1512-1703): dx[b, r] = sum over the row's tiles and
//     columns of fp4(w) * (S * dy)
template <bool DX>
__global__ void k_b4_tc_reduce(const float* __restrict__ part, int kslices, int B, LayerView L, B4View V,
                               const float* __restrict__ actT, float* __restrict__ out) {
    const int64_t M = DX ? L.n_in : L.n_out;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)B * M) return;
    const int64_t b = t / M, m = t % M;
    float v = 0.0f;
    for (int k = 0; k < kslices; ++k) v += part[(int64_t)k * B * M + t];
    float add = v * (DX ? L.vs[m] : L.os[m]);
    if (!isfinite(add)) {
        float acc = 0.0f;
        if (!DX) {
            const int64_t bc = m >> 2;
            const int lj = (int)(m & 3);
            for (int q = V.cptr[bc]; q < V.cptr[bc + 1]; ++q) {
                const uint4 tw = V.tile[V.ctile[q]];
                const uint32_t word = lj == 0 ? tw.x : lj == 1 ? tw.y : lj == 2 ? tw.z : tw.w;
                for (int li = 0; li < 4; ++li) {
                    const int64_t r = (int64_t)V.cbr[q] * 4 + li;
                    if (r >= L.n_in) break;
                    acc += actT[r * B + b] * (fp4_decode((word >> (8 * li)) & 0xFu) * (L.vs[r] * L.os[m]));
                }
            }
        } else {
            const int64_t br = m >> 2;
            const int li = (int)(m & 3);
            const int64_t es = V.es[br];
            for (int q = 0; q < V.nt[br]; ++q) {
                const uint4 tw = V.tile[es + q];
                const uint32_t words[4] = {tw.x, tw.y, tw.z, tw.w};
                for (int lj = 0; lj < 4; ++lj) {
                    const int64_t c = (int64_t)V.bc[es + q] * 4 + lj;
                    if (c >= L.n_out) break;
                    acc += fp4_decode((words[lj] >> (8 * li)) & 0xFu) * ((L.vs[m] * L.os[c]) * actT[c * B + b]);
                }
            }
        }
        add = acc;
    }
    out[t] += add;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

int64_t dims_m(const LayerView& L, bool dx) { return dx ? L.n_in : L.n_out; }
int64_t dims_k(const LayerView& L, bool dx) { return dx ? L.n_out : L.n_in; }

}  // namespace

bool b4_tc_applies(const LayerView& L, const B4View& V, int B) {
    return L.rank == 1 && V.BC > 0 && B >= 16 && L.n_in > 0 && L.n_out > 0 && V.cptr != nullptr;
}

int64_t b4_tc_scratch_floats(const LayerView& L, int B, bool dx, int* kslices) {
    const int64_t panels = (dims_m(L, dx) + kPanel - 1) / kPanel;
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t chunks = (dims_k(L, dx) + kChunk - 1) / kChunk;
    // slices of the summed dimension so that panels x groups x slices fill the
    // SMs about twice (two CTAs fit per SM: 84 KB of shared memory, 256
    // tensor-memory columns each), at least 4 chunks per slice
    int64_t k = std::max<int64_t>(1, (2 * 148) / std::max<int64_t>(1, panels * groups));
    k = std::min<int64_t>(k, std::max<int64_t>(1, chunks / 4));
    *kslices = (int)k;
    return k * (int64_t)B * dims_m(L, dx);
}

int64_t b4_tc_pmap_elems(const LayerView& L, bool dx) {
    const int64_t panels = (dims_m(L, dx) + kPanel - 1) / kPanel;
    const int64_t chunks = (dims_k(L, dx) + kChunk - 1) / kChunk;
    return panels * chunks * 512;
}

void launch_b4_panel_map(const LayerView& L, const B4View& V, bool dx, int* pmap, cudaStream_t s) {
    const int64_t chunks = (dims_k(L, dx) + kChunk - 1) / kChunk;
    cudaMemsetAsync(pmap, 0xFF, (size_t)b4_tc_pmap_elems(L, dx) * sizeof(int), s);
    if (V.BR > 0) {
        k_b4_panel_map<<<(unsigned)((V.BR + 7) / 8), 256, 0, s>>>(V, dx ? 1 : 0, chunks, pmap);
        count_launch();
    }
}

int64_t b4_tc_xsplit_elems(const LayerView& L, int B, bool dx) {
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t kpad = (dims_k(L, dx) + kChunk - 1) / kChunk * kChunk;
    return (int64_t)groups * kN * kpad;
}

template <bool DX>
static int launch_tc(const LayerView& L, const B4View& V, const float* actT, int B, float* out, uint16_t* xsplit,
                     float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(SILI_ECUDA, "block4 tensor-core kernel: cuTensorMapEncodeTiled unavailable");
    const int64_t M = dims_m(L, DX), K = dims_k(L, DX);
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t kpad = (K + kChunk - 1) / kChunk * kChunk;
    const int64_t chunks = kpad / kChunk;
    k_b4_xsplit<<<(unsigned)std::min<int64_t>((groups * kBatch * kpad + 255) / 256, 148 * 32), 256, 0, s>>>(
        actT, DX ? L.os : L.vs, K, B, groups, kpad, xsplit);
    count_launch();
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    const cuuint64_t dims[2] = {(cuuint64_t)kpad, (cuuint64_t)groups * kN};
    const cuuint64_t strides[1] = {(cuuint64_t)kpad * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)kN};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xsplit, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SILI_ECUDA, "block4 tensor-core kernel: tensor map encoding failed");
    TcArgs P;
    P.M = M; P.K = K; P.B = B; P.groups = groups; P.kslices = kslices;
    P.chunks_per_slice = (int)((chunks + kslices - 1) / kslices);
    P.tile = V.tile; P.pmap = pmap; P.chunks = chunks;
    P.part = part; P.err = err;
    const size_t smem = sizeof(TcSmem) + 1024;
    static unsigned long long attr_devices = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(attr_devices & (1ull << dev))) {
        cudaFuncSetAttribute(k_b4_tc<DX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr_devices |= 1ull << dev;
    }
    dim3 g((unsigned)((M + kPanel - 1) / kPanel), (unsigned)kslices, (unsigned)groups);
    k_b4_tc<DX><<<g, 128, smem, s>>>(map, P);
    const int64_t n = (int64_t)B * M;
    k_b4_tc_reduce<DX><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, kslices, B, L, V, actT, out);
    count_launch(2);
    return SILI_OK;
}

int launch_b4_forward_tc(const LayerView& L, const B4View& V, const float* xT, int B, float* y, uint16_t* xsplit,
                         float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s) {
    return launch_tc<false>(L, V, xT, B, y, xsplit, part, kslices, pmap, err, s);
}

int launch_b4_dx_tc(const LayerView& L, const B4View& V, const float* dyT, int B, float* dx, uint16_t* xsplit,
                    float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s) {
    return launch_tc<true>(L, V, dyT, B, dx, xsplit, part, kslices, pmap, err, s);
}

}  // namespace sili
