// The block4 forward on the tensor cores (tcgen05, sm_100a).
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

struct TcArgs {
    int64_t n_in, n_out;
    int B, groups;          // batch, batch groups of 64
    int kslices;            // input-row slices (grid.y)
    int chunks_per_slice;
    int64_t BC;             // block-columns
    const int* cptr;        // tile column index
    const int* ctile;
    const int* cbr;
    const uint4* tile;
    const int* pmap;        // [panels][chunks][16 block-rows][32 block-columns] tile slot or -1
    int64_t chunks;         // chunks of the input rows in all
    float* part;            // [kslices][B][n_out] partial sums
    unsigned int* err;      // set when a wait gave up
};

__global__ void __launch_bounds__(128, 1) k_b4_forward_tc(const __grid_constant__ CUtensorMap xmap, TcArgs P) {
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
    // this thread's four tiles of a chunk: block-column panel * 32 + lane,
    // block-rows 4 warp .. 4 warp + 3 of the chunk, through the panel map;
    // the next chunk's are loaded while the current one is built
    const int* pm = P.pmap + ((int64_t)panel * P.chunks + chunk0) * 512 + warp * 128 + lane;
    uint4 nt[4];
    auto fetch = [&](int i) {
        int id[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) id[j] = pm[(int64_t)i * 512 + j * 32];
#pragma unroll
        for (int j = 0; j < 4; ++j) nt[j] = id[j] >= 0 ? P.tile[id[j]] : make_uint4(0, 0, 0, 0);
    };
    const int64_t left = (P.n_in + kChunk - 1) / kChunk - chunk0;
    const int nchunks = (int)(left < P.chunks_per_slice ? left : P.chunks_per_slice);
    constexpr uint32_t idesc = idesc_bf16(kPanel, kN);
    bool ok = true;
    uint32_t tma_phase[2] = {0, 0}, mma_phase[2] = {0, 0};
    int issued[2] = {0, 0};   // MMA groups committed to each buffer and not yet waited for
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
        if (issued[s]) {
            if (threadIdx.x == 0 && !mbar_wait(&S.mma_bar[s], mma_phase[s])) ok = false;
            mma_phase[s] ^= 1;
            issued[s] = 0;
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
            const int k0 = 4 * (4 * warp + j);   // the tile's first row within the chunk
            const uint32_t words[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int lj = 0; lj < 4; ++lj) {
                const uint32_t wd = words[lj];   // slots lj*4 + li, li = 0..3 (bytes)
                const uint32_t h0 = S.ftab[wd & 0xFu], h1 = S.ftab[(wd >> 8) & 0xFu];
                const uint32_t h2 = S.ftab[(wd >> 16) & 0xFu], h3 = S.ftab[(wd >> 24) & 0xFu];
                const uint2 v = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
                *reinterpret_cast<uint2*>(A + sw128_off(lane * 4 + lj, k0)) = v;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        bool mma_started = false;
        if (threadIdx.x == 0) {
            if (!mbar_wait(&S.tma_bar[s], tma_phase[s])) {
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
        tma_phase[s] ^= 1;
        issued[s] = __syncthreads_or(mma_started ? 1 : 0);
        // every thread learns whether thread 0's wait gave up
        ok = __syncthreads_and(ok ? 1 : 0) != 0;
    }
    // the last MMAs complete (a give-up still waits, bounded, for what it started)
    bool fin = true;
    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s)
            if (issued[s] && !mbar_wait(&S.mma_bar[s], mma_phase[s])) fin = false;
    }
    ok = __syncthreads_and((ok && fin) ? 1 : 0) != 0;
    if (!ok && threadIdx.x == 0) atomicOr(P.err, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;");
    __syncthreads();
    if (ok && nchunks > 0) {
        // D row = output column panel * 128 + 32 warp + lane; columns p * 64 + b
        const int64_t col = (int64_t)panel * kPanel + warp * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        float* out = P.part + (int64_t)slice * P.B * P.n_out;
        for (int c16 = 0; c16 < kBatch / 16; ++c16) {
            float hi[16], mi[16], lo[16];
            tmem_ld16(lane_addr + c16 * 16, hi);
            tmem_ld16(lane_addr + kBatch + c16 * 16, mi);
            tmem_ld16(lane_addr + 2 * kBatch + c16 * 16, lo);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int v = 0; v < 16; ++v) {
                const int b = group * kBatch + c16 * 16 + v;
                if (b < P.B && col < P.n_out) out[(int64_t)b * P.n_out + col] = hi[v] + mi[v] + lo[v];
            }
        }
    } else if (nchunks <= 0) {
        const int64_t col = (int64_t)panel * kPanel + warp * 32 + lane;
        float* out = P.part + (int64_t)slice * P.B * P.n_out;
        for (int v = 0; v < kBatch; ++v) {
            const int b = group * kBatch + v;
            if (b < P.B && col < P.n_out) out[(int64_t)b * P.n_out + col] = 0.0f;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// The panel map: for every tile, its slot at [bc / 32][br / 16][br % 16][bc % 32]
// (a warp per block-row, lanes over its tiles); the map starts all -1.
__global__ void k_b4_panel_map(B4View V, int64_t chunks, int* __restrict__ pmap) {
    const int lane = threadIdx.x & 31;
    const int64_t br = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (br >= V.BR) return;
    const int64_t es = V.es[br];
    const int n = V.nt[br];
    for (int k = lane; k < n; k += 32) {
        const int64_t slot = es + k;
        const int64_t bc = V.bc[slot];
        pmap[((bc >> 5) * chunks + (br >> 4)) * 512 + (br & 15) * 32 + (bc & 31)] = (int)slot;
    }
}

// x' = x * vs split into bf16 hi, mid, lo: row
// (group * 192 + p * 64 + b), column r of a [groups * 192, K_pad] array;
// samples past B and rows past n_in are 0
__global__ void k_b4_xsplit(const float* __restrict__ xT, const float* __restrict__ vs, int64_t n_in, int B,
                            int groups, int64_t kpad, uint16_t* __restrict__ xs) {
    const int64_t total = (int64_t)groups * kBatch * kpad;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t % kpad, gb = t / kpad;
        const int g = (int)(gb / kBatch), bl = (int)(gb % kBatch);
        const int b = g * kBatch + bl;
        const float v = (r < n_in && b < B) ? __fmul_rn(xT[r * B + b], vs[r]) : 0.0f;
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

// y[b, c] += os[c] * (partials summed in slice order); a non-finite result is
// recomputed term by term over the column's tiles in the reference's form
// x * (fp4(w) * S) (no zero-input skip in the block4 forward), so that a NaN
// or an infinity comes out as the exact path gives it
__global__ void k_b4_tc_reduce(const float* __restrict__ part, int kslices, int B, int64_t n_out,
                               const float* __restrict__ os, const float* __restrict__ vs, const float* __restrict__ xT,
                               int64_t n_in, const int* __restrict__ cptr, const int* __restrict__ ctile,
                               const int* __restrict__ cbr, const uint4* __restrict__ tile, float* __restrict__ y) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)B * n_out) return;
    const int64_t b = t / n_out, c = t % n_out;
    float v = 0.0f;
    for (int k = 0; k < kslices; ++k) v += part[(int64_t)k * B * n_out + t];
    float add = v * os[c];
    if (!isfinite(add)) {
        const int64_t bc = c >> 2;
        const int lj = (int)(c & 3);
        float acc = 0.0f;
        for (int q = cptr[bc]; q < cptr[bc + 1]; ++q) {
            const uint4 tw = tile[ctile[q]];
            const uint32_t word = lj == 0 ? tw.x : lj == 1 ? tw.y : lj == 2 ? tw.z : tw.w;
            for (int li = 0; li < 4; ++li) {
                const int64_t r = (int64_t)cbr[q] * 4 + li;
                if (r >= n_in) break;
                acc += xT[r * B + b] * (fp4_decode((word >> (8 * li)) & 0xFu) * (vs[r] * os[c]));
            }
        }
        add = acc;
    }
    y[t] += add;
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

}  // namespace

bool b4_tc_applies(const LayerView& L, const B4View& V, int B) {
    return L.rank == 1 && V.BC > 0 && B >= 16 && L.n_in > 0 && V.cptr != nullptr;
}

int64_t b4_tc_scratch_floats(const LayerView& L, int B, int* kslices) {
    const int64_t panels = (L.n_out + kPanel - 1) / kPanel;
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t chunks = (L.n_in + kChunk - 1) / kChunk;
    // slices of the input rows so that panels x groups x slices fill the
    // SMs about twice (two CTAs fit per SM: 88 KB of shared memory, 256
    // tensor-memory columns each), at least 4 chunks per slice
    int64_t k = std::max<int64_t>(1, (2 * 148) / std::max<int64_t>(1, panels * groups));
    k = std::min<int64_t>(k, std::max<int64_t>(1, chunks / 4));
    *kslices = (int)k;
    return k * (int64_t)B * L.n_out;
}

int64_t b4_tc_pmap_elems(const LayerView& L) {
    const int64_t panels = (L.n_out + kPanel - 1) / kPanel;
    const int64_t chunks = (L.n_in + kChunk - 1) / kChunk;
    return panels * chunks * 512;
}

void launch_b4_panel_map(const LayerView& L, const B4View& V, int* pmap, cudaStream_t s) {
    const int64_t chunks = (L.n_in + kChunk - 1) / kChunk;
    cudaMemsetAsync(pmap, 0xFF, (size_t)b4_tc_pmap_elems(L) * sizeof(int), s);
    if (V.BR > 0) {
        k_b4_panel_map<<<(unsigned)((V.BR + 7) / 8), 256, 0, s>>>(V, chunks, pmap);
        count_launch();
    }
}

int64_t b4_tc_xsplit_elems(const LayerView& L, int B) {
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t kpad = (L.n_in + kChunk - 1) / kChunk * kChunk;
    return (int64_t)groups * kN * kpad;
}

int launch_b4_forward_tc(const LayerView& L, const B4View& V, const float* xT, int B, float* y, uint16_t* xsplit,
                         float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(SILI_ECUDA, "block4 tensor-core forward: cuTensorMapEncodeTiled unavailable");
    const int groups = (B + kBatch - 1) / kBatch;
    const int64_t kpad = (L.n_in + kChunk - 1) / kChunk * kChunk;
    const int64_t chunks = kpad / kChunk;
    k_b4_xsplit<<<(unsigned)std::min<int64_t>((groups * kBatch * kpad + 255) / 256, 148 * 32), 256, 0, s>>>(
        xT, L.vs, L.n_in, B, groups, kpad, xsplit);
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
    if (r != CUDA_SUCCESS) return set_error(SILI_ECUDA, "block4 tensor-core forward: tensor map encoding failed");
    TcArgs P;
    P.n_in = L.n_in; P.n_out = L.n_out; P.B = B; P.groups = groups; P.kslices = kslices;
    P.chunks_per_slice = (int)((chunks + kslices - 1) / kslices);
    P.BC = V.BC; P.cptr = V.cptr; P.ctile = V.ctile; P.cbr = V.cbr; P.tile = V.tile;
    P.pmap = pmap; P.chunks = chunks;
    P.part = part; P.err = err;
    const size_t smem = sizeof(TcSmem) + 1024;
    static unsigned long long attr_devices = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(attr_devices & (1ull << dev))) {
        cudaFuncSetAttribute(k_b4_forward_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr_devices |= 1ull << dev;
    }
    dim3 g((unsigned)((L.n_out + kPanel - 1) / kPanel), (unsigned)kslices, (unsigned)groups);
    k_b4_forward_tc<<<g, 128, smem, s>>>(map, P);
    const int64_t n = (int64_t)B * L.n_out;
    k_b4_tc_reduce<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, kslices, B, L.n_out, L.os, L.vs, xT, L.n_in,
                                                              V.cptr, V.ctile, V.cbr, V.tile, y);
    count_launch(2);
    return SILI_OK;
}

}  // namespace sili
