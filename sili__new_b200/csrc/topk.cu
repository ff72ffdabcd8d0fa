// The top-k |dy^T x| growth rule on the device: exact top-k of
// |sum_b x[b,r] dy[b,c]| over non-existing (r, c), prune as many existing
// synapses of smallest |w * S(r,c)|, rebuild the delta-CSR.  No reference
// function exists; the rule is defined (and restated on the CPU by
// oracle/sili_oracle.c, o_topk_dyx_*) as: s = fma(x[b,r], dy[b,c], s) for
// b = 0..B-1 from s = 0 (so the score is bit-reproducible), ties toward lower
// (r, c) on both sides, new synapses stored as delta_csr_synap_row_step
// stores them (weight 0, importance fp4(score)).
#include "common.cuh"
#include "kernels.cuh"

namespace sili {

// existence bitmap [n_in, ceil(n_out/32)] from the decoded columns
__global__ void k_exist_bits(const int* __restrict__ rowptr, const int* __restrict__ abs_cols, int64_t n_in,
                             int64_t words, uint32_t* __restrict__ bits) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n_in) return;
    for (int f = rowptr[r] + lane; f < rowptr[r + 1]; f += 32) {
        const int c = abs_cols[f];
        atomicOr(bits + r * words + (c >> 5), 1u << (c & 31));
    }
}
void launch_exist_bits(const int* rowptr, const int* abs_cols, int64_t n_in, int64_t words, uint32_t* bits,
                       cudaStream_t s) {
    if (n_in == 0) return;
    k_exist_bits<<<(unsigned)((n_in + 7) / 8), 256, 0, s>>>(rowptr, abs_cols, n_in, words, bits);
    count_launch();
}

// Scores as 32-bit keys: 0 for an existing synapse, bits(|s|) + 1 otherwise
// (|s| >= 0, so key order is score order).  128 x 128 output tile per block,
// 8 x 8 per thread (rows ty*8.., columns tx*8..: both read from shared memory
// as two 16-byte loads), samples staged 16 at a time; each output
// accumulates its fma chain over b in ascending order, as the rule defines.
// With row lengths that are multiples of 4 floats (ASYNC), the next 16
// samples' x and dy tiles are copied by cp.async into the second of two
// buffers while the current ones are consumed.
constexpr int kTM = 128, kTN = 128, kTK = 16;

__device__ __forceinline__ void sc_cp16(float* smem, const float* gmem, bool take) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gmem), "r"(take ? 16 : 0)
                 : "memory");
}

template <bool ASYNC>
__global__ void __launch_bounds__(256) k_dyx_scores(const float* __restrict__ x, const float* __restrict__ dy, int B,
                                                    int64_t n_in, int64_t n_out, const uint32_t* __restrict__ bits,
                                                    int64_t words, uint32_t* __restrict__ keys) {
    __shared__ __align__(16) float xs[ASYNC ? 2 : 1][kTK][kTM];
    __shared__ __align__(16) float ds[ASYNC ? 2 : 1][kTK][kTN];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t r0 = (int64_t)blockIdx.y * kTM, c0 = (int64_t)blockIdx.x * kTN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    // 16 samples x 128 floats of x and of dy: 512 16-byte groups each, two
    // per thread; groups past B or past the matrix edge are zero-filled
    auto stage_async = [&](int buf, int b0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int t = threadIdx.x + h * 256;
            const int k = t >> 5, i4 = (t & 31) * 4;
            const int b = b0 + k;
            const bool tx_ = b < B && r0 + i4 < n_in;
            const bool td = b < B && c0 + i4 < n_out;
            sc_cp16(&xs[buf][k][i4], tx_ ? x + (int64_t)b * n_in + r0 + i4 : x, tx_);
            sc_cp16(&ds[buf][k][i4], td ? dy + (int64_t)b * n_out + c0 + i4 : dy, td);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    auto compute = [&](int buf, int kn) {
        for (int k = 0; k < kn; ++k) {
            const float4 xa = *reinterpret_cast<const float4*>(&xs[buf][k][ty * 8]);
            const float4 xb = *reinterpret_cast<const float4*>(&xs[buf][k][ty * 8 + 4]);
            const float4 da = *reinterpret_cast<const float4*>(&ds[buf][k][tx * 8]);
            const float4 db = *reinterpret_cast<const float4*>(&ds[buf][k][tx * 8 + 4]);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            const float dv[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(xv[i], dv[j], acc[i][j]);
        }
    };
    if (ASYNC) {
        int buf = 0;
        if (B > 0) stage_async(0, 0);
        for (int b0 = 0; b0 < B; b0 += kTK) {
            if (b0 + kTK < B) {
                stage_async(buf ^ 1, b0 + kTK);
                asm volatile("cp.async.wait_group 1;\n" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            }
            __syncthreads();
            compute(buf, min(kTK, B - b0));
            __syncthreads();   // the buffer is refilled two tiles on
            buf ^= 1;
        }
    } else {
        for (int b0 = 0; b0 < B; b0 += kTK) {
            for (int t = threadIdx.x; t < kTK * kTM; t += 256) {
                const int k = t / kTM, i = t % kTM;
                const int b = b0 + k;
                xs[0][k][i] = (b < B && r0 + i < n_in) ? x[(int64_t)b * n_in + r0 + i] : 0.0f;
                ds[0][k][i] = (b < B && c0 + i < n_out) ? dy[(int64_t)b * n_out + c0 + i] : 0.0f;
            }
            __syncthreads();
            compute(0, min(kTK, B - b0));
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t r = r0 + ty * 8 + i;
        if (r >= n_in) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t c = c0 + tx * 8 + j;
            if (c >= n_out) continue;
            const bool ex = (bits[r * words + (c >> 5)] >> (c & 31)) & 1u;
            keys[r * n_out + c] = ex ? 0u : __float_as_uint(fabsf(acc[i][j])) + 1u;
        }
    }
}
void launch_dyx_scores(const float* x, const float* dy, int B, int64_t n_in, int64_t n_out, const uint32_t* bits,
                       int64_t words, uint32_t* keys, cudaStream_t s) {
    if (n_in == 0 || n_out == 0) return;
    dim3 g((unsigned)((n_out + kTN - 1) / kTN), (unsigned)((n_in + kTM - 1) / kTM));
    // 16-byte copies need 16-byte aligned rows and bases
    const bool async = (n_in % 4 == 0) && (n_out % 4 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)dy % 16 == 0);
    if (async) k_dyx_scores<true><<<g, 256, 0, s>>>(x, dy, B, n_in, n_out, bits, words, keys);
    else k_dyx_scores<false><<<g, 256, 0, s>>>(x, dy, B, n_in, n_out, bits, words, keys);
    count_launch();
}

// Radix select of the k-th largest key, 8 bits at a time from the top, with
// its state on the device (no host round trip per digit):
// k_sel_init -> 4 x (histogram of the digit among keys matching the prefix so
// far, k_digit_pick) -> prefix = the k-th largest key, need = how many keys
// equal to it are taken, eq_count = how many there are.
__global__ void k_sel_init(SelState* st, int64_t need) {
    st->prefix = 0u;
    st->mask = 0u;
    st->need = need;
    st->eq_count = 0;
}
void launch_sel_init(SelState* st, int64_t need, cudaStream_t s) {
    k_sel_init<<<1, 1, 0, s>>>(st, need);
    count_launch();
}

__global__ void k_digit_hist(const uint32_t* __restrict__ keys, int64_t n, int shift, const SelState* __restrict__ st,
                             unsigned int* __restrict__ hist) {
    __shared__ unsigned int h[256];
    const uint32_t mask = st->mask, prefix = st->prefix;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t k = keys[i];
        if ((k & mask) == prefix) atomicAdd(&h[(k >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (h[i]) atomicAdd(hist + i, h[i]);
}
void launch_digit_hist(const uint32_t* keys, int64_t n, int shift, const SelState* st, unsigned int* hist, int sms,
                       cudaStream_t s) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
    k_digit_hist<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, s>>>(keys, n, shift, st, hist);
    count_launch();
}

// the digit holding the need-th largest key; clears the histogram for the next pass
__global__ void k_digit_pick(unsigned int* __restrict__ hist, int shift, SelState* __restrict__ st) {
    if (threadIdx.x == 0) {
        int64_t cum = 0;
        int d = 255;
        for (; d > 0; --d) {
            if (cum + (int64_t)hist[d] >= st->need) break;
            cum += hist[d];
        }
        st->need -= cum;
        st->eq_count = hist[d];
        st->prefix |= (uint32_t)d << shift;
        st->mask |= 0xFFu << shift;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
}
void launch_digit_pick(unsigned int* hist, int shift, SelState* st, cudaStream_t s) {
    k_digit_pick<<<1, 256, 0, s>>>(hist, shift, st);
    count_launch();
}

// flat indices of every key >= thr (the caller has checked that this is
// exactly the k wanted: every key equal to the threshold is taken), appended
// in arbitrary order with one atomic per warp; the caller sorts them
__global__ void k_select_ge(const uint32_t* __restrict__ keys, int64_t n, const SelState* __restrict__ st,
                            int64_t* __restrict__ out, unsigned long long* __restrict__ count, int64_t cap) {
    const uint32_t thr = st->prefix;
    const int lane = threadIdx.x & 31;
    const int64_t n4 = n >> 2;   // whole 16-byte groups; the tail below
    const uint4* k4 = reinterpret_cast<const uint4*>(keys);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    auto emit = [&](bool sel, int64_t i) {   // warp-wide: one atomic per warp
        const unsigned m = __ballot_sync(0xffffffffu, sel);
        if (m == 0u) return;
        unsigned long long b = 0;
        if (lane == 0) b = atomicAdd(count, (unsigned long long)__popc(m));
        b = __shfl_sync(0xffffffffu, b, 0);
        if (sel) {
            const int64_t slot = (int64_t)b + __popc(m & ((1u << lane) - 1u));
            if (slot < cap) out[slot] = i;
        }
    };
    for (int64_t g0 = (int64_t)blockIdx.x * blockDim.x; g0 < n4; g0 += stride) {   // warp-uniform trip count
        const int64_t g = g0 + threadIdx.x;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        const bool ok = g < n4;
        if (ok) v = __ldg(k4 + g);
        emit(ok && v.x >= thr, 4 * g + 0);
        emit(ok && v.y >= thr, 4 * g + 1);
        emit(ok && v.z >= thr, 4 * g + 2);
        emit(ok && v.w >= thr, 4 * g + 3);
    }
    if (blockIdx.x == 0 && threadIdx.x < 32) {
        const int64_t i = 4 * n4 + threadIdx.x;
        emit(i < n && keys[i] >= thr, i);
    }
}
void launch_select_ge(const uint32_t* keys, int64_t n, const SelState* st, int64_t* out, unsigned long long* count,
                      int64_t cap, int sms, cudaStream_t s) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
    k_select_ge<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, s>>>(keys, n, st, out, count, cap);
    count_launch();
}

// prune keys: bits(|w * S(r, c)|) per existing synapse, in export order
__global__ void k_prune_keys(LayerView L, const float* __restrict__ w, uint32_t* __restrict__ keys,
                             int* __restrict__ ids) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= L.n_in) return;
    for (int f = L.rowptr[r] + lane; f < L.rowptr[r + 1]; f += 32) {
        const int64_t c = L.abs_cols[f];
        float S = 0.0f;
        for (int k = 0; k < L.rank; ++k) S = __fmaf_rn(L.vs[r * L.rank + k], L.os[c * L.rank + k], S);
        keys[f] = __float_as_uint(fabsf(__fmul_rn(w[f], S)));
        ids[f] = f;
    }
}
void launch_prune_keys(const LayerView& L, const float* w, uint32_t* keys, int* ids, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_prune_keys<<<(unsigned)((L.n_in + 7) / 8), 256, 0, s>>>(L, w, keys, ids);
    count_launch();
}

// drop flags for the first npr synapses of the sorted order; out_degree -1
__global__ void k_mark_drop(const int* __restrict__ sorted_ids, int npr, const int* __restrict__ abs_cols,
                            uint8_t* __restrict__ drop, int* __restrict__ out_degree) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= npr) return;
    const int f = sorted_ids[i];
    drop[f] = 1;
    atomicSub(out_degree + abs_cols[f], 1);
}
void launch_mark_drop(const int* sorted_ids, int npr, const int* abs_cols, uint8_t* drop, int* out_degree,
                      cudaStream_t s) {
    if (npr <= 0) return;
    k_mark_drop<<<(unsigned)((npr + 255) / 256), 256, 0, s>>>(sorted_ids, npr, abs_cols, drop, out_degree);
    count_launch();
}

// candidate flat indices (sorted) -> per-row pointers over the candidate list
__global__ void k_cand_rowptr(const int64_t* __restrict__ cand, int nc, int64_t n_out, int64_t n_in,
                              int* __restrict__ cptr) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r > n_in) return;
    int lo = 0, hi = nc;
    while (lo < hi) { const int mid = (lo + hi) >> 1; if (cand[mid] / n_out < r) lo = mid + 1; else hi = mid; }
    cptr[r] = lo;
}
void launch_cand_rowptr(const int64_t* cand, int nc, int64_t n_out, int64_t n_in, int* cptr, cudaStream_t s) {
    k_cand_rowptr<<<(unsigned)((n_in + 256) / 256), 256, 0, s>>>(cand, nc, n_out, n_in, cptr);
    count_launch();
}

// Per row: kept old synapses merged with the row's candidates by column
// (candidates are non-existing positions, so no column appears twice).
// One warp per row.  pass 0 counts into cnt[r]; pass 1 writes at newptr[r]:
// a kept old synapse at (kept synapses before it) + (candidates of smaller
// column, binary search in the row's few candidates); a candidate at (its
// index among the row's candidates) + (kept synapses of smaller column:
// lower bound in the row's ascending columns minus the dropped ones before).
__global__ void k_topk_merge(LayerView L, const float* __restrict__ w, const float* __restrict__ imp,
                             const uint8_t* __restrict__ drop, const int64_t* __restrict__ cand,
                             const uint32_t* __restrict__ keys, const int* __restrict__ cptr, int pass,
                             int* __restrict__ cnt, const int* __restrict__ newptr, int* __restrict__ nidx,
                             float* __restrict__ nw, float* __restrict__ nimp, int* __restrict__ out_degree) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= L.n_in) return;
    const int f0 = L.rowptr[r], f1 = L.rowptr[r + 1];
    const int a0 = cptr[r], a1 = cptr[r + 1];
    if (pass == 0) {
        int kept = 0;
        for (int f = f0 + lane; f < f1; f += 32) kept += drop[f] ? 0 : 1;
        for (int o = 16; o > 0; o >>= 1) kept += __shfl_xor_sync(0xffffffffu, kept, o);
        if (lane == 0) cnt[r] = kept + (a1 - a0);
        return;
    }
    const int base = newptr[r];
    // kept old synapses
    int carry = 0;
    for (int c0 = f0; c0 < f1; c0 += 32) {
        const int f = c0 + lane;
        const bool valid = f < f1;
        const bool keep = valid && !drop[f];
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const int col = L.abs_cols[f];
            int lo = a0, hi = a1;   // candidates with column < col
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (cand[mid] % L.n_out < col) lo = mid + 1; else hi = mid;
            }
            const int o = base + carry + __popc(m & ((1u << lane) - 1u)) + (lo - a0);
            nidx[o] = col; nw[o] = w[f]; nimp[o] = imp[f];
        }
        carry += __popc(m);
    }
    // candidates
    for (int a = a0 + lane; a < a1; a += 32) {
        const int64_t cc = cand[a] % L.n_out;
        int lo = f0, hi = f1;        // first old synapse with column > cc
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (L.abs_cols[mid] < cc) lo = mid + 1; else hi = mid;
        }
        int dropped = 0;
        for (int f = f0; f < lo; ++f) dropped += drop[f] ? 1 : 0;
        const int o = base + (a - a0) + (lo - f0 - dropped);
        const float score = __uint_as_float(keys[cand[a]] - 1u);
        nidx[o] = (int)cc; nw[o] = 0.0f; nimp[o] = fp4_decode(fp4_encode(score));
        atomicAdd(out_degree + cc, 1);
    }
}
void launch_topk_merge(const LayerView& L, const float* w, const float* imp, const uint8_t* drop, const int64_t* cand,
                       const uint32_t* keys, const int* cptr, int pass, int* cnt, const int* newptr, int* nidx,
                       float* nw, float* nimp, int* out_degree, cudaStream_t s) {
    if (L.n_in == 0) return;
    k_topk_merge<<<(unsigned)((L.n_in + 7) / 8), 256, 0, s>>>(L, w, imp, drop, cand, keys, cptr, pass, cnt, newptr,
                                                             nidx, nw, nimp, out_degree);
    count_launch();
}

}  // namespace sili
