// Synaptogenesis on the device: delta_csr_synap_row_step
// (delta_csr_memory.hpp:1019-1258) with block4 promotion / demotion
// (block4_maybe_promote :593-702, block4_demote_tile :946-1003) over a sweep
// of rows, bit-exact with the reference's single-thread result.
//
// Work split.  A row's step reads and writes only its own scattered row, the
// tiles of its block-row (input rows 4br..4br+3) and, through promotion and
// demotion, the other scattered rows of that block-row.  Block-rows are
// therefore independent except through three global quantities: the
// block4 byte budgets (the reference throws / drops when a running total
// would pass them), out_degree's clamp at zero, and the first row that runs
// out of blank space (the reference stops the sweep there).  The kernel runs
// one warp per block-row, taking its rows in sweep order; the host
// checks afterwards whether any of the three could have depended on the
// order and, if so, restores the snapshot and re-runs exactly: truncated at
// the first failing row, or in one thread over the whole sweep in order.
//
// Sorting uses the same introsort as GCC's std::sort (the reference's
// orderings are std::sort, which is not stable), so ties among the 15
// stored importance values are broken exactly as the reference breaks them.
#include "common.cuh"
#include "kernels.cuh"

namespace sili {

namespace {

// ── std::sort (GCC libstdc++ introsort), iterative, on int index arrays ──
// Comparators: 0 = key ascending, 1 = key descending (float keys),
// 2 = unsigned key descending.
struct SortKeys {
    const float* f;
    const uint32_t* u;
    int mode;
    __device__ __forceinline__ bool lt(int a, int b) const {
        if (mode == 0) return f[a] < f[b];
        if (mode == 1) return f[a] > f[b];
        return u[a] > u[b];
    }
};

__device__ void ss_adjust_heap(int* f, int hole, int len, int val, const SortKeys& K) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (K.lt(f[child], f[child - 1])) child--;
        f[hole] = f[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        f[hole] = f[child - 1];
        hole = child - 1;
    }
    int parent = (hole - 1) / 2;
    while (hole > top && K.lt(f[parent], val)) {
        f[hole] = f[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    f[hole] = val;
}
__device__ void ss_heapsort(int* f, int n, const SortKeys& K) {
    if (n >= 2)
        for (int parent = (n - 2) / 2;; --parent) {
            ss_adjust_heap(f, parent, n, f[parent], K);
            if (parent == 0) break;
        }
    for (int last = n; last > 1;) {
        --last;
        const int v = f[last];
        f[last] = f[0];
        ss_adjust_heap(f, 0, last, v, K);
    }
}
__device__ __forceinline__ void ss_swap(int* a, int* b) { const int t = *a; *a = *b; *b = t; }
__device__ void ss_linear_insert(int* p, const SortKeys& K) {
    const int v = *p;
    int* q = p - 1;
    while (K.lt(v, *q)) { *p = *q; p = q; --q; }
    *p = v;
}
__device__ void ss_insertion(int* f, int* l, const SortKeys& K) {
    if (f == l) return;
    for (int* i = f + 1; i != l; ++i) {
        if (K.lt(*i, *f)) {
            const int v = *i;
            for (int* j = i; j != f; --j) *j = *(j - 1);
            *f = v;
        } else {
            ss_linear_insert(i, K);
        }
    }
}
// __unguarded_partition_pivot: median of three moved to f, Hoare partition
// of [f + 1, l) around it; returns the cut
__device__ int* ss_partition(int* f, int* l, const SortKeys& K) {
    int *x = f + 1, *y = f + (l - f) / 2, *z = l - 1;
    if (K.lt(*x, *y)) {
        if (K.lt(*y, *z)) ss_swap(f, y);
        else if (K.lt(*x, *z)) ss_swap(f, z);
        else ss_swap(f, x);
    } else if (K.lt(*x, *z)) ss_swap(f, x);
    else if (K.lt(*y, *z)) ss_swap(f, z);
    else ss_swap(f, y);
    int *lo = f + 1, *hi = l;
    for (;;) {
        while (K.lt(*lo, *f)) ++lo;
        --hi;
        while (K.lt(*f, *hi)) --hi;
        if (!(lo < hi)) break;
        ss_swap(lo, hi);
        ++lo;
    }
    return lo;
}
// std::sort's permutation (GCC's introsort: ranges of more than 16 are
// partitioned, depth-limited to 2 log2 n with heapsort beyond, then one
// insertion pass), produced front to back on demand: extend(m) makes
// positions [0, m) final, extend(n) is the whole std::sort.  Ranges are kept
// on an explicit stack: partitions of disjoint ranges do not interact, so
// they may be visited in any order.  Partial extension is valid for keys in
// a strict weak order (no NaN): after a partition every element right of the cut is not less than every
// element left of it, and the final insertion passes move an element only
// leftwards past strictly greater ones, so no element ever crosses a cut.
// Hence the prefix [0, P) -- P the start of the leftmost range not yet
// partitioned -- is final once every range starting below P is partitioned
// and the insertion passes of std::sort have run over [0, P); ranges starting
// at or beyond the requested end are left for later calls.  Each range is
// partitioned from the same contents as in std::sort (nothing else touches
// it first), so the permutation is std::sort's.
struct LazySort {
    struct Frame { int* f; int* l; int depth; };
    int* a;
    int n;
    int done;   // [0, done) final
    int sp;
    Frame st[64];
    __device__ void init(int* arr, int len) {
        a = arr; n = len; done = 0; sp = 0;
        if (n <= 1) { done = n; return; }
        int lg = 0;
        while ((1 << (lg + 1)) <= n) ++lg;
        st[sp++] = {a, a + n, 2 * lg};
    }
    __device__ void extend(int m, const SortKeys& K) {
        if (m <= done) return;
        m = m < 16 ? 16 : m;
        if (m > n) m = n;
        // partition every pending range that starts below m
        for (;;) {
            int pick = -1;
            for (int i = 0; i < sp; ++i)
                if (st[i].f - a < m) { pick = i; break; }
            if (pick < 0) break;
            const Frame fr = st[pick];
            st[pick] = st[--sp];
            int* f = fr.f;
            int* l = fr.l;
            int depth = fr.depth;
            while (l - f > 16) {
                if (depth == 0) { ss_heapsort(f, (int)(l - f), K); break; }
                --depth;
                int* lo = ss_partition(f, l, K);
                if (sp < 64) st[sp++] = {lo, l, depth};
                l = lo;
            }
        }
        int P = n;
        for (int i = 0; i < sp; ++i)
            if ((int)(st[i].f - a) < P) P = (int)(st[i].f - a);
        // std::sort's insertion passes over [done, P)
        int i0 = done;
        if (done == 0) {
            ss_insertion(a, a + (n > 16 ? 16 : n), K);
            i0 = 16;
        }
        for (int i = i0; i < P; ++i) ss_linear_insert(a + i, K);
        done = P > done ? P : done;
    }
};

__device__ __forceinline__ int uleb_len(uint32_t v) { int n = 0; do { v >>= 7; ++n; } while (v); return n; }
__device__ __forceinline__ int uleb_put(uint32_t v, uint8_t* p) {
    int n = 0;
    do { uint8_t b = v & 0x7Fu; v >>= 7; if (v) b |= 0x80u; p[n++] = b; } while (v);
    return n;
}
__device__ __forceinline__ uint32_t uleb_get(const uint8_t* buf, int64_t& pos) {
    uint32_t v = 0; int sh = 0;
    for (;;) { const uint8_t b = buf[pos++]; v |= (uint32_t)(b & 0x7Fu) << sh; if (!(b & 0x80u)) break; sh += 7; }
    return v;
}
__device__ __forceinline__ uint32_t tb(const uint4& t, int s) {
    const uint32_t w = s < 8 ? (s < 4 ? t.x : t.y) : (s < 12 ? t.z : t.w);
    return (w >> ((s & 3) * 8)) & 0xFFu;
}
__device__ __forceinline__ void set_tb(uint4& t, int s, uint32_t b) {
    const uint32_t sh = (uint32_t)(s & 3) * 8u, m = ~(0xFFu << sh), v = (b & 0xFFu) << sh;
    if (s < 4) t.x = (t.x & m) | v;
    else if (s < 8) t.y = (t.y & m) | v;
    else if (s < 12) t.z = (t.z & m) | v;
    else t.w = (t.w & m) | v;
}
__device__ __forceinline__ int live_of(const uint4& t) {
    int n = 0;
    for (int s = 0; s < 16; ++s) n += tb(t, s) != 0;
    return n;
}
__device__ __forceinline__ int64_t tlen(const uint4& t, uint8_t sp) {
    const int n = live_of(t);
    return sp ? 1 + (n + 1) / 2 + n : 16;
}

constexpr int kOK = 0, kENOMEM = 2, kEHEADROOM = 3;

// The block-row's context: the layer state plus its scratch.  All 32 lanes
// of the block-row's warp run the row step together: the scalar logic on
// every lane from the same data (so control flow stays uniform), the scans
// over a row's entries (ULEB128 decode, rewrite, searches, filters) spread
// over the lanes, and every write of layer state or scratch that the lanes
// do not split among themselves -- the block4 store, the counters, the
// sorted orders -- by lane 0, followed by __syncwarp before the lanes read
// it again.
struct Ctx {
    SynView V;
    int64_t R, C, BR;
    // scratch (per block-row)
    uint32_t* rc;   // row-op columns [M]
    uint8_t* rv;    // row-op values  [M]
    // block4 running totals (sequential mode only; lane 0's copy is the one used)
    int64_t tot_idx, tot_tile;
    bool seq;
    int lane;
};
constexpr unsigned kFull = 0xffffffffu;

// ── scattered rows ──
__device__ int row_nnz(const Ctx& c, int64_t r) { return (int)(c.V.ee[r] - c.V.es[r]); }
// the row's absolute columns into cols (all lanes).  Each step reads the next
// 32 bytes; the bytes without a continuation bit end the entries; a lane
// ending an entry gathers its 7-bit groups (at most 5 count: uleb_get's
// shifts past 31 bits drop the rest) and a warp scan of the deltas gives the
// columns.  An entry longer than 32 bytes (never written by this library)
// is decoded by lane 0 alone.
__device__ int decode_row(const Ctx& c, int64_t r, uint32_t* cols) {
    const int n = row_nnz(c, r);
    const int lane = c.lane;
    int64_t pos = c.V.bs[r];
    const int64_t cap_end = c.V.bs[r + 1];
    uint32_t carry = 0;
    int k = 0;
    while (k < n) {
        const uint32_t b = pos + lane < cap_end ? (uint32_t)c.V.idx[pos + lane] : 0u;
        const unsigned T = __ballot_sync(kFull, (b & 0x80u) == 0u);
        const int m = min(__popc(T), n - k);
        if (m == 0) {
            if (lane == 0) {
                int64_t p = pos;
                uint32_t col = carry;
                for (int q = k; q < n; ++q) { col += uleb_get(c.V.idx, p); cols[q] = col; }
            }
            break;
        }
        const unsigned below = T & ((1u << lane) - 1u);
        const int rank = __popc(below);
        const bool take = ((T >> lane) & 1u) && rank < m;
        const int S = below ? 32 - __clz(below) : 0;   // this lane's entry starts after the previous end
        uint32_t v = 0;
#pragma unroll
        for (int t = 0; t < 5; ++t) {
            const uint32_t bj = __shfl_sync(kFull, b, min(S + t, 31));
            if (S + t <= lane) v |= (bj & 0x7Fu) << (7 * t);
        }
        uint32_t d = take ? v : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(kFull, d, o);
            if (lane >= o) d += t;
        }
        if (take) cols[k + rank] = carry + d;
        const int last = __ffs(__ballot_sync(kFull, take && rank == m - 1)) - 1;
        carry += __shfl_sync(kFull, d, last);
        pos += last + 1;
        k += m;
    }
    __syncwarp();
    return n;
}
// first index in [0, n) whose column satisfies the test (eq: == col, else
// >= col), or n; all lanes
__device__ int find_col(const Ctx& c, const uint32_t* cols, int n, uint32_t col, bool eq) {
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + c.lane;
        const bool hit = k < n && (eq ? cols[k] == col : cols[k] >= col);
        const unsigned m = __ballot_sync(kFull, hit);
        if (m) return k0 + __ffs(m) - 1;
    }
    return n;
}
// The new row of n entries, entry k being (as is) k, (drop) k < i ? k : k + 1,
// or (insert) k < i ? k : k == i ? (col, val) : k - 1 of the scratch row
// rc / rv.
struct RowMap {
    int mode;   // 0 as is, 1 drop entry i, 2 insert (col, val) at i
    int i;
    uint32_t col;
    uint8_t val;
    __device__ __forceinline__ void get(const Ctx& c, int k, uint32_t& col_k, uint8_t& v_k) const {
        if (mode == 1) {
            const int s = k < i ? k : k + 1;
            col_k = c.rc[s]; v_k = c.rv[s];
        } else if (mode == 2 && k >= i) {
            if (k == i) { col_k = col; v_k = val; }
            else { col_k = c.rc[k - 1]; v_k = c.rv[k - 1]; }
        } else {
            col_k = c.rc[k]; v_k = c.rv[k];
        }
    }
};
// rewrite the live part of row r (the state delta_csr_row_remove_col /
// _insert_col leave behind, delta_csr_memory.hpp:429-585), all lanes: each
// lane encodes its entries at offsets from a warp scan of the encoded lengths
__device__ int row_write(Ctx& c, int64_t r, const RowMap& M, int n) {
    const int lane = c.lane;
    long long nb = 0;
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        if (k < n) {
            uint32_t ck, cp = 0;
            uint8_t v;
            M.get(c, k, ck, v);
            if (k > 0) M.get(c, k - 1, cp, v);
            nb += uleb_len(ck - cp);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nb += __shfl_xor_sync(kFull, nb, o);
    if (nb > c.V.bs[r + 1] - c.V.bs[r]) return kEHEADROOM;
    if (n > c.V.es[r + 1] - c.V.es[r]) return kEHEADROOM;
    int64_t bp = c.V.bs[r];
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        uint32_t ck = 0, cp = 0;
        uint8_t v = 0, vp;
        int len = 0;
        if (k < n) {
            M.get(c, k, ck, v);
            if (k > 0) M.get(c, k - 1, cp, vp);
            len = uleb_len(ck - cp);
        }
        int incl = len;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += t;
        }
        if (k < n) {
            uleb_put(ck - cp, c.V.idx + bp + (incl - len));
            c.V.val[c.V.es[r] + k] = v;
        }
        bp += __shfl_sync(kFull, incl, 31);
    }
    if (lane == 0) {
        c.V.be[r] = c.V.bs[r] + nb;
        atomicAdd(c.V.nnz_delta, (unsigned long long)(long long)(n - row_nnz(c, r)));
        c.V.ee[r] = c.V.es[r] + n;
    }
    __syncwarp();
    return kOK;
}
// the row's value bytes into rv (all lanes)
__device__ void load_vals(Ctx& c, int64_t r, int n) {
    for (int k = c.lane; k < n; k += 32) c.rv[k] = c.V.val[c.V.es[r] + k];
    __syncwarp();
}
__device__ bool insert_fits(const Ctx& c, int64_t r, const uint32_t* cols, int n, int i, uint32_t col) {
    const uint32_t prev = i > 0 ? cols[i - 1] : 0u;
    int64_t delta = uleb_len(col - prev);
    if (i < n) delta += uleb_len(cols[i] - col) - uleb_len(cols[i] - prev);
    const int64_t used = c.V.be[r] - c.V.bs[r];
    if (delta > 0 && delta > (c.V.bs[r + 1] - c.V.bs[r]) - used) return false;
    if (n >= c.V.es[r + 1] - c.V.es[r]) return false;
    return true;
}
__device__ bool sc_remove_col(Ctx& c, int64_t r, uint32_t col) {
    const int n = decode_row(c, r, c.rc);
    const int i = find_col(c, c.rc, n, col, true);
    if (i == n) return false;
    load_vals(c, r, n);
    row_write(c, r, RowMap{1, i, 0u, 0}, n - 1);
    return true;
}
// delta_csr_row_insert_col with ValueAccessor::set (deterministic codes)
__device__ bool sc_insert_col(Ctx& c, int64_t r, uint32_t col, float w, float imp) {
    const int n = decode_row(c, r, c.rc);
    const int i = find_col(c, c.rc, n, col, false);
    if (i < n && c.rc[i] == col) return false;
    if (!insert_fits(c, r, c.rc, n, i, col)) return false;
    load_vals(c, r, n);
    row_write(c, r, RowMap{2, i, col, (uint8_t)((fp4_encode(w) << 4) | fp4_encode(imp))}, n + 1);
    return true;
}

// ── block4 store (reference accounting, block4.hpp) ──
__device__ int b4_find(const Ctx& c, int64_t br, int bc) {
    const int nt = c.V.nt[br];
    const int64_t base = c.V.b4_es[br];
    for (int e = 0; e < nt; ++e) {
        const int v = c.V.b4_bc[base + e];
        if (v == bc) return e;
        if (v > bc) break;
    }
    return -1;
}
__device__ int64_t b4_tile_used(const Ctx& c, int64_t br) {
    int64_t u = 0;
    const int64_t base = c.V.b4_es[br];
    for (int e = 0; e < c.V.nt[br]; ++e) u += tlen(c.V.b4_tile[base + e], c.V.b4_sparse[base + e]);
    return u;
}
__device__ int64_t b4_idx_used(const Ctx& c, int64_t br) {
    int64_t u = 0;
    uint32_t prev = 0;
    const int64_t base = c.V.b4_es[br];
    for (int e = 0; e < c.V.nt[br]; ++e) {
        const uint32_t v = (uint32_t)c.V.b4_bc[base + e];
        u += uleb_len(v - prev);
        prev = v;
    }
    return u;
}
__device__ int64_t& A_idx(Ctx& c, int64_t br) { return c.V.alloc[br]; }
__device__ int64_t& A_tile(Ctx& c, int64_t br) { return c.V.alloc[c.BR + br]; }
__device__ int64_t& A_elem(Ctx& c, int64_t br) { return c.V.alloc[2 * c.BR + br]; }

// block4_row_shift (block4.hpp:497-609) / block4_grow_last_row (:611-646)
__device__ int b4_ensure_headroom(Ctx& c, int64_t br) {
    int64_t ti = A_idx(c, br) + 5, tt = A_tile(c, br) + 1, te = A_elem(c, br) + 1;
    if (br + 1 < c.BR) {
        ti = max(ti, b4_idx_used(c, br));
        tt = max(tt, b4_tile_used(c, br));
        te = max(te, (int64_t)c.V.nt[br]);
        if (A_idx(c, br) != ti) {
            if (c.seq && ti > A_idx(c, br) && c.tot_idx + (ti - A_idx(c, br)) > c.V.max_idx) return kENOMEM;
            c.tot_idx += ti - A_idx(c, br);
            atomicAdd(c.V.grow, (unsigned long long)(ti - A_idx(c, br)));
            A_idx(c, br) = ti;
        }
        if (A_tile(c, br) != tt) {
            if (c.seq && tt > A_tile(c, br) && c.tot_tile + (tt - A_tile(c, br)) > c.V.max_tile) return kENOMEM;
            c.tot_tile += tt - A_tile(c, br);
            atomicAdd(c.V.grow + 1, (unsigned long long)(tt - A_tile(c, br)));
            A_tile(c, br) = tt;
        }
        A_elem(c, br) = te;
    } else {
        if (ti > A_idx(c, br)) {
            if (c.seq && c.tot_idx + (ti - A_idx(c, br)) > c.V.max_idx) return kENOMEM;
            c.tot_idx += ti - A_idx(c, br);
            atomicAdd(c.V.grow, (unsigned long long)(ti - A_idx(c, br)));
            A_idx(c, br) = ti;
        }
        if (tt > A_tile(c, br)) {
            if (c.seq && c.tot_tile + (tt - A_tile(c, br)) > c.V.max_tile) return kENOMEM;
            c.tot_tile += tt - A_tile(c, br);
            atomicAdd(c.V.grow + 1, (unsigned long long)(tt - A_tile(c, br)));
            A_tile(c, br) = tt;
        }
        if (te > A_elem(c, br)) A_elem(c, br) = te;
    }
    return kOK;
}
// block4_row_insert_tile (block4.hpp:670-771): an empty sparse tile
__device__ bool b4_insert_tile(Ctx& c, int64_t br, int bc) {
    const int nt = c.V.nt[br];
    const int64_t base = c.V.b4_es[br];
    int p = 0;
    while (p < nt && c.V.b4_bc[base + p] < bc) ++p;
    if (p < nt && c.V.b4_bc[base + p] == bc) return false;
    const uint32_t prev = p > 0 ? (uint32_t)c.V.b4_bc[base + p - 1] : 0u;
    int64_t delta = uleb_len((uint32_t)bc - prev);
    if (p < nt) {
        const uint32_t nx = (uint32_t)c.V.b4_bc[base + p];
        delta += uleb_len(nx - (uint32_t)bc) - uleb_len(nx - prev);
    }
    if (delta > 0 && delta > A_idx(c, br) - b4_idx_used(c, br)) return false;
    if (nt >= A_elem(c, br)) return false;
    if (1 > A_tile(c, br) - b4_tile_used(c, br)) return false;
    if (base + nt + 1 > c.V.b4_es[br + 1]) { atomicOr(c.V.flags, 4); return false; }   // device capacity
    for (int e = nt; e > p; --e) {
        c.V.b4_bc[base + e] = c.V.b4_bc[base + e - 1];
        c.V.b4_tile[base + e] = c.V.b4_tile[base + e - 1];
        c.V.b4_sparse[base + e] = c.V.b4_sparse[base + e - 1];
    }
    c.V.b4_bc[base + p] = bc;
    c.V.b4_tile[base + p] = make_uint4(0, 0, 0, 0);
    c.V.b4_sparse[base + p] = 1;
    c.V.nt[br] = nt + 1;
    return true;
}
// commit_dirty_sparse_tile (block4.hpp:1223-1268)
__device__ void b4_commit(Ctx& c, int64_t br, int e, const uint4& t) {
    const int64_t ti = c.V.b4_es[br] + e;
    const int n = live_of(t);
    const bool sp = (uint32_t)n <= c.V.switch_point;
    const int64_t nl = sp ? 1 + (n + 1) / 2 + n : 16;
    const int64_t cl = tlen(c.V.b4_tile[ti], c.V.b4_sparse[ti]);
    if (nl > cl) {
        const int64_t head = A_tile(c, br) - b4_tile_used(c, br);
        if (nl - cl > head) {
            const int64_t sf = nl - cl - head;
            if (c.seq && c.tot_tile + sf > c.V.max_tile) { atomicAdd(c.V.counters, 1ull); return; }
            c.tot_tile += sf;
            atomicAdd(c.V.grow + 1, (unsigned long long)sf);
            A_tile(c, br) += sf;
        }
    }
    c.V.b4_tile[ti] = t;
    c.V.b4_sparse[ti] = sp ? 1 : 0;
}
__device__ void b4_write(Ctx& c, int64_t br, int e, const uint4& t) {
    const int64_t ti = c.V.b4_es[br] + e;
    if (c.V.b4_sparse[ti]) b4_commit(c, br, e, t);
    else c.V.b4_tile[ti] = t;
}
__device__ void b4_maybe_compress(Ctx& c, int64_t br, int e) {
    const int64_t ti = c.V.b4_es[br] + e;
    if (c.V.b4_sparse[ti] || (uint32_t)live_of(c.V.b4_tile[ti]) > c.V.switch_point) return;
    c.V.b4_sparse[ti] = 1;
}
__device__ void b4_erase(Ctx& c, int64_t br, int bc) {
    const int e = b4_find(c, br, bc);
    if (e < 0) return;
    const int nt = c.V.nt[br];
    const int64_t base = c.V.b4_es[br];
    for (int k = e; k + 1 < nt; ++k) {
        c.V.b4_bc[base + k] = c.V.b4_bc[base + k + 1];
        c.V.b4_tile[base + k] = c.V.b4_tile[base + k + 1];
        c.V.b4_sparse[base + k] = c.V.b4_sparse[base + k + 1];
    }
    c.V.nt[br] = nt - 1;
}
// block4_demote_tile (delta_csr_memory.hpp:946-1003)
__device__ int b4_demote(Ctx& c, int64_t br, int bc) {
    const int e = b4_find(c, br, bc);
    if (e < 0) return kOK;
    const uint4 t = c.V.b4_tile[c.V.b4_es[br] + e];
    for (int li = 0; li < 4; ++li) {
        const int64_t row = br * 4 + li;
        if (row >= c.R) continue;
        for (int lj = 0; lj < 4; ++lj) {
            const uint32_t byte = tb(t, lj * 4 + li);
            if (byte == 0) continue;
            const int64_t col = (int64_t)bc * 4 + lj;
            if (col >= c.C) continue;
            if (!sc_insert_col(c, row, (uint32_t)col, fp4_decode(byte & 0xFu), fp4_decode(byte >> 4))) return kEHEADROOM;
        }
    }
    if (c.lane == 0) b4_erase(c, br, bc);
    __syncwarp();
    return kOK;
}
// block4_maybe_promote (delta_csr_memory.hpp:593-702)
__device__ int b4_maybe_promote(Ctx& c, int64_t row, uint32_t col) {
    const int64_t br = row / 4;
    const int bc = (int)(col / 4), li = (int)(row % 4), lj = (int)(col % 4);
    const int lane = c.lane;
    int e = b4_find(c, br, bc);
    if (e >= 0) {
        const int n = decode_row(c, row, c.rc);
        const int k = find_col(c, c.rc, n, col, true);
        if (k == n) return kOK;
        if (lane == 0) {
            const uint8_t v = c.V.val[c.V.es[row] + k];
            uint4 t = c.V.b4_tile[c.V.b4_es[br] + e];
            set_tb(t, lj * 4 + li, fp4_encode(fp4_decode(v >> 4)) | (fp4_encode(fp4_decode(v & 0xFu)) << 4));
            b4_write(c, br, e, t);
            b4_maybe_compress(c, br, e);
        }
        __syncwarp();
        sc_remove_col(c, row, col);
        return kOK;
    }
    // the block's scattered entries, rows ascending, each row's entries in
    // stored order, at most 16 (every lane keeps the list)
    const int64_t row_lo = br * 4, row_hi = min(row_lo + 4, c.R);
    const int64_t col_lo = (int64_t)bc * 4, col_hi = min(col_lo + 4, c.C);
    int fr[16], fcol[16];
    uint8_t fv[16];
    int nf = 0;
    for (int64_t r = row_lo; r < row_hi; ++r) {
        const int n = decode_row(c, r, c.rc);
        for (int k0 = 0; k0 < n && nf < 16; k0 += 32) {
            const int k = k0 + lane;
            uint32_t ck = 0;
            uint8_t vk = 0;
            bool hit = false;
            if (k < n) {
                ck = c.rc[k];
                hit = (int64_t)ck >= col_lo && (int64_t)ck < col_hi;
                if (hit) vk = c.V.val[c.V.es[r] + k];
            }
            unsigned m = __ballot_sync(kFull, hit);
            while (m && nf < 16) {
                const int src = __ffs(m) - 1;
                m &= m - 1u;
                fr[nf] = (int)r;
                fcol[nf] = (int)__shfl_sync(kFull, ck, src);
                fv[nf] = (uint8_t)__shfl_sync(kFull, (uint32_t)vk, src);
                ++nf;
            }
        }
    }
    if (nf < 2) return kOK;
    // Block4Store::get_or_create (block4.hpp:1168-1184), by lane 0
    int rc = kOK;
    bool stop = false;
    if (lane == 0) {
        if (!b4_insert_tile(c, br, bc)) {
            if (*c.V.flags & 4) {
                stop = true;
            } else {
                rc = b4_ensure_headroom(c, br);
                if (rc) {
                    stop = true;
                } else {
                    b4_insert_tile(c, br, bc);
                    if (*c.V.flags & 4) stop = true;
                }
            }
        }
        if (!stop) e = b4_find(c, br, bc);
        if (!stop && e >= 0) {
            uint4 t = c.V.b4_tile[c.V.b4_es[br] + e];
            for (int f = 0; f < nf; ++f)
                set_tb(t, (fcol[f] - (int)col_lo) * 4 + (fr[f] - (int)row_lo),
                       fp4_encode(fp4_decode(fv[f] >> 4)) | (fp4_encode(fp4_decode(fv[f] & 0xFu)) << 4));
            b4_write(c, br, e, t);
            b4_maybe_compress(c, br, e);
        }
    }
    rc = __shfl_sync(kFull, rc, 0);
    stop = __shfl_sync(kFull, stop ? 1 : 0, 0) != 0;
    __syncwarp();
    if (stop) return rc;
    for (int f = 0; f < nf; ++f) sc_remove_col(c, fr[f], (uint32_t)fcol[f]);
    return kOK;
}

// out_degree decrement with the reference's clamp (if > 0), by lane 0
__device__ void od_dec(Ctx& c, uint32_t col) {
    if (c.lane == 0) {
        atomicAdd(c.V.od_decs + col, 1);
        int cur = c.V.out_degree[col];
        while (cur > 0) {
            const int prev = atomicCAS(c.V.out_degree + col, cur, cur - 1);
            if (prev == cur) break;
            cur = prev;
        }
    }
    __syncwarp();
}

// delta_csr_synap_row_step for one row (oracle: o_synap_row_step), all lanes
__device__ int synap_row(Ctx& c, int64_t r, const SynParams& P, uint32_t* ecol, float* eimp, uint8_t* eb4, int* by,
                         uint32_t* pcs, float* pss, int* pidx, uint32_t* rmc, uint8_t* rmb, int* rperm, uint32_t* addc,
                         float* adds, bool* did) {
    *did = false;
    const int lane = c.lane;
    const int n_sc = row_nnz(c, r);
    const bool has_probes = c.V.n_probes > 0;
    const int64_t br = r / 4;
    const int li = (int)(r % 4);
    const int nt = c.V.nt[br];
    // the existing synapses: the scattered row, then the row's tile slots in
    // tile order
    decode_row(c, r, ecol);
    for (int k = lane; k < n_sc; k += 32) { eimp[k] = fp4_decode(c.V.val[c.V.es[r] + k] & 0xFu); eb4[k] = 0; }
    int n_exist = n_sc;
    const int64_t base = c.V.b4_es[br];
    for (int e0 = 0; e0 < nt; e0 += 32) {
        const int e = e0 + lane;
        uint4 t = make_uint4(0u, 0u, 0u, 0u);
        int64_t c0 = 0;
        int cnt = 0;
        if (e < nt) {
            t = c.V.b4_tile[base + e];
            c0 = (int64_t)c.V.b4_bc[base + e] * 4;
            for (int lj = 0; lj < 4; ++lj) cnt += (tb(t, lj * 4 + li) != 0 && c0 + lj < c.C) ? 1 : 0;
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
        }
        int q = n_exist + incl - cnt;
        for (int lj = 0; lj < 4 && e < nt; ++lj) {
            const uint32_t byte = tb(t, lj * 4 + li);
            if (byte == 0 || c0 + lj >= c.C) continue;
            ecol[q] = (uint32_t)(c0 + lj);
            eimp[q] = fp4_decode(byte >> 4);
            eb4[q] = 1;
            ++q;
        }
        n_exist += __shfl_sync(kFull, incl, 31);
    }
    __syncwarp();
    if (n_exist == 0 && !has_probes) return kOK;
    // probes of this row, COO order
    const int q0 = c.V.pr_ptr[r];
    const int np = c.V.pr_ptr[r + 1] - q0;
    for (int q = lane; q < np; q += 32) {
        const int p = c.V.pr_idx[q0 + q];
        pcs[q] = (uint32_t)c.V.pcol[p];
        pss[q] = c.V.pval[p];
    }
    for (int i = lane; i < n_exist; i += 32) by[i] = i;
    for (int i = lane; i < np; i += 32) pidx[i] = i;
    bool key_nan = false, score_nan = false;
    for (int i = lane; i < n_exist; i += 32) key_nan = key_nan || isnan(eimp[i]);
    for (int i = lane; i < np; i += 32) score_nan = score_nan || isnan(pss[i]);
    key_nan = __any_sync(kFull, key_nan);
    score_nan = __any_sync(kFull, score_nan);
    __syncwarp();
    // removals by stored importance ascending (:1147-1167), lane 0.  Without
    // a NaN key the removals are a prefix of the sorted order (the clamped
    // importance only grows along it and keep only shrinks, so the first
    // position not taken ends the scan), and only that prefix is sorted.
    LazySort ls;   // lane 0's; one frame stack for the three sorts (extend(n) is std::sort)
    int nrm = 0;
    if (lane == 0) {
        const SortKeys K0{eimp, nullptr, 0};
        ls.init(by, n_exist);
        if (key_nan) ls.extend(n_exist, K0);
        for (int a = 0; a < n_exist && nrm < P.max_prune; ++a) {
            if (!key_nan) ls.extend(a + 1, K0);
            const int k = by[a];
            const int keep = n_exist - nrm;
            const float fl = (eimp[k] < P.eps) ? P.eps : eimp[k];
            if (fl < P.cutoff || keep > P.max_rw) {
                rmc[nrm] = ecol[k]; rmb[nrm] = eb4[k]; ++nrm;
            } else if (!key_nan) {
                break;
            }
        }
        for (int i = 0; i < nrm; ++i) rperm[i] = i;
        ls.init(rperm, nrm);
        ls.extend(nrm, SortKeys{nullptr, rmc, 2});
        // adds by score descending (:1171-1201), produced as far as the scan reads it
        ls.init(pidx, np);
        if (score_nan) ls.extend(np, SortKeys{pss, nullptr, 1});
    }
    nrm = __shfl_sync(kFull, nrm, 0);
    __syncwarp();
    const unsigned long long slots = (unsigned long long)((long long)P.max_rw - (long long)(n_exist - nrm));
    int nadd = 0;
    for (int a = 0; a < np; ++a) {
        if ((unsigned long long)nadd >= slots) break;
        int cand = 0;
        if (lane == 0) {
            if (!score_nan) ls.extend(a + 1, SortKeys{pss, nullptr, 1});
            cand = pidx[a];
        }
        cand = __shfl_sync(kFull, cand, 0);
        const uint32_t col = pcs[cand];
        if (find_col(c, ecol, n_exist, col, true) == n_exist) {
            if (lane == 0) { addc[nadd] = col; adds[nadd] = pss[cand]; }
            ++nadd;
        }
    }
    __syncwarp();
    // removals, highest column first (:1203-1233)
    for (int q = 0; q < nrm; ++q) {
        const uint32_t col = rmc[rperm[q]];
        if (rmb[rperm[q]]) {
            const int bc = (int)(col / 4), lj = (int)(col % 4);
            bool demote = false;
            if (lane == 0) {
                const int e = b4_find(c, br, bc);
                if (e >= 0) {
                    uint4 t = c.V.b4_tile[base + e];
                    if (tb(t, lj * 4 + li) != 0) {
                        set_tb(t, lj * 4 + li, 0u);
                        demote = live_of(t) < 2;
                        b4_write(c, br, e, t);
                    }
                }
            }
            demote = __shfl_sync(kFull, demote ? 1 : 0, 0) != 0;
            __syncwarp();
            if (demote) {
                const int rc = b4_demote(c, br, bc);
                if (rc) return rc;
            }
        } else {
            sc_remove_col(c, r, col);
        }
        od_dec(c, col);
    }
    // inserts in score order, each followed by the block4 promotion (:1235-1255)
    for (int a = 0; a < nadd; ++a) {
        if (!sc_insert_col(c, r, addc[a], 0.0f, adds[a])) return kEHEADROOM;
        if (lane == 0) atomicAdd(c.V.out_degree + addc[a], 1);
        __syncwarp();
        const int rc = b4_maybe_promote(c, r, addc[a]);
        if (rc) return rc;
        if (*c.V.flags & 4) return kOK;
    }
    *did = true;
    return kOK;
}

}  // namespace

// One warp per block-row (or one warp for the whole sweep when sequential).
// Sweep position i covers row (row0 + i) % R; rows at positions > limit are
// left alone.
__global__ void k_synap(SynView V, SynParams P, int sequential) {
    const int64_t R = V.n_in, BR = (R + 3) / 4;
    const int lane = threadIdx.x & 31;
    const int64_t tid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (sequential ? tid != 0 : tid >= BR) return;
    Ctx c;
    c.V = V;
    c.R = R; c.C = V.n_out; c.BR = BR;
    c.seq = sequential != 0;
    c.tot_idx = V.tot_idx0; c.tot_tile = V.tot_tile0;
    c.lane = lane;
    const int64_t M = V.scratch_m, PM = V.scratch_p;
    uint8_t* sb = V.scratch + (size_t)(sequential ? 0 : tid) * (size_t)V.scratch_stride;
    // carve the block-row's scratch: row ops, exist lists, probe lists
    auto take = [&](size_t bytes) { uint8_t* p = sb; sb += (bytes + 15) & ~(size_t)15; return p; };
    c.rc = (uint32_t*)take((size_t)M * 4);
    c.rv = take((size_t)M);
    uint32_t* ecol = (uint32_t*)take((size_t)M * 4);
    float* eimp = (float*)take((size_t)M * 4);
    uint8_t* eb4 = take((size_t)M);
    int* by = (int*)take((size_t)M * 4);
    uint32_t* rmc = (uint32_t*)take((size_t)M * 4);
    uint8_t* rmb = take((size_t)M);
    int* rperm = (int*)take((size_t)M * 4);
    uint32_t* pcs = (uint32_t*)take((size_t)PM * 4);
    float* pss = (float*)take((size_t)PM * 4);
    int* pidx = (int*)take((size_t)PM * 4);
    uint32_t* addc = (uint32_t*)take((size_t)PM * 4);
    float* adds = (float*)take((size_t)PM * 4);
    if (R == 0) return;
    const int64_t row0 = ((P.row0 % R) + R) % R;
    if (sequential) {
        for (int64_t i = 0; i < P.nrows && i <= P.limit; ++i) {
            const int64_t r = (row0 + i) % R;
            bool did = false;
            const int rc = synap_row(c, r, P, ecol, eimp, eb4, by, pcs, pss, pidx, rmc, rmb, rperm, addc, adds, &did);
            if (lane == 0 && V.did) V.did[i] = did ? 1 : 0;
            __syncwarp();
            if (rc || (*V.flags & 4)) {
                if (rc && lane == 0) { atomicMin(V.err_i, (long long)i); atomicMax(V.err_code, rc); }
                return;
            }
        }
        return;
    }
    // rows of block-row tid in sweep order: positions i = (4*tid + li - row0) mod R + k*R
    const int64_t br = tid;
    int64_t next[4];
    for (int li = 0; li < 4; ++li) {
        const int64_t r = br * 4 + li;
        next[li] = r < R ? ((r - row0) % R + R) % R : INT64_MAX;
    }
    for (;;) {
        int best = -1;
        for (int li = 0; li < 4; ++li)
            if (next[li] < P.nrows && next[li] <= P.limit && (best < 0 || next[li] < next[best])) best = li;
        if (best < 0) break;
        const int64_t i = next[best];
        next[best] += R;
        bool did = false;
        const int rc = synap_row(c, br * 4 + best, P, ecol, eimp, eb4, by, pcs, pss, pidx, rmc, rmb, rperm, addc,
                                 adds, &did);
        if (lane == 0 && V.did) V.did[i] = did ? 1 : 0;
        __syncwarp();
        if (rc) {
            if (lane == 0) { atomicMin(V.err_i, (long long)i); atomicMax(V.err_code, rc); }
            return;
        }
        if (*V.flags & 4) return;
    }
}

void launch_synap(const SynView& V, const SynParams& P, bool sequential, cudaStream_t s) {
    const int64_t BR = (V.n_in + 3) / 4;
    if (sequential) {
        k_synap<<<1, 32, 0, s>>>(V, P, 1);
    } else {
        k_synap<<<(unsigned)((BR + 3) / 4), 128, 0, s>>>(V, P, 0);
    }
    count_launch();
}

// ptr[k] = first position of key k in sorted_keys (k = 0..nkeys)
__global__ void k_lower_bound(const int* __restrict__ keys, int n, int64_t nkeys, int* __restrict__ ptr) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k > nkeys) return;
    int lo = 0, hi = n;
    while (lo < hi) { const int mid = (lo + hi) >> 1; if (keys[mid] < (int)k) lo = mid + 1; else hi = mid; }
    ptr[k] = lo;
}
void launch_lower_bound(const int* sorted_keys, int n, int64_t nkeys, int* ptr, cudaStream_t s) {
    k_lower_bound<<<(unsigned)((nkeys + 256) / 256), 256, 0, s>>>(sorted_keys, n, nkeys, ptr);
    count_launch();
}

// out_degree clamp check: a column whose decrements exceed its starting count
// could have been clamped in an order-dependent way
__global__ void k_od_check(const int* __restrict__ od0, const int* __restrict__ decs, int64_t n, int* __restrict__ flags) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && decs[i] > od0[i]) atomicOr(flags, 1);
}
void launch_od_check(const int* od0, const int* decs, int64_t n, int* flags, cudaStream_t s) {
    if (n == 0) return;
    k_od_check<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(od0, decs, n, flags);
    count_launch();
}

}  // namespace sili
