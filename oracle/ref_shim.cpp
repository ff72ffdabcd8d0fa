// Test-infrastructure harness around the reference's own C++ headers.
//
// TEST INFRASTRUCTURE ONLY: built by oracle/build_ref.py into oracle/_ref/
// and loaded (via ctypes) only by tests/golden/make_golden.py and tests that
// pin the CPU restatement (oracle/sili_oracle.c) against the reference.
//
// The reference's pybind11 module (sili._cpu) hides the delta-CSR internals
// (ULEB128 bytes, FP4 value bytes, per-row offsets, block4 tiles).  This file
// drives the same reference functions with the same template arguments the
// pybind class SparseLinearLayerImpl uses (sili/cpu_backend.cpp:349-1013) and
// exports that internal state through a C ABI.  Every call runs with
// num_cpus = 1, so the reference's thread-local stochastic-rounding stream is
// the calling thread's and fp4_seed_stochastic_rng() makes it reproducible.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "linear_disldo.hpp"
#include "sisldo_ops.hpp"
#include "csr.hpp"
#include "fp4quant.hpp"

namespace {

using S = int;
using V = float;
using COL = uint32_t;
using Weights = SparseLinearWeightsDelta<S, FP4BiPacked, COL>;

struct RefLayer {
    Weights w;
    std::vector<V> in_acc, grad_acc;
    std::size_t idx_budget = 4096, val_budget = 64;
    std::size_t synap_row = 0, eq_row = 0, b4_eq_row = 0;
    std::string err;
};

// Mirrors SparseLinearLayerImpl's constructor (cpu_backend.cpp:375-447).
RefLayer* make_layer(int n_in, int n_out, int max_weights) {
    auto* L = new RefLayer();
    L->idx_budget = static_cast<std::size_t>(max_weights) * 8 + 4096;
    L->val_budget = static_cast<std::size_t>(max_weights) + 64;
    std::vector<S> ptrs(static_cast<std::size_t>(n_in) + 1, 0), idx;
    std::vector<V> wv, iv;
    L->w.connections = delta_csr_from_absolute<S, FP4BiPacked, COL>(
        ptrs, idx, wv, iv, n_in, n_out, L->idx_budget, L->val_budget);
    L->w.connections.set_limits(L->idx_budget, ValueAccessor<FP4BiPacked>::projected_byte_size(L->val_budget));
    L->w.block4.init(n_in, n_out);
    L->w.block4.set_limits(static_cast<std::size_t>(max_weights) * 8 + 4096,
        std::max<std::size_t>(4, static_cast<std::size_t>(max_weights) / BLOCK4_TILE_SLOTS) * BLOCK4_TILE_SLOTS);
    L->w.recompute_stats();
    L->w.probes.rows = n_in;
    L->w.probes.cols = n_out;
    L->in_acc.assign(n_in, 0.f);
    L->grad_acc.assign(n_out, 0.f);
    L->w.out_degree.assign(n_out, 0);
    return L;
}

}  // namespace

extern "C" {

void* ref_create(int n_in, int n_out, int max_weights) { return make_layer(n_in, n_out, max_weights); }
void ref_destroy(void* h) { delete static_cast<RefLayer*>(h); }
const char* ref_last_error(void* h) { return static_cast<RefLayer*>(h)->err.c_str(); }

// cpu_backend.cpp:859-901 (load_weights).
void ref_load_weights(void* h, const int* ptrs, const int* idx, const float* vals, int nnz) {
    auto* L = static_cast<RefLayer*>(h);
    const std::size_t rows = L->w.connections.layout.rows, cols = L->w.connections.layout.cols;
    std::vector<S> p(ptrs, ptrs + rows + 1), ix(idx, idx + nnz);
    std::vector<V> wv(vals, vals + nnz), imp(nnz, 0.f);
    const std::size_t ib = std::max(L->idx_budget, static_cast<std::size_t>(nnz) * 8 + 4096);
    const std::size_t vb = std::max(L->val_budget, static_cast<std::size_t>(nnz) + 64);
    L->w.connections = delta_csr_from_absolute<S, FP4BiPacked, COL>(p, ix, wv, imp, rows, cols, ib, vb);
    L->idx_budget = ib; L->val_budget = vb;
    L->w.connections.set_limits(ib, ValueAccessor<FP4BiPacked>::projected_byte_size(vb));
    L->w.recompute_stats();
    L->w.out_degree.assign(cols, 0);
    for (S c : ix) ++L->w.out_degree[c];
}

// Writes raw stored codes (weight code, importance code) at the element
// positions of the current layout, bypassing quantization -- used to give
// importance non-zero starting values in fixtures.
void ref_set_value_bytes(void* h, const uint8_t* bytes, int64_t n) {
    auto* L = static_cast<RefLayer*>(h);
    auto& d = *L->w.connections.values._data;
    for (int64_t i = 0; i < n && static_cast<std::size_t>(i) < d.size(); ++i) d[i] = bytes[i];
}

void ref_set_scale_rank(void* h, int rank) { static_cast<RefLayer*>(h)->w.scale_rank = rank; }
void ref_set_value_scale_raw_k(void* h, int row, int k, float v) { static_cast<RefLayer*>(h)->w.set_value_scale_raw_k(row, k, v); }
void ref_set_output_scale_raw_k(void* h, int col, int k, float v) { static_cast<RefLayer*>(h)->w.set_output_scale_raw_k(col, k, v); }
void ref_set_importance_scale_raw(void* h, int row, float v) { static_cast<RefLayer*>(h)->w.set_importance_scale_raw(row, v); }
void ref_set_output_importance_scale_raw(void* h, int col, float v) { static_cast<RefLayer*>(h)->w.set_output_importance_scale_raw(col, v); }
float ref_get_value_scale_k(void* h, int row, int k) { return static_cast<RefLayer*>(h)->w.get_value_scale_k(row, k); }
float ref_get_output_scale_k(void* h, int col, int k) { return static_cast<RefLayer*>(h)->w.get_output_scale_k(col, k); }
float ref_get_value_scale_importance_k(void* h, int row, int k) { return static_cast<RefLayer*>(h)->w.get_value_scale_importance_k(row, k); }
float ref_get_output_scale_importance_k(void* h, int col, int k) { return static_cast<RefLayer*>(h)->w.get_output_scale_importance_k(col, k); }
float ref_get_value_scale_momentum_k(void* h, int row, int k) { return static_cast<RefLayer*>(h)->w.get_value_scale_momentum_k(row, k); }
uint32_t ref_get_value_scale_step_k(void* h, int row, int k) { return static_cast<RefLayer*>(h)->w.get_value_scale_step_k(row, k); }
uint32_t ref_get_output_scale_step_k(void* h, int col, int k) { return static_cast<RefLayer*>(h)->w.get_output_scale_step_k(col, k); }

void ref_seed_rng(uint64_t seed) { fp4_seed_stochastic_rng(seed); }

// cpu_backend.cpp:475-492, num_cpus = 1.
void ref_forward_dense(void* h, const float* x, int batch, float* y) {
    auto* L = static_cast<RefLayer*>(h);
    const std::size_t n = static_cast<std::size_t>(batch) * L->w.connections.layout.cols;
    std::fill(y, y + n, 0.f);
    disldo_forward<S, FP4BiPacked, COL>(x, batch, static_cast<S>(L->w.connections.layout.rows), L->w, y, 1);
}

// cpu_backend.cpp:496-529 (SparseLinearLayer / SparseLinearLayerDeterministic; policy 1:
// SparseLinearLayerNoScale / SparseLinearLayerNoScaleDeterministic, :998, :1013; policy 2:
// SparseLinearLayerResync / SparseLinearLayerResyncDeterministic, :993, :1012), num_cpus = 1.
void ref_backward_dense(void* h, const float* x, const float* dy, int batch, float lr,
                        int lr_per_row_nnz, int damp, float beta2, float eps, int stochastic, int policy, float* dx) {
    auto* L = static_cast<RefLayer*>(h);
    const S n_in = static_cast<S>(L->w.connections.layout.rows);
    std::fill(dx, dx + static_cast<std::size_t>(batch) * n_in, 0.f);
#define REF_BWD(POLICY, DEFER, STOCH)                                                            \
    disldo_backward<S, FP4BiPacked, COL, POLICY, DEFER, STOCH>(                                   \
        x, batch, n_in, dy, L->w, dx, L->in_acc.data(), L->grad_acc.data(), lr, 1,                \
        lr_per_row_nnz != 0, damp != 0, beta2, eps, 0.9f, 0.0f, 2.0f, 100.0f)
    if (policy == 1) {
        if (stochastic) REF_BWD(NoScalePolicy<float>, false, true);
        else REF_BWD(NoScalePolicy<float>, false, false);
    } else if (policy == 2) {
        if (stochastic) REF_BWD(RMSpropScalePolicy<float>, true, true);
        else REF_BWD(RMSpropScalePolicy<float>, true, false);
    } else {
        if (stochastic) REF_BWD(RMSpropScalePolicy<float>, false, true);
        else REF_BWD(RMSpropScalePolicy<float>, false, false);
    }
#undef REF_BWD
}

static CSRInput<S, V> make_csr(const int* ptrs, const int* idx, const float* vals, int rows, int cols) {
    CSRInput<S, V> c;
    const int nz = ptrs[rows];
    c.rows = rows; c.cols = cols;
    c.ptrs[0] = std::make_shared<std::vector<S>>(ptrs, ptrs + rows + 1);
    c.indices[0] = std::make_shared<std::vector<S>>(idx, idx + nz);
    c.values[0] = std::make_shared<std::vector<V>>(vals, vals + nz);
    return c;
}

// cpu_backend.cpp:571-585, num_cpus = 1.
void ref_forward_sparse(void* h, const int* ptrs, const int* idx, const float* vals, int batch, float* y) {
    auto* L = static_cast<RefLayer*>(h);
    const std::size_t n = static_cast<std::size_t>(batch) * L->w.connections.layout.cols;
    std::fill(y, y + n, 0.f);
    auto in = make_csr(ptrs, idx, vals, batch, static_cast<int>(L->w.connections.layout.rows));
    sisldo_forward<S, FP4BiPacked, COL>(in, L->w, y, 1);
}

// cpu_backend.cpp:587-603, num_cpus = 1.
void ref_backward_sparse(void* h, const float* x, const int* dptrs, const int* didx, const float* dvals,
                         int batch, float lr, int lr_per_row_nnz, int damp, float beta2, float eps, float* dx) {
    auto* L = static_cast<RefLayer*>(h);
    const S n_in = static_cast<S>(L->w.connections.layout.rows);
    std::fill(dx, dx + static_cast<std::size_t>(batch) * n_in, 0.f);
    auto g = make_csr(dptrs, didx, dvals, batch, static_cast<int>(L->w.connections.layout.cols));
    disldo_backward_sparse_grad<S, FP4BiPacked, COL>(x, batch, L->w, g, dx, L->in_acc.data(), L->grad_acc.data(),
                                                    lr, 1, lr_per_row_nnz != 0, damp != 0, beta2, eps);
}

void ref_build_probes(void* h, int k, int per_row) {
    auto* L = static_cast<RefLayer*>(h);
    delta_csr_build_probes<S, FP4BiPacked, COL>(L->w, L->in_acc.data(), L->grad_acc.data(), k, per_row != 0);
}

int64_t ref_num_probes(void* h) {
    auto* L = static_cast<RefLayer*>(h);
    return L->w.probes.indices[0] ? static_cast<int64_t>(L->w.probes.indices[0]->size()) : 0;
}
void ref_get_probes(void* h, int* rows, int* cols, float* scores) {
    auto* L = static_cast<RefLayer*>(h);
    const int64_t n = ref_num_probes(h);
    for (int64_t i = 0; i < n; ++i) {
        rows[i] = (*L->w.probes.indices[0])[i];
        cols[i] = (*L->w.probes.indices[1])[i];
        scores[i] = (*L->w.probes.values[0])[i];
    }
}

// Returns 1 if the row step did something, 0 if not, -1 on a C++ exception
// (message in ref_last_error).
int ref_synap_row_step(void* h, int row, float cutoff, int max_rw, int max_prune, float imp_eps) {
    auto* L = static_cast<RefLayer*>(h);
    std::size_t r = static_cast<std::size_t>(row);
    try {
        return delta_csr_synap_row_step<S, FP4BiPacked, COL>(L->w, r, cutoff, max_rw, max_prune, imp_eps) ? 1 : 0;
    } catch (const std::exception& e) {
        L->err = e.what();
        return -1;
    }
}

int ref_equalizer_step(void* h) {
    auto* L = static_cast<RefLayer*>(h);
    try {
        delta_csr_equalize_step<S, FP4BiPacked, COL>(L->w.connections, L->eq_row);
        L->w.block4.equalize_step(L->b4_eq_row);
    } catch (const std::exception& e) {
        L->err = e.what();
        return -1;
    }
    return 0;
}

void ref_compact(void* h) {
    auto* L = static_cast<RefLayer*>(h);
    L->w.connections = ::compact<S, FP4BiPacked, COL>(L->w.connections);
    L->w.connections.set_limits(L->idx_budget, ValueAccessor<FP4BiPacked>::projected_byte_size(L->val_budget));
}

int ref_expand_headroom(void* h, float blank_fraction) {
    auto* L = static_cast<RefLayer*>(h);
    try {
        L->w.connections = ::expand_headroom<S, FP4BiPacked, COL>(L->w.connections, blank_fraction);
    } catch (const std::exception& e) { L->err = e.what(); return -1; }
    L->w.connections.set_limits(L->idx_budget, ValueAccessor<FP4BiPacked>::projected_byte_size(L->val_budget));
    return 0;
}

int ref_expand_headroom_to(void* h, int min_nnz_per_row, float blank_fraction) {
    auto* L = static_cast<RefLayer*>(h);
    try {
        L->w.connections = ::expand_headroom_to<S, FP4BiPacked, COL>(L->w.connections, min_nnz_per_row, blank_fraction);
    } catch (const std::exception& e) { L->err = e.what(); return -1; }
    L->w.connections.set_limits(L->idx_budget, ValueAccessor<FP4BiPacked>::projected_byte_size(L->val_budget));
    return 0;
}

// ── state export ────────────────────────────────────────────────────────────
// sizes[0..5] = rows, cols, total_nnz, indices_buf bytes, value bytes, block4 tiles
void ref_sizes(void* h, int64_t* sizes) {
    auto* L = static_cast<RefLayer*>(h);
    const auto& dc = L->w.connections;
    sizes[0] = dc.layout.rows;
    sizes[1] = dc.layout.cols;
    sizes[2] = dc.layout.total_nnz;
    sizes[3] = dc.indices_buf.size();
    sizes[4] = dc.values.size();
    sizes[5] = L->w.block4.n_tiles();
}

void ref_layout(void* h, int64_t* byte_start, int64_t* byte_end, int64_t* elem_start, int64_t* elem_end) {
    auto* L = static_cast<RefLayer*>(h);
    const auto& lay = L->w.connections.layout;
    for (std::size_t r = 0; r <= lay.rows; ++r) { byte_start[r] = lay.byte_start[r]; elem_start[r] = lay.elem_start[r]; }
    for (std::size_t r = 0; r < lay.rows; ++r) { byte_end[r] = lay.byte_end[r]; elem_end[r] = lay.elem_end[r]; }
}

void ref_indices_buf(void* h, uint8_t* out) {
    auto* L = static_cast<RefLayer*>(h);
    std::memcpy(out, L->w.connections.indices_buf.data(), L->w.connections.indices_buf.size());
}

void ref_value_bytes(void* h, uint8_t* out) {
    auto* L = static_cast<RefLayer*>(h);
    const auto& d = L->w.connections.values._data;
    if (d) std::memcpy(out, d->data(), d->size());
}

void ref_accums(void* h, float* in_acc, float* grad_acc) {
    auto* L = static_cast<RefLayer*>(h);
    std::memcpy(in_acc, L->in_acc.data(), L->in_acc.size() * sizeof(float));
    std::memcpy(grad_acc, L->grad_acc.data(), L->grad_acc.size() * sizeof(float));
}
void ref_set_accums(void* h, const float* in_acc, const float* grad_acc) {
    auto* L = static_cast<RefLayer*>(h);
    std::memcpy(L->in_acc.data(), in_acc, L->in_acc.size() * sizeof(float));
    std::memcpy(L->grad_acc.data(), grad_acc, L->grad_acc.size() * sizeof(float));
}

void ref_out_degree(void* h, int* out) {
    auto* L = static_cast<RefLayer*>(h);
    for (std::size_t i = 0; i < L->w.out_degree.size(); ++i) out[i] = L->w.out_degree[i];
}

// stats[0..5] = value_l1, value_l2_sq, value_max_abs, importance_l1, importance_l2_sq, importance_max_abs
void ref_stats(void* h, double* stats) {
    auto* L = static_cast<RefLayer*>(h);
    stats[0] = L->w.value_l1; stats[1] = L->w.value_l2_sq; stats[2] = L->w.value_max_abs;
    stats[3] = L->w.importance_l1; stats[4] = L->w.importance_l2_sq; stats[5] = L->w.importance_max_abs;
}

// Combined (scattered + block4) absolute-CSR export, cpu_backend.cpp:946-983.
int64_t ref_export_nnz(void* h) {
    auto* L = static_cast<RefLayer*>(h);
    std::vector<S> op, oi; std::vector<V> ow, oimp;
    delta_csr_combined_to_absolute<S, FP4BiPacked, COL>(L->w, op, oi, ow, oimp);
    return static_cast<int64_t>(oi.size());
}
void ref_export(void* h, int* ptrs, int* idx, float* w, float* imp) {
    auto* L = static_cast<RefLayer*>(h);
    std::vector<S> op, oi; std::vector<V> ow, oimp;
    delta_csr_combined_to_absolute<S, FP4BiPacked, COL>(L->w, op, oi, ow, oimp);
    std::copy(op.begin(), op.end(), ptrs);
    std::copy(oi.begin(), oi.end(), idx);
    std::copy(ow.begin(), ow.end(), w);
    std::copy(oimp.begin(), oimp.end(), imp);
}

// Logical block4 export: for every live tile, (br, bc) and its 16 slot bytes
// in Block4Tile slot order (slot = lj*4 + li, block4.hpp:306-310).
int64_t ref_block4_tiles(void* h) { return static_cast<int64_t>(static_cast<RefLayer*>(h)->w.block4.n_tiles()); }
void ref_block4_export(void* h, int* br_out, int* bc_out, uint8_t* slots) {
    auto* L = static_cast<RefLayer*>(h);
    auto& st = L->w.block4;
    std::size_t t = 0;
    for (std::size_t br = 0; br < st.block_layout.rows; ++br) {
        const std::size_t n_bc = st.block_layout.row_nnz(br);
        auto cur = st.row_cursor(br);
        for (std::size_t k = 0; k < n_bc; ++k, ++t) {
            const uint32_t bc = cur.advance();
            const auto tile = st.find(static_cast<uint32_t>(br), bc);
            br_out[t] = static_cast<int>(br);
            bc_out[t] = static_cast<int>(bc);
            for (uint32_t li = 0; li < BLOCK4_TILE; ++li)
                for (uint32_t lj = 0; lj < BLOCK4_TILE; ++lj)
                    slots[t * 16 + lj * 4 + li] = tile.at(li, lj);
        }
    }
}

// load_dense_codes (cpu_backend.cpp:910-921)
int ref_load_dense_codes(void* h, const uint8_t* wc, const uint8_t* ic) {
    auto* L = static_cast<RefLayer*>(h);
    const std::size_t rows = L->w.connections.layout.rows, cols = L->w.connections.layout.cols;
    try {
        block4_load_dense<S, FP4BiPacked, COL>(L->w, wc, ic, rows, cols);
    } catch (const std::exception& e) { L->err = e.what(); return -1; }
    L->w.out_degree.assign(cols, S(rows));
    return 0;
}
int ref_b4_expand_headroom(void* h, float bf) {
    auto* L = static_cast<RefLayer*>(h);
    try { block4_expand_headroom<S, FP4BiPacked, COL>(L->w, bf); }
    catch (const std::exception& e) { L->err = e.what(); return -1; }
    return 0;
}
int ref_b4_compact(void* h) {
    auto* L = static_cast<RefLayer*>(h);
    try { block4_compact<S, FP4BiPacked, COL>(L->w); }
    catch (const std::exception& e) { L->err = e.what(); return -1; }
    return 0;
}
void ref_b4_set_switch_point(void* h, uint32_t v) { static_cast<RefLayer*>(h)->w.block4.switch_point = v; }
// per block-row: idx alloc, idx used, tile alloc, tile used, elem alloc, tiles
int64_t ref_b4_rows_n(void* h) { return static_cast<int64_t>(static_cast<RefLayer*>(h)->w.block4.block_layout.rows); }
void ref_b4_rows(void* h, int64_t* out) {
    auto& st = static_cast<RefLayer*>(h)->w.block4;
    const auto& BL = st.block_layout;
    for (std::size_t br = 0; br < BL.rows; ++br) {
        out[6 * br + 0] = BL.byte_start[br + 1] - BL.byte_start[br];
        out[6 * br + 1] = BL.byte_end[br] - BL.byte_start[br];
        out[6 * br + 2] = st.tile_byte_start[br + 1] - st.tile_byte_start[br];
        out[6 * br + 3] = st.tile_byte_end[br] - st.tile_byte_start[br];
        out[6 * br + 4] = BL.elem_start[br + 1] - BL.elem_start[br];
        out[6 * br + 5] = BL.elem_end[br] - BL.elem_start[br];
    }
}
// sparse flag of every tile, in export order
void ref_b4_sparse(void* h, uint8_t* out) {
    auto& st = static_cast<RefLayer*>(h)->w.block4;
    std::size_t t = 0;
    for (std::size_t br = 0; br < st.block_layout.rows; ++br)
        for (std::size_t e = st.block_layout.elem_start[br]; e < st.block_layout.elem_end[br]; ++e) out[t++] = st.tile_is_sparse[e];
}
// Block4View counters (cpu_backend.cpp:51-98)
void ref_b4_view(void* h, int64_t* v) {
    auto& st = static_cast<RefLayer*>(h)->w.block4;
    v[0] = st.n_tiles(); v[1] = st.live_synapses(); v[2] = st.switch_point; v[3] = st.dropped_growth_events;
    v[4] = st.row_merge_overflow_events; v[5] = st.row_merge_overflow_bytes_dropped;
    v[6] = st.total_tile_used_bytes(); v[7] = st.total_tile_alloc_bytes();
}
// std::sort of indices by float keys, with the comparators the synaptogenesis
// step uses (delta_csr_memory.hpp:1149-1152, :1182-1185)
void ref_std_sort_keys(const float* keys, int64_t n, int desc, int64_t* perm) {
    std::vector<std::size_t> idx(static_cast<std::size_t>(n));
    for (std::size_t i = 0; i < idx.size(); ++i) idx[i] = i;
    if (desc) std::sort(idx.begin(), idx.end(), [&](std::size_t a, std::size_t b) { return keys[a] > keys[b]; });
    else std::sort(idx.begin(), idx.end(), [&](std::size_t a, std::size_t b) { return keys[a] < keys[b]; });
    for (std::size_t i = 0; i < idx.size(); ++i) perm[i] = static_cast<int64_t>(idx[i]);
}

// Codec entry points (fp4quant.hpp:68-121, :238-273) for pinning the restatement.
float ref_fp4_decode(uint8_t code) { return fp4_decode_bits(code); }
uint8_t ref_fp4_encode(float v) { return fp4_encode_bits(v); }
uint8_t ref_fp4_quantize_stochastic(float v) { return fp4_quantize_stochastic(v); }

// dense_to_top_k_csr (cpu_backend.cpp:3118-3143): returns nnz; fills outputs.
int ref_top_k_csr(const float* x, int rows, int cols, int k, int* ptrs, int* idx, float* vals) {
    auto csr = top_k_csr<int, float>(const_cast<float*>(x), rows, cols, k, 1);
    const int nnz = static_cast<int>(csr.indices[0]->size());
    std::copy(csr.ptrs[0]->begin(), csr.ptrs[0]->end(), ptrs);
    std::copy(csr.indices[0]->begin(), csr.indices[0]->end(), idx);
    std::copy(csr.values[0]->begin(), csr.values[0]->end(), vals);
    return nnz;
}

}  // extern "C"
