// Launch wrappers for the sili_b200 kernels (host-callable, stream-ordered).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <string>

namespace sili {

// process-wide count of kernel launches made through the launch_* wrappers
void count_launch(int n = 1);
long long launch_count();

// Everything a kernel needs to read or write one layer's device state.
struct LayerView {
    int64_t n_in, n_out;
    int rank;
    const int64_t* bs;   // byte_start [n_in+1]
    const int64_t* be;   // byte_end   [n_in]
    const int64_t* es;   // elem_start [n_in+1]
    const int64_t* ee;   // elem_end   [n_in]
    const uint8_t* idx;  // ULEB128 column deltas
    uint8_t* val;        // FP4BiPacked bytes: weight code << 4 | importance code
    float* vs;           // value_scale [n_in*rank]
    float* os;           // output_scale [n_out*rank]
    float* vsi;          // value_scale_importance [n_in*rank]
    float* osi;          // output_scale_importance [n_out*rank]
    float* vsm;          // value_scale_momentum [n_in*rank]
    uint32_t* vstep;     // value_scale_step [n_in*rank]
    uint32_t* ostep;     // output_scale_step [n_out*rank]
    const float* is;     // importance_scale [n_in]
    const float* ois;    // output_importance_scale [n_out]
    // derived index (rebuilt after structural changes)
    const int* rowptr;   // [n_in+1] exclusive scan of row nnz
    const int* abs_cols; // [nnz] absolute column of every live synapse, row-major
    const int* colptr;   // [n_out+1] CSC shadow, each column padded to a multiple of 8 entries:
                         // column c at [colptr[c], colptr[c+1])
    const int* crow;     // their rows, ascending within a column; padding: row n_in (the zero input row)
    const int* cvpos;    // their positions in val[]; padding: -1 (weight 0)
    const int* b4_nt = nullptr;  // [ceil(n_in/4)] block4 tiles per block-row (null: no block4)
    const int* colptr_x = nullptr;  // [n_out+1] exact (unpadded) column offsets of the same CSC
    const int* cpack = nullptr;     // per padded CSC entry: row << 4 | weight code (padding: n_in << 4)
    // when set, kernels that rewrite weight codes also rewrite their packed
    // words: fcpos[f] = the padded CSC position of synapse f (row-major order)
    int* cpack_upd = nullptr;
    // the Resync classes' true-units weight for dx at learning rate 0:
    // (w * vs) * os of component 0, the reference build's association
    // (linear_disldo.hpp:702), instead of w * S
    bool true_units = false;
    const int* fcpos = nullptr;
};

// One layer's block4 store (4x4 dense FP4 tiles, block4.hpp:1016-1490) on the
// device.  Block-row br (input rows 4br..4br+3) owns the tile slots
// [es[br], es[br] + capacity) of which the first nt[br] are live, in
// ascending block-column.  A tile is 16 slot bytes, slot = lj*4 + li
// (Block4Tile::slot_index, block4.hpp:309), byte = importance << 4 | weight.
// sparse[] and alloc[] carry the reference's packed-tile flag and per
// block-row allocations (index bytes, tile bytes, tile slots), which decide
// growth, budget errors and eviction exactly as the reference's do.
struct B4View {
    int64_t BR = 0, BC = 0;
    const int64_t* es = nullptr;    // [BR+1] tile region start per block-row
    int* nt = nullptr;              // [BR] live tiles per block-row
    int* bc = nullptr;              // [cap] block-column of each tile
    uint4* tile = nullptr;          // [cap] 16 slot bytes
    uint8_t* sparse = nullptr;      // [cap] packed-tile flag
    int64_t* alloc = nullptr;       // [3*BR] idx bytes, tile bytes, tile slots
    unsigned long long* counters = nullptr;  // [3] dropped growth, overflow events, overflow bytes
    uint32_t switch_point = 10;
    // tile column index (rebuilt after structural changes): tiles of
    // block-column c at [cptr[c], cptr[c+1]), ascending block-row
    const int* cptr = nullptr;
    const int* ctile = nullptr;     // global tile slot
    const int* cbr = nullptr;       // its block-row
};

struct UpdateParams {
    float lr, beta2, eps;
    bool lr_per_row_nnz, damp, stochastic, os_trainable;
    uint64_t call_key;
    const float* pow_tab;  // pow_tab[s] = powf(beta2, s) (host libm), s < pow_n
    int pow_n;
    float* colg;           // [n_out*rank] output_scale gradient sums (os_trainable)
    float* colc;           // [n_out*rank] forward-contribution sums
    double* stats;         // [4] importance l1 new-old, l2 new-old (sums)
    float* stat_max;       // [1] importance max (float bits as uint max)
    // *dy_flag == dy_tag: this call's dy holds an inf or NaN (null: unknown,
    // treated as "may hold one")
    const unsigned long long* dy_flag = nullptr;
    unsigned long long dy_tag = 0;
    // column shard of a layer (dense update only): the rows' global synapse
    // counts divide the learning rate, and each row's value_scale sums go to
    // row_part[2*(r*rank+k) + {0,1}] instead of being applied
    const int* row_nnz_g = nullptr;
    double* row_part = nullptr;
    // NoScalePolicy (delta_csr_types.hpp:528-537): the dense backward's
    // value_scale and output_scale steps (ScalePolicy::update,
    // linear_disldo.hpp:914-925, 2075) do nothing
    bool scale_noop = false;
    // DeferredScaleWrite (the Resync classes, linear_disldo.hpp:686-790):
    // the update keeps each synapse's true-units (cw, ci) in def_cw / def_ci
    // at its value position, stored as codes by launch_resync_store once the
    // scales are final
    bool resync = false;
    float* def_cw = nullptr;
    float* def_ci = nullptr;
};

void launch_transpose(const float* in, float* out, int64_t R, int64_t C, cudaStream_t s);
// out[0..C) = in[0..C), out[C] = 0 (a one-row input and its zero row)
void launch_copy_pad(const float* in, float* out, int64_t C, cudaStream_t s);
// nonfinite (optional): set to `tag` when some |x| is inf or NaN
void launch_accum_abs(const float* x, float* acc, int B, int64_t n, cudaStream_t s,
                      unsigned long long* nonfinite = nullptr, unsigned long long tag = 0);
void launch_accum_abs_t(const float* xT, float* acc, int B, int64_t n, cudaStream_t s);
// out = in^T ([R, C] -> [C, R]) with launch_accum_abs(in, acc, R, C, nonfinite, tag) fused
void launch_transpose_accum(const float* in, float* out, int64_t R, int64_t C, float* acc,
                            unsigned long long* nonfinite, unsigned long long tag, cudaStream_t s);
// forward: y[B, n_out] from xT [n_in, B]; sparse_formula selects the
// sisldo_forward arithmetic (sisldo_ops.hpp:289-308) over disldo_forward's.
void launch_forward(const LayerView& L, const float* xT, int B, float* y, bool sparse_formula,
                    cudaStream_t s);
// dense backward at lr == 0: dx [B, n_in] from dyT [n_out, B] (bit-exact order)
void launch_backward_dx(const LayerView& L, const float* dyT, int B, float* dx, cudaStream_t s);
// dense backward at lr != 0: fused per-synapse update + dxT [n_in, B]
// The forward with x rows staged in shared memory per row tile (kernels_forward.cu):
// needs L.cpack and L.colptr_x; returns false (launching nothing) when the
// shape is better served by launch_forward.
bool launch_forward_rows(const LayerView& L, const float* xT, int B, float* y, bool sparse_formula,
                         cudaStream_t s);
// whether launch_forward_rows would run for this shape (it needs L.cpack)
bool forward_rows_applies(const LayerView& L, int B);

// The suffix layers of one folded layer (same n_in, n_out = n_folds *
// out_dim, scale rank 1), for the one-launch FoldedLayer forward.
constexpr int kFoldedMaxSuffixes = 4;
struct FoldedView {
    int ns = 0;
    int n_in = 0;
    int64_t n_cols = 0, out_dim = 0;
    int n_folds = 0;
    bool fold_sum = true;
    int J = 1;   // output columns per CTA (set by the launcher)
    const int* colptr[kFoldedMaxSuffixes] = {};
    const int* colptr_x[kFoldedMaxSuffixes] = {};
    const int* cpack[kFoldedMaxSuffixes] = {};
    const float* vs[kFoldedMaxSuffixes] = {};
    const float* os[kFoldedMaxSuffixes] = {};
};
bool folded_forward_applies(const FoldedView& F, int B);
// The block4 forward on the tensor cores (block4_tc.cu): rank 1, B >= 16.
// Scratch: the split activations (b4_tc_xsplit_elems bf16) and the partial
// sums (b4_tc_scratch_floats, which also picks the input-row slices).
// dx = false: the forward (y [B, n_out] += ...), true: the lr = 0 dx
// (dx [B, n_in] += ...).
bool b4_tc_applies(const LayerView& L, const B4View& V, int B);
int64_t b4_tc_scratch_floats(const LayerView& L, int B, bool dx, int* kslices);
int64_t b4_tc_xsplit_elems(const LayerView& L, int B, bool dx);
// the panel map (tile slot per 32 x 16 block cell), rebuilt when the tile
// layout changes
int64_t b4_tc_pmap_elems(const LayerView& L, bool dx);
void launch_b4_panel_map(const LayerView& L, const B4View& V, bool dx, int* pmap, cudaStream_t s);
int launch_b4_forward_tc(const LayerView& L, const B4View& V, const float* xT, int B, float* y, uint16_t* xsplit,
                         float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s);
int launch_b4_dx_tc(const LayerView& L, const B4View& V, const float* dyT, int B, float* dx, uint16_t* xsplit,
                    float* part, int kslices, const int* pmap, unsigned int* err, cudaStream_t s);
int set_error(int code, const std::string& msg);

// y = [B, out_dim] (fold_sum) or [B, n_cols]; false when the shape rules
// (folded_forward_applies) do not hold
bool launch_folded_forward(FoldedView F, const float* xT, int B, float* y, cudaStream_t s);
// y[b, c] = 0 + raw_0[b, c] + raw_1[b, c] + ... (n raws of [B, n_cols])
void launch_suffix_sum(const float* const* raws, int n, int64_t count, float* y, cudaStream_t s);
// L.cpack from crow / cvpos / val over the padded CSC (its length is colptr[n_out])
void launch_pack_csc(const LayerView& L, int64_t bound, int* cpack, cudaStream_t s);
void launch_backward_update(const LayerView& L, const float* xT, const float* dyT, int B,
                            const UpdateParams& P, float* dxT, cudaStream_t s);
// the same for B <= 128 (kernels_update.cu); launch_backward_update calls it
void launch_backward_update_tiled(const LayerView& L, const float* xT, const float* dyT, int B,
                                  const UpdateParams& P, float* dxT, cudaStream_t s);
// the deferred stores of a Resync update under the final scales
// (linear_disldo.hpp:2083-2112)
void launch_resync_store(const LayerView& L, const UpdateParams& P, cudaStream_t s);
void launch_output_scale_update(const LayerView& L, const int* out_degree, const UpdateParams& P,
                                cudaStream_t s);
// column shards: this shard's part of the dead-row sums S[b,k] (over its
// columns), and the row steps from the parts summed over every shard
void launch_dead_S(const LayerView& L, const float* dy, int B, double* S, cudaStream_t s);
void launch_apply_row_part(const LayerView& L, const int* row_nnz_g, int64_t g_n_out, const double* part,
                           const float* xT, int B, const UpdateParams& P, cudaStream_t s);
void launch_dead_rows(const LayerView& L, const float* xT, const float* dy, int B, double* scratchS,
                      const UpdateParams& P, cudaStream_t s);
// sparse-gradient backward: dyT/presT dense [n_out, B] with a presence mask
void launch_backward_sparse(const LayerView& L, const float* xT, const float* dyT,
                            const uint8_t* presT, int B, const UpdateParams& P, double* sgs,
                            double* sgc, float* dxT, cudaStream_t s);
void launch_sparse_scale_update(const LayerView& L, const double* sgs, const double* sgc,
                                const UpdateParams& P, cudaStream_t s);
// densify a row-major CSR [rows, cols] into a transposed dense [cols, rows]
// (+ optional presence bytes); outputs must be zero-filled by the caller.
void launch_csr_to_dense_t(const int* ptrs, const int* idx, const float* vals, int rows, int cols,
                           float* outT, uint8_t* presT, cudaStream_t s);

// structural index
void launch_row_nnz(const int64_t* es, const int64_t* ee, int64_t n_in, int* rowptr_plus1, cudaStream_t s);
void launch_decode_rows(const LayerView& L, int* abs_cols, int* frow, int* fvpos, int* colcount,
                        cudaStream_t s);
void launch_gather_csc(const int* sorted_f, const int* sorted_col, const int* frow, const int* fvpos,
                       const int* colptr, const int* pcolptr, int64_t nnz, int* crow, int* cvpos, int* fcpos,
                       cudaStream_t s);
void launch_pad_csc(const int* colcount, const int* pcolptr, int64_t n_cols, int n_in, int* crow, int* cvpos,
                    cudaStream_t s);
void launch_pad_counts(const int* colcount, int64_t n, int* out, cudaStream_t s);

// state helpers
void launch_fill_f32(float* p, int64_t n, float v, cudaStream_t s);
void launch_fill_scale_default(float* p, int64_t begin, int64_t end, int rank, cudaStream_t s);
void launch_recode_values(uint8_t* val, int64_t n, cudaStream_t s);
void launch_stats(const LayerView& L, double* sums, float* maxes, cudaStream_t s);
void launch_export(const LayerView& L, int* idx, float* w, float* imp, cudaStream_t s);
void launch_copy_rows(const LayerView& L, const int64_t* new_bs, const int64_t* new_es, uint8_t* new_idx,
                      uint8_t* new_val, bool recode, cudaStream_t s);
// load_weights import (delta_csr_from_absolute): per-synapse ULEB128 length,
// per-row byte/elem counts, and the encode/write pass.
void launch_import_lengths(const int* ptrs, const int* idx, int n_in, int* len, cudaStream_t s);
void launch_import_rows(const int* ptrs, const int* boff, int n_in, int64_t* row_bytes, int64_t* row_n,
                        cudaStream_t s);
void launch_import_write(const int* ptrs, const int* idx, const float* vals, const float* imps, const int* boff,
                         int n_in, const int64_t* bs, const int64_t* es, uint8_t* ibuf, uint8_t* vbuf, cudaStream_t s);
void launch_add_offset(int64_t* p, int64_t begin, int64_t end, int64_t delta, cudaStream_t s);
void launch_rescale_row(const LayerView& L, int row, float old_scale, float new_scale, bool weight,
                        cudaStream_t s);
void launch_set_bytes(uint8_t* dst, const uint8_t* src, int64_t n, cudaStream_t s);
void launch_fp4_quantize(const float* v, uint8_t* out, int64_t n, cudaStream_t s);
void launch_dense_to_csr_count(const float* x, int rows, int cols, float thr, int* counts, cudaStream_t s);
void launch_dense_to_csr_fill(const float* x, int rows, int cols, float thr, const int* ptrs, int* idx,
                              float* vals, cudaStream_t s);
void launch_abs_keys(const float* x, int64_t n, uint32_t* keys, int* ids, cudaStream_t s);
void launch_topk_emit(const float* x, const int* flat_sorted, int64_t k, int cols, int* rowcount,
                      int* idx, float* vals, cudaStream_t s);

// probes (delta_csr_build_probes)
void launch_iota(int* p, int64_t n, cudaStream_t s);
void launch_probe_flags(const LayerView& L, const int* in_sorted, int kin, const int* out_sorted, int kout,
                        int* flags, cudaStream_t s);
void launch_probe_emit(const int* in_sorted, int kin, const int* out_sorted, int kout, const int* flags,
                       const int* pos, const float* in_acc, const float* grad_acc, int* prow, int* pcol,
                       float* pval, cudaStream_t s);
void launch_probe_per_row(const LayerView& L, const int* in_sorted, int kin, const int* out_sorted,
                          int64_t n_out, int k, const float* in_acc, const float* grad_acc, int* prow,
                          int* pcol, float* pval, int* counts, cudaStream_t s);

}  // namespace sili

namespace sili {
// ── synaptogenesis (csrc/synap.cu) ──────────────────────────────────────────
struct SynView {
    int64_t n_in = 0, n_out = 0;
    const int64_t* bs = nullptr;
    int64_t* be = nullptr;
    const int64_t* es = nullptr;
    int64_t* ee = nullptr;
    uint8_t* idx = nullptr;
    uint8_t* val = nullptr;
    int* out_degree = nullptr;
    int* od_decs = nullptr;                 // [n_out] decrements requested per column
    // block4 (same layout as B4View)
    const int64_t* b4_es = nullptr;
    int* nt = nullptr;
    int* b4_bc = nullptr;
    uint4* b4_tile = nullptr;
    uint8_t* b4_sparse = nullptr;
    int64_t* alloc = nullptr;
    unsigned long long* counters = nullptr;
    uint32_t switch_point = 10;
    int64_t max_idx = 0, max_tile = 0, tot_idx0 = 0, tot_tile0 = 0;
    unsigned long long* grow = nullptr;     // [2] allocation growth: index bytes, tile bytes
    // probes (COO in the reference's order) and their per-row index
    int64_t n_probes = 0;
    const int* pcol = nullptr;
    const float* pval = nullptr;
    const int* pr_ptr = nullptr;            // [n_in+1]
    const int* pr_idx = nullptr;            // probe ids grouped by row, COO order kept
    // results
    unsigned long long* nnz_delta = nullptr;
    long long* err_i = nullptr;             // first failing sweep position
    int* err_code = nullptr;
    int* flags = nullptr;                   // 1: out_degree clamp possible, 4: tile capacity short
    uint8_t* did = nullptr;                 // per sweep position
    // per-thread scratch
    uint8_t* scratch = nullptr;
    int64_t scratch_stride = 0, scratch_m = 0, scratch_p = 0;
};
struct SynParams {
    int64_t row0 = 0, nrows = 0, limit = 0;
    float cutoff = 0.0f, eps = 1e-3f;
    int max_rw = 0, max_prune = 8;
};
void launch_synap(const SynView& V, const SynParams& P, bool sequential, cudaStream_t s);
void launch_od_check(const int* od0, const int* decs, int64_t n, int* flags, cudaStream_t s);
void launch_lower_bound(const int* sorted_keys, int n, int64_t nkeys, int* ptr, cudaStream_t s);
// bytes of per-thread scratch for rows of up to m entries and p probes
inline int64_t synap_scratch_stride(int64_t m, int64_t p) {
    auto r = [](int64_t b) { return (b + 15) & ~int64_t(15); };
    return r(m * 4) + r(m) + r(m * 4) + r(m * 4) + r(m) + r(m * 4) + r(m * 4) + r(m) + r(m * 4) +
           5 * r(p * 4);
}

// ── block4 (csrc/block4.cu) ──────────────────────────────────────────────────
// load_dense_codes: every tile of the [BR, BC] grid from row-major codes;
// row_used[br] receives the reference's packed byte length of the row.
// FoldedLayer fold sum: y[B, out_dim] from raw[B, n_folds*out_dim]
void launch_fold_sum(const float* raw, int B, int n_folds, int64_t out_dim, float* y, cudaStream_t s);
void launch_fold_broadcast(const float* dy, int B, int64_t out_dim, int64_t j0, int64_t w, int n_folds, float* raw,
                           cudaStream_t s);

// ── top-k |dy^T x| growth rule (csrc/topk.cu) ───────────────────────────────
void launch_exist_bits(const int* rowptr, const int* abs_cols, int64_t n_in, int64_t words, uint32_t* bits,
                       cudaStream_t s);
void launch_dyx_scores(const float* x, const float* dy, int B, int64_t n_in, int64_t n_out, const uint32_t* bits,
                       int64_t words, uint32_t* keys, cudaStream_t s);
// device-side radix select state (csrc/topk.cu)
struct SelState {
    unsigned int prefix, mask;   // the key bits fixed so far
    long long need;              // keys still to take at or below the prefix
    long long eq_count;          // keys equal to the final prefix
};
void launch_sel_init(SelState* st, int64_t need, cudaStream_t s);
void launch_digit_hist(const uint32_t* keys, int64_t n, int shift, const SelState* st, unsigned int* hist, int sms,
                       cudaStream_t s);
void launch_digit_pick(unsigned int* hist, int shift, SelState* st, cudaStream_t s);
void launch_select_ge(const uint32_t* keys, int64_t n, const SelState* st, int64_t* out, unsigned long long* count,
                      int64_t cap, int sms, cudaStream_t s);
void launch_prune_keys(const LayerView& L, const float* w, uint32_t* keys, int* ids, cudaStream_t s);
void launch_mark_drop(const int* sorted_ids, int npr, const int* abs_cols, uint8_t* drop, int* out_degree,
                      cudaStream_t s);
void launch_cand_rowptr(const int64_t* cand, int nc, int64_t n_out, int64_t n_in, int* cptr, cudaStream_t s);
void launch_topk_merge(const LayerView& L, const float* w, const float* imp, const uint8_t* drop, const int64_t* cand,
                       const uint32_t* keys, const int* cptr, int pass, int* cnt, const int* newptr, int* nidx,
                       float* nw, float* nimp, int* out_degree, cudaStream_t s);

void launch_b4_load_dense(const uint8_t* wc, const uint8_t* ic, int64_t n_in, int64_t n_out, const B4View& V,
                          int64_t* row_used, cudaStream_t s);
// per block-row [3*BR]: packed tile bytes in use, ULEB128 index bytes, live slots
void launch_b4_row_used(const B4View& V, int64_t* out, cudaStream_t s);
// forward contribution y[B, n_out] += block4 part (after the scattered part)
void launch_b4_forward(const LayerView& L, const B4View& V, const float* xT, int B, float* y, cudaStream_t s);
// dx at lr == 0: dx[B, n_in] += block4 part, tiles in stored order per row
void launch_b4_dx(const LayerView& L, const B4View& V, const float* dyT, int B, float* dx, cudaStream_t s);
// lr != 0: fused update of every tile slot + dxT [n_in, B] += block4 part,
// then merge_row_workspace's eviction and the block4 value_scale step
void launch_b4_update(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                      const UpdateParams& P, float* dxT, cudaStream_t s);
// the same update as passes with every tile in parallel (block-rows
// [br0, br1); scratch hsb: 4*B floats, mrb: 4*rank*2 doubles, mcb (when the
// output scale trains): 16*rank*2 floats per tile slot from part_base =
// es[br0] to es[br1]; needs the tile column index); only when n_out % 4 == 0
bool b4_update_split_applies(const LayerView& L);
void launch_b4_update_split(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                            const UpdateParams& P, float* dxT, int64_t br0, int64_t br1, int64_t part_base,
                            float* hsb, double* mrb, float* mcb, cudaStream_t s);
// the eviction pass after every chunk's update (a half-warp per block-row)
// the warp-per-row update (no per-tile scratch; the packed flags are left to
// launch_b4_evict_rows, which refreshes them)
bool b4_update_rows_applies(const LayerView& L, int B);
void launch_b4_update_rows(const LayerView& L, const B4View& V, const float* xT, const float* dyT, int B,
                           const UpdateParams& P, float* dxT, int64_t br0, int64_t br1, int64_t part_base,
                           float* mcb, cudaStream_t s);
void launch_b4_evict_rows(const LayerView& L, const B4View& V, cudaStream_t s);
// the tiles of every block-row moved to new offsets (new arrays)
void launch_b4_move(int64_t BR, const int64_t* old_es, const int64_t* new_es, const int* nt, const int* bc,
                    const uint4* tile, const uint8_t* sp, int* nbc, uint4* ntile, uint8_t* nsp, cudaStream_t s);
// sparse-input forward block4 windows: y[B, n_out] += (xT/presT [n_in, B])
void launch_b4_forward_sparse(const LayerView& L, const B4View& V, const float* xT, const uint8_t* presT, int B,
                              float* y, cudaStream_t s);
// sparse-gradient backward block4 part (dyT/presT [n_out, B]); dxT [n_in, B] +=
void launch_b4_backward_sparse(const LayerView& L, const B4View& V, const float* xT, const float* dyT,
                               const uint8_t* presT, int B, const UpdateParams& P, float* dxT, cudaStream_t s);
// tile list for the column index: (bc key, global slot, block-row) of every live tile
void launch_b4_list(const B4View& V, const int* tile_off, int* keys, int* slots, int* brs, cudaStream_t s);
void launch_b4_index(const int* sorted_keys, const int* perm, int n, int64_t BC, const int* slots, const int* brs,
                     int* cptr, int* ctile, int* cbr, cudaStream_t s);
}  // namespace sili
