/* CPU restatement of sili's FP4 delta-CSR sparse-layer path.
 *
 * TEST INFRASTRUCTURE ONLY -- this is the parity checker, never the product.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.  Every function cites the reference file:line it restates
 * (paths relative to the reference project root).
 *
 * Pinning: tests/test_oracle_vs_reference.py and the fixtures under
 * tests/golden/ (made by tests/golden/make_golden.py from the reference's own
 * code built here) check this restatement against the reference.
 *
 * Floating-point contract: the file is compiled with -ffp-contract=off and
 * every fused multiply-add is written explicitly (fmaf), so the GPU kernels
 * can reproduce the same operation sequence bit for bit.
 */
#ifndef SILI_ORACLE_H
#define SILI_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct OLayer OLayer;

/* status codes (same values as include/sili_b200.h) */
#define O_OK 0
#define O_EINVAL 1
#define O_ENOMEM 2       /* budget exceeded: reference throws std::bad_alloc */
#define O_EHEADROOM 3    /* row ran out of blank space: std::runtime_error */

/* codec, sili/lib/headers/fp4quant.hpp */
float   o_fp4_decode(uint8_t code);
uint8_t o_fp4_encode(float v);
uint8_t o_fp4_quantize_stochastic_r(float v, uint64_t r);
uint64_t o_rng_draw(uint64_t seed, uint64_t call, uint64_t elem, uint32_t lane);
uint64_t o_xorshift_next(uint64_t* state);

/* layer */
OLayer* o_create(int n_in, int n_out, int max_weights);
void    o_destroy(OLayer* L);
int     o_load_weights(OLayer* L, const int* ptrs, const int* idx, const float* vals, int nnz);
void    o_set_value_bytes(OLayer* L, const uint8_t* bytes, int64_t n);
void    o_set_stochastic(OLayer* L, int stochastic, uint64_t seed);
void    o_set_scale_policy(OLayer* L, int policy);
int     o_set_scale_rank(OLayer* L, int rank);
int     o_get_scale_rank(const OLayer* L);
void    o_set_value_scale_raw_k(OLayer* L, int row, int k, float v);
void    o_set_output_scale_raw_k(OLayer* L, int col, int k, float v);
void    o_set_importance_scale_raw(OLayer* L, int row, float v);
void    o_set_output_importance_scale_raw(OLayer* L, int col, float v);
float   o_get_value_scale_k(const OLayer* L, int row, int k);
float   o_get_output_scale_k(const OLayer* L, int col, int k);
float   o_get_importance_scale(const OLayer* L, int row);
float   o_get_output_importance_scale(const OLayer* L, int col);
float   o_get_value_scale_importance_k(const OLayer* L, int row, int k);
float   o_get_output_scale_importance_k(const OLayer* L, int col, int k);
float   o_get_value_scale_momentum_k(const OLayer* L, int row, int k);
uint32_t o_get_value_scale_step_k(const OLayer* L, int row, int k);
uint32_t o_get_output_scale_step_k(const OLayer* L, int col, int k);
float   o_get_scale(const OLayer* L, int row, int col);
int     o_output_scale_trainable(const OLayer* L);

void    o_forward_dense(OLayer* L, const float* x, int batch, float* y);
void    o_backward_dense(OLayer* L, const float* x, const float* dy, int batch, float lr,
                         int lr_per_row_nnz, int damp, float beta2, float eps, float* dx);
/* column shards: global row synapse counts, this shard's part of the row
 * sums ([2*rows*rank] (sgs, sgc) pairs then [batch*rank] dead-row S), the
 * row steps from the summed parts */
int     o_set_row_shard(OLayer* L, const int* global_row_nnz, int64_t n, int64_t global_n_out);
int64_t o_row_part_len(const OLayer* L, int batch);
int     o_backward_dense_shard(OLayer* L, const float* x, const float* dy, int batch, float lr, int lr_per_row_nnz,
                               int damp, float beta2, float eps, float* dx, double* part);
void    o_apply_row_part(OLayer* L, const float* x, int batch, float lr, float beta2, float eps, const double* part);
void    o_forward_sparse(OLayer* L, const int* ptrs, const int* idx, const float* vals, int batch, float* y);
void    o_backward_sparse(OLayer* L, const float* x, const int* dptrs, const int* didx, const float* dvals,
                          int batch, float lr, int lr_per_row_nnz, int damp, float beta2, float eps, float* dx);

void    o_build_probes(OLayer* L, int k, int per_row);
int64_t o_num_probes(const OLayer* L);
void    o_get_probes(const OLayer* L, int* rows, int* cols, float* scores);
void    o_set_probes(OLayer* L, const int* rows, const int* cols, const float* scores, int64_t n);
int     o_synap_row_step(OLayer* L, int row, float cutoff, int max_rw, int max_prune, float imp_eps, int* did);
int     o_equalizer_step(OLayer* L, int row);
int     o_equalize_to_capacity(OLayer* L, int target_elems, int target_bytes);
void    o_compact(OLayer* L);
int     o_expand_headroom(OLayer* L, float blank_fraction);
int     o_expand_headroom_to(OLayer* L, int min_nnz_per_row, float blank_fraction);
void    o_rescale_value_row(OLayer* L, int row, float new_scale);
void    o_rescale_importance_row(OLayer* L, int row, float new_scale);

/* state export */
void    o_sizes(const OLayer* L, int64_t* sizes);   /* rows, cols, nnz, idx bytes, val bytes, tiles */
void    o_layout(const OLayer* L, int64_t* bs, int64_t* be, int64_t* es, int64_t* ee);
void    o_indices_buf(const OLayer* L, uint8_t* out);
void    o_value_bytes(const OLayer* L, uint8_t* out);
void    o_accums(const OLayer* L, float* in_acc, float* grad_acc);
void    o_set_accums(OLayer* L, const float* in_acc, const float* grad_acc);
void    o_zero_accum(OLayer* L);
void    o_out_degree(const OLayer* L, int* out);
void    o_stats(const OLayer* L, double* stats);
void    o_recompute_stats(OLayer* L);
int64_t o_export_nnz(const OLayer* L);
void    o_export(const OLayer* L, int* ptrs, int* idx, float* w, float* imp);

/* block4 tiles, sili/lib/headers/block4.hpp + delta_csr_memory.hpp:769-945 */
int     o_load_dense_codes(OLayer* L, const uint8_t* weight_codes, const uint8_t* importance_codes);
int     o_b4_expand_headroom(OLayer* L, float blank_fraction, int64_t min_slack);
int     o_b4_equalize_step(OLayer* L, int64_t row);
void    o_b4_set_switch_point(OLayer* L, uint32_t v);
/* sparse-gradient block4 draws from the reference's xorshift64* stream (pinning) */
void    o_set_ref_stream(OLayer* L, int on, uint64_t seed);
int64_t o_b4_ntiles(const OLayer* L);
void    o_b4_export(const OLayer* L, int* br, int* bc, uint8_t* slots, uint8_t* sparse);
void    o_b4_rows(const OLayer* L, int64_t* out);   /* 6 per block-row */
void    o_b4_view(const OLayer* L, int64_t* v);     /* 8 counters */

/* libstdc++ std::sort restatement (permutation of 0..n-1 by keys) */
void    o_std_sort_keys(const float* keys, int64_t n, int desc, int64_t* perm);

/* activation sparsifiers, sili/cpu_backend.cpp:3075-3143 */
int64_t o_dense_to_csr(const float* x, int rows, int cols, float threshold, int* ptrs, int* idx, float* vals);
int64_t o_top_k_csr(const float* x, int rows, int cols, int64_t k, int* ptrs, int* idx, float* vals);

/* the top-k growth rule (no reference function): exact top-k of |dy^T x| */
int64_t o_topk_dyx_candidates(const OLayer* L, const float* x, const float* dy, int batch, int64_t k,
                              int* rows, int* cols, float* scores);
int     o_topk_dyx_step(OLayer* L, const float* x, const float* dy, int batch, int64_t k);
/* its second half for a given candidate list (ascending (row, col)) */
int     o_topk_apply(OLayer* L, const int* rows, const int* cols, const float* scores, int64_t n);
/* the rule's score at given positions */
void    o_dyx_scores_at(const float* x, const float* dy, int batch, int64_t n_in, int64_t n_out, const int* rows,
                        const int* cols, int64_t n, float* out);

#ifdef __cplusplus
}
#endif
#endif
