/* sili_b200 -- C ABI of the B200 (sm_100a) FP4 delta-CSR sparse-layer library.
 *
 * One opaque handle per sparse linear layer.  The layer's state (ULEB128
 * column-delta bytes, FP4 weight/importance bytes, per-row offsets and
 * headroom, per-row/per-column scales, synaptogenesis accumulators, probes)
 * lives in device memory of the device the layer was created on.
 *
 * Every entry point mirrors one method of the reference's pybind11 class
 * sili._cpu.SparseLinearLayer (sili/cpu_backend.cpp:349-1013, bound at
 * :1506-1738) and is cited below.  Conventions:
 *
 *  - Return value: SILI_OK (0) or an error code.  sili_last_error() gives the
 *    message of the calling thread's last failure.  The pybind11 module maps
 *    SILI_EINVAL -> ValueError, SILI_ENOMEM -> MemoryError, SILI_EHEADROOM and
 *    SILI_ECUDA -> RuntimeError, as the reference's C++ exceptions map.
 *  - Array pointers may be host or device memory (detected per pointer).
 *    Host arrays are copied in / out inside the call and the call returns
 *    after the copy back; device arrays are used in place and the work is
 *    enqueued on `stream` (NULL = the layer's own stream) without a host
 *    synchronisation.  Device input arrays must be complete on that stream's
 *    timeline.  Entry points without a stream argument (setters, getters,
 *    structural calls) work on the layer's own stream and return after it
 *    drains; a caller that enqueued work on another stream orders the two
 *    itself (e.g. synchronises that stream first).
 *  - Activations and gradients are fp32, row-major [batch, features].
 *  - Sizes are C int, as in the reference (S = int, cpu_backend.cpp:353).
 *
 * There is no CPU fallback: every compute entry point runs CUDA kernels and
 * fails with SILI_ECUDA when no CUDA device is usable.
 */
#ifndef SILI_B200_H
#define SILI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SILI_OK 0
#define SILI_EINVAL 1     /* std::invalid_argument -> ValueError */
#define SILI_ENOMEM 2     /* std::bad_alloc (budget) -> MemoryError */
#define SILI_EHEADROOM 3  /* std::runtime_error (row out of blank space) */
#define SILI_ECUDA 4      /* CUDA error / no device */
#define SILI_ETIMEOUT 5   /* a bounded device-side wait gave up */

/* backward flags */
#define SILI_LR_PER_ROW_NNZ 1u
#define SILI_DAMP_BY_IMPORTANCE 2u

typedef struct sili_layer sili_layer;

const char* sili_last_error(void);
int sili_device_count(int* count);
/* Number of CUDA kernels this library has launched in this process (all
 * layers, all devices) -- lets a caller count the device work of a region. */
int sili_kernel_launches(int64_t* count);
/* Profiling: when enabled, every compute call records CUDA events around its
 * main kernel; sili_layer_kernel_ms returns the last forward / backward main
 * kernels' durations in milliseconds (synchronising the layer's stream). */
int sili_layer_set_kernel_timing(sili_layer* h, int enable);
int sili_layer_kernel_ms(sili_layer* h, float* forward_ms, float* backward_ms);
/* device memory the layer holds, in bytes (allocated capacities): the
 * delta-CSR format with its headroom (index bytes, value bytes, row
 * offsets), the derived column index, and everything including scales,
 * statistics and kept scratch.  No reference counterpart (the reference's
 * layer lives in host memory); any pointer may be NULL. */
int sili_layer_device_bytes(sili_layer* h, int64_t* format, int64_t* index, int64_t* total);
/* Measurement utility, no counterpart in the reference: the device's FP32
 * FMA throughput (16 independent fma chains per thread, every SM full, best
 * of 4 timed launches of `iters` iterations), the denominator of the FP32
 * fraction reported for the issue-bound kernels.  ms (may be NULL) gets the
 * best launch's duration. */
int sili_fp32_fma_peak(int device, int iters, double* tflops, double* ms);

/* ── lifetime / loading ──────────────────────────────────────────────────── */
/* SparseLinearLayerImpl(n_inputs, n_outputs, max_weights, num_cpus),
 * cpu_backend.cpp:375-447.  stochastic = 1 for SparseLinearLayer,
 * 0 for SparseLinearLayerDeterministic (aliases :992-1013). */
int sili_layer_create(int n_in, int n_out, int max_weights, int device, int stochastic,
                      sili_layer** out);
int sili_layer_destroy(sili_layer* h);
/* load_weights(ptrs, indices, weights), cpu_backend.cpp:859-901 */
int sili_layer_load_weights(sili_layer* h, const int* ptrs, const int* idx, const float* vals, int nnz);
/* fp4_seed_stochastic_rng(seed), fp4quant.hpp:186-188 (per-layer here) */
int sili_layer_seed_rng(sili_layer* h, uint64_t seed);
int sili_layer_sync(sili_layer* h);

/* ── scales (cpu_backend.cpp:465-471, :792-829, bindings :1578-1650) ────── */
#define SILI_SCALE_VALUE 0              /* value_scale[row*rank+k]          */
#define SILI_SCALE_OUTPUT 1             /* output_scale[col*rank+k]         */
#define SILI_SCALE_IMPORTANCE 2         /* importance_scale[row]            */
#define SILI_SCALE_OUTPUT_IMPORTANCE 3  /* output_importance_scale[col]     */
#define SILI_SCALE_VALUE_IMPORTANCE 4   /* value_scale_importance (read)    */
#define SILI_SCALE_OUTPUT_SCALE_IMPORTANCE 5 /* output_scale_importance (read) */
#define SILI_SCALE_VALUE_MOMENTUM 6     /* value_scale_momentum (read)      */
int sili_layer_set_scale_rank(sili_layer* h, int rank);
int sili_layer_get_scale_rank(sili_layer* h, int* rank);
/* set_*_scale_raw(_k): kind SILI_SCALE_VALUE/OUTPUT/IMPORTANCE/OUTPUT_IMPORTANCE */
int sili_layer_set_scale(sili_layer* h, int kind, int index, int k, float v);
int sili_layer_get_scale(sili_layer* h, int kind, int index, int k, float* v);
/* bulk write of entries [0, n) of a scale vector's [n_rows_or_cols * rank]
 * view (kind VALUE / OUTPUT / IMPORTANCE / OUTPUT_IMPORTANCE; host or device
 * array): n calls of set_*_scale_raw(_k) in one copy, with their effects
 * (the vector's logical size grows to n; setting output scales makes them
 * trainable, cpu_backend.cpp:792-829) */
int sili_layer_set_scales(sili_layer* h, int kind, const float* v, int n);
/* bulk read of a whole scale vector (n entries of the [n_rows_or_cols * rank] view) */
int sili_layer_get_scales(sili_layer* h, int kind, float* out, int n);
/* value_scale_step / output_scale_step counters (bias correction) */
int sili_layer_get_steps(sili_layer* h, int which /*0 value, 1 output*/, uint32_t* out, int n);
/* rescale_value_row / rescale_importance_row, cpu_backend.cpp:815-829 */
int sili_layer_rescale_row(sili_layer* h, int kind, int row, float new_scale);

/* ── compute ─────────────────────────────────────────────────────────────── */
/* forward_dense(x), cpu_backend.cpp:475-492 -> disldo_forward
 * (linear_disldo.hpp:68-345).  Keeps x as the layer's last input. */
int sili_layer_forward_dense(sili_layer* h, const float* x, int batch, float* y, void* stream);
/* forward_dense without any allocation.  No counterpart in the reference:
 * for callers that cannot call cudaMalloc.  x [batch, n_in] and y
 * [batch, n_out] must be device pointers; the transposed-input scratch (plus
 * one zero row) is a fixed per-device array of SILI_STATIC_FWD_MAX_ELEMS
 * floats (4 MiB), so batch * (n_in + 1) above that is rejected with
 * SILI_EINVAL.  The column index
 * must be current (one forward_dense after load_weights or a structural
 * change), else SILI_EINVAL; so must the block4 tile index when the layer
 * holds block4 tiles (their part is added as forward_dense adds it).  The
 * scattered part always runs the per-synapse gather kernels, never the
 * row-tiled one forward_dense picks for wide rank-1 layers (its packed
 * column index is a rebuildable buffer), so on wide layers this entry point
 * is slower than forward_dense; results are equal.  Does not keep x for
 * backward_dense.  The first
 * call on a device looks up the scratch address (cudaGetSymbolAddress); make
 * it before work that must see only launches.  Calls on one device share the
 * scratch: overlapping calls race, so order them (one stream). */
#define SILI_STATIC_FWD_MAX_ELEMS 1048576
int sili_layer_forward_dense_static(sili_layer* h, const float* x, int batch, float* y, void* stream);
/* backward_dense(dy, lr, lr_per_row_nnz, damp_by_importance, beta2, eps),
 * cpu_backend.cpp:496-529 -> disldo_backward (linear_disldo.hpp:462-2113)
 * with beta1 0.9, min_decay_frac 0, max_abs_delta 2, max_ci 100.
 * x = NULL uses the last forward input. */
int sili_layer_backward_dense(sili_layer* h, const float* x, const float* dy, int batch, float lr,
                              unsigned flags, float beta2, float eps, float* dx, void* stream);
/* forward_sparse(ptrs, indices, values, batch), cpu_backend.cpp:571-585
 * -> sisldo_forward (sisldo_ops.hpp:198-551) */
int sili_layer_forward_sparse(sili_layer* h, const int* ptrs, const int* idx, const float* vals,
                              int nnz, int batch, float* y, void* stream);
/* backward_sparse(x, dy_ptrs, dy_indices, dy_values, batch, lr, ...),
 * cpu_backend.cpp:587-603 -> disldo_backward_sparse_grad (sisldo_ops.hpp:589-1104) */
int sili_layer_backward_sparse(sili_layer* h, const float* x, const int* dptrs, const int* didx,
                               const float* dvals, int dnnz, int batch, float lr, unsigned flags,
                               float beta2, float eps, float* dx, void* stream);

/* ── synaptogenesis and headroom management ─────────────────────────────── */
/* build_probes(k, per_row), cpu_backend.cpp:607-610 -> delta_csr_build_probes
 * (delta_csr_memory.hpp:1308-1427) */
int sili_layer_build_probes(sili_layer* h, int k, int per_row);
int sili_layer_num_probes(sili_layer* h, int64_t* n);
int sili_layer_get_probes(sili_layer* h, int* rows, int* cols, float* scores);
/* synap_row_step over the sweep rows (row0 + i) % n_in, i = 0..nrows-1,
 * cpu_backend.cpp:611-635 -> delta_csr_synap_row_step
 * (delta_csr_memory.hpp:1019-1258, with block4 promotion / demotion) once per
 * row in sweep order; the result equals nrows calls of the reference's
 * synap_row_step.  did (may be NULL; host or device, nrows bytes) receives
 * each step's return value.  A row that runs out of blank space stops the
 * sweep there with SILI_EHEADROOM (the reference's runtime_error), rows
 * before it done, that row partly done as the reference leaves it; a block4
 * budget overrun gives SILI_ENOMEM the same way. */
int sili_layer_synap_rows(sili_layer* h, int row0, int nrows, float importance_cutoff,
                          int max_row_weights, int max_prune_per_step, float importance_eps,
                          uint8_t* did);
/* equalizer_step() for one row, cpu_backend.cpp:649-657 -> delta_csr_equalize_step */
int sili_layer_equalize_row(sili_layer* h, int row);
/* equalize_to_capacity, cpu_backend.cpp:684-729 */
int sili_layer_equalize_to_capacity(sili_layer* h, int target_elems_per_row, int target_bytes_per_row);
/* compact / expand_headroom / expand_headroom_to, cpu_backend.cpp:737-785 */
int sili_layer_compact(sili_layer* h);
int sili_layer_expand_headroom(sili_layer* h, float blank_fraction);
int sili_layer_expand_headroom_to(sili_layer* h, int min_nnz_per_row, float blank_fraction);
/* zero_accum(), cpu_backend.cpp:851-854 */
int sili_layer_zero_accum(sili_layer* h);
/* the top-k growth rule (no reference function): exact top-k of
 * |sum_b x[b,r]*dy[b,c]| over non-existing (r,c), prune the same number of
 * smallest |FP4(w)*S(r,c)|, rebuild the arrays.  x [batch,n_in], dy [batch,n_out]. */
int sili_layer_topk_dyx_step(sili_layer* h, const float* x, const float* dy, int batch, int64_t k,
                             void* stream);

/* ── state export (cpu_backend.cpp:946-983, 1667-1738) ──────────────────── */
/* sizes[0..5] = n_in, n_out, nnz, index bytes, value bytes, block4 tiles */
int sili_layer_sizes(sili_layer* h, int64_t* sizes);
/* absolute CSR of the live synapses: ptrs[n_in+1], idx[nnz], weights
 * (stored FP4 units), importance (stored FP4 units) -- any may be NULL */
int sili_layer_export(sili_layer* h, int* ptrs, int* idx, float* w, float* imp);
/* raw delta-CSR state: byte_start[n_in+1], byte_end[n_in], elem_start[n_in+1],
 * elem_end[n_in] (int64), indices bytes, value bytes -- any may be NULL */
int sili_layer_raw(sili_layer* h, int64_t* byte_start, int64_t* byte_end, int64_t* elem_start,
                   int64_t* elem_end, uint8_t* indices, uint8_t* values);
/* overwrite the stored value bytes (weight code << 4 | importance code) */
int sili_layer_set_value_bytes(sili_layer* h, const uint8_t* values, int64_t n);
/* Checkpoint image: the layer's whole training state in one flat buffer
 * (host or device memory), written by one copy per state array.  It holds
 * what the reference's state dict (sili/sparse_rnn.py:817-851: weights,
 * value_scale, importance_scale) holds and what it cannot restore: the
 * importance codes, the delta-CSR layout with its headroom, every scale
 * optimiser vector and step counter, the accumulators, out_degree, the
 * running statistics and the stochastic-rounding seed and call counter, so a
 * layer loaded from it continues training bit for bit.  load_state needs a
 * layer of the same n_inputs x n_outputs (its scale rank follows the image)
 * and drops the last forward input.  Layers holding block4 tiles:
 * SILI_EINVAL. */
int sili_layer_state_size(sili_layer* h, int64_t* bytes);
int sili_layer_save_state(sili_layer* h, void* buf, int64_t bytes, void* stream);
int sili_layer_load_state(sili_layer* h, const void* buf, int64_t bytes, void* stream);
int sili_layer_accums(sili_layer* h, float* input_accum, float* grad_accum);
int sili_layer_set_accums(sili_layer* h, const float* input_accum, const float* grad_accum);
int sili_layer_out_degree(sili_layer* h, int* out);
/* stats[0..5] = value_l1, value_l2_sq, value_max_abs, importance_l1,
 * importance_l2_sq, importance_max_abs (delta_csr_types.hpp:1265-1270) */
int sili_layer_stats(sili_layer* h, double* stats);
int sili_layer_recompute_stats(sili_layer* h);
/* last forward input [batch, n_in] (NULL out -> only batch/cols) */
int sili_layer_last_input(sili_layer* h, float* out, int* batch, int* cols);
/* the last forward_sparse input as a dense [batch, n_in] array (NULL out ->
 * only batch/cols).  No reference counterpart: the reference's SISLDOLayer
 * (sili/sparse_rnn.py:764-810) hands backward_sparse the layer's last_input,
 * meaning the dense form of its forward_sparse input, which the reference's
 * module never stores; the pybind layer passes this one for x = None. */
int sili_layer_last_sparse_input(sili_layer* h, float* out, int* batch, int* cols);

/* ── block4 tiles (4x4 dense FP4 tiles beside the scattered synapses) ───── */
/* synapses in the combined export (scattered + live block4 slots) -- the
 * reference's nnz(), cpu_backend.cpp:451 */
int sili_layer_export_nnz(sili_layer* h, int64_t* n);
/* load_dense_codes(weight_codes, importance_codes), cpu_backend.cpp:910-921 ->
 * block4_load_dense (delta_csr_memory.hpp:843-945): u8 [n_in, n_out] codes
 * each, host or device */
int sili_layer_load_dense_codes(sili_layer* h, const uint8_t* weight_codes, const uint8_t* importance_codes);
/* expand_block4_headroom(blank_fraction) / compact_block4 (min_slack 16 / 0,
 * blank 0), cpu_backend.cpp:932-942 -> block4_expand_headroom
 * (delta_csr_memory.hpp:769-823) */
int sili_layer_b4_expand_headroom(sili_layer* h, float blank_fraction, int64_t min_slack);
/* the block4 half of equalizer_step (Block4Store::equalize_step,
 * block4.hpp:1208-1221); row is the block-row cursor */
int sili_layer_b4_equalize_row(sili_layer* h, int64_t row);
/* The block4 forward and lr = 0 dx on the tensor cores (no counterpart in
 * the reference, whose block4 forward is linear_disldo.hpp:128-339 and
 * block4 dx :1512-1703): enable = 1 runs the block4 part of forward_dense,
 * and of backward_dense's dx at learning_rate 0, for rank-1 layers at batch
 * >= 16 as tcgen05 MMAs (FP4 codes exact in bf16, x * value_scale or
 * dy * output_scale split into three bf16 terms, fp32 accumulation) --
 * within fp32 summation tolerance of the exact CUDA-core path, which is the
 * default (enable = 0).  A bounded
 * device-side wait that gives up is reported as SILI_ETIMEOUT by the next
 * synchronising call (sili_layer_sync, or a forward with host arrays). */
int sili_layer_set_b4_tensor_cores(sili_layer* h, int enable);

/* The layer's scale policy, the ScalePolicy template argument of the
 * reference's classes (cpu_backend.cpp:993-1013):
 *   SILI_SCALE_POLICY_RMSPROP  SparseLinearLayer{,Deterministic} (default)
 *   SILI_SCALE_POLICY_NONE     SparseLinearLayerNoScale{,Deterministic}:
 *                              NoScalePolicy (delta_csr_types.hpp:528-537),
 *                              whose update does nothing -- the dense
 *                              backward's value_scale step
 *                              (linear_disldo.hpp:901-925) and output_scale
 *                              step (:2051-2080) are skipped, their step
 *                              counters and importance states untouched; the
 *                              block4 value_scale step, the dead-row
 *                              bootstrap and the sparse-gradient backward's
 *                              steps, written inline in the reference rather
 *                              than through the policy, still run.
 *   SILI_SCALE_POLICY_RESYNC   SparseLinearLayerResync{,Deterministic}:
 *                              RMSpropScalePolicy with DeferredScaleWrite
 *                              (linear_disldo.hpp:686-790, 918-923,
 *                              2083-2112): the scattered update runs the old
 *                              true-units step, its component-0 scale sums
 *                              come from the stored code, and the new codes
 *                              are stored after the value_scale and
 *                              output_scale steps, under the final scales.
 *                              Here: scale rank 1 (set_scale_rank(k > 1)
 *                              and this call at rank > 1 give SILI_EINVAL)
 *                              and batches of at most 128 for a learning
 *                              rate != 0; not column-sharded.
 * The stochastic / deterministic rounding choice stays with
 * sili_layer_create. */
#define SILI_SCALE_POLICY_RMSPROP 0
#define SILI_SCALE_POLICY_NONE 1
#define SILI_SCALE_POLICY_RESYNC 2
int sili_layer_set_scale_policy(sili_layer* h, int policy);
/* Block4View.switch_point setter (cpu_backend.cpp:61-62) */
int sili_layer_b4_set_switch_point(sili_layer* h, uint32_t v);
/* Block4View counters, cpu_backend.cpp:51-98: tiles, synapses, switch_point,
 * dropped_growth_events, row_merge_overflow_events,
 * row_merge_overflow_bytes_dropped, used_bytes, alloc_bytes */
int sili_layer_b4_view(sili_layer* h, int64_t* v8);
/* live tiles in block-row order: block-row, block-column, 16 slot bytes
 * (slot = lj*4 + li, byte = importance << 4 | weight), packed flag;
 * sizes[5] of sili_layer_sizes is the tile count */
int sili_layer_b4_export(sili_layer* h, int* br, int* bc, uint8_t* slots, uint8_t* sparse);
/* per block-row: index-byte alloc, index bytes used, tile-byte alloc, tile
 * bytes used, tile-slot alloc, tiles (the reference's Block4Store layout) */
int sili_layer_b4_rows(sili_layer* h, int64_t* out6);

/* ── folded stacks ─────────────────────────────────────────────────────── */
/* FoldedLayer's fold sum (sili/sparse_rnn.py:1120-1125) on device arrays:
 * y[b, j] = sum over folds f ascending of raw[b, f*out_dim + j] */
int sili_fold_sum(const float* raw, int batch, int n_folds, int64_t out_dim, float* y, void* stream);
/* FoldedLayer.forward (sili/sparse_rnn.py:1096-1125) in one call: every
 * suffix layer (each n_in -> n_folds * out_dim, one device) on the same x
 * [batch, n_in], their outputs summed in suffix order and, with fold_sum,
 * the folds summed: y [batch, out_dim]; without fold_sum (FoldedColumnLayer.
 * in_proj, :1340-1362) y is the suffix sum [batch, n_folds * out_dim].  One
 * transposed copy of x serves every layer and stays each layer's last input
 * (backward_dense works as after forward_dense).  Two to four rank-1 suffix
 * layers without block4 tiles, at batch >= 16 and a multiple of 4, run as
 * one kernel launch that sums in shared memory; a single suffix runs its
 * layer's forward and the fold sum (two launches, measured faster).  Host or
 * device x / y. */
int sili_folded_forward(sili_layer* const* layers, int n_layers, const float* x, int batch, int n_folds,
                        int64_t out_dim, int fold_sum, float* y, void* stream);
/* The backward of the fold sum for one rank's column slice (the np.tile of
 * FoldedLayer's backward, sili/sparse_rnn.py:1144-1148, restricted to output
 * columns [j0, j0 + width)): raw[b, f*width + j] = dy[b, j0 + j], dy being
 * [batch, out_dim] and raw [batch, n_folds * width]; device arrays. */
int sili_fold_broadcast(const float* dy, int batch, int64_t out_dim, int64_t j0, int64_t width, int n_folds,
                        float* raw, void* stream);

/* Column shards of one layer.  A folded stack split by output column over
 * ranks gives each rank every row of the stack but only some columns.  The
 * synapse updates of disldo_backward (linear_disldo.hpp:790-925) are local
 * to their (row, column); three things couple a row's columns: the
 * learning rate lr / nnz_row, the row's value_scale step from sums over all
 * its synapses (:901-925) and the dead-row bootstrap from sums over all
 * columns (:1985-2042).  After sili_layer_set_row_shard(global synapse count
 * per row, global column count) a shard's backward is
 *   sili_layer_backward_dense_shard(...)  -> partial dx over its columns and
 *                                            `part` (its part of the row sums)
 *   sum dx and part over the ranks (e.g. two NCCL all-reduces)
 *   sili_layer_apply_row_part(summed part) -> the row steps, same on every rank
 * so every rank's value_scale stays equal to the unsharded layer's (up to
 * the order of the double sums).  part holds sili_layer_row_part_len
 * doubles: (value-gradient, contribution) sums per (row, rank-k), then the
 * dead-row S[batch, rank].  Host or device part arrays; no other forward or
 * backward of the layer between the two calls.  Not for layers with block4
 * tiles (SILI_EINVAL).  n = 0 switches sharding off. */
int sili_layer_set_row_shard(sili_layer* h, const int* global_row_nnz, int64_t n, int64_t global_n_out);
int sili_layer_row_part_len(sili_layer* h, int batch, int64_t* n);
int sili_layer_backward_dense_shard(sili_layer* h, const float* x, const float* dy, int batch, float lr,
                                    unsigned flags, float beta2, float eps, float* dx, double* part,
                                    void* stream);
int sili_layer_apply_row_part(sili_layer* h, const double* part, void* stream);

/* ── module functions (cpu_backend.cpp:3075-3196) ───────────────────────── */
/* fp4_quantize_array: deterministic FP4 encode, fp4quant.hpp:86-121 */
int sili_fp4_quantize(const float* vals, uint8_t* codes, int64_t n, void* stream);
/* dense_to_csr(x, threshold): |v| > threshold, row-major.  Two-phase: call
 * with idx/vals NULL to get nnz in *nnz_out and ptrs, then again to fill. */
int sili_dense_to_csr(const float* x, int rows, int cols, float threshold, int* ptrs, int* idx,
                      float* vals, int64_t* nnz_out, void* stream);
/* dense_to_top_k_csr(x, k): global exact top-k by |v|, row-major CSR,
 * ascending columns; ties at the k-th magnitude go to the lower flat index. */
int sili_dense_to_top_k_csr(const float* x, int rows, int cols, int64_t k, int* ptrs, int* idx,
                            float* vals, void* stream);

/* csr_union(ptrs_a, idx_a, vals_a, ptrs_b, idx_b, vals_b, n_rows, prefer),
 * cpu_backend.cpp:3200-3238 -> csr_union (csr.hpp:505-580): per row the
 * two-pointer merge of A's and B's column lists; prefer 0 keeps A's value on
 * an overlap, 1 B's, 2 their sum (anything else: SILI_EINVAL).  Host or
 * device arrays.  Two-phase like sili_dense_to_csr: out_idx / out_vals NULL
 * gives out_ptrs[n_rows+1] and *nnz_out only. */
int sili_csr_union(const int* ptrs_a, const int* idx_a, const float* vals_a, const int* ptrs_b, const int* idx_b,
                   const float* vals_b, int n_rows, int prefer, int* out_ptrs, int* out_idx, float* out_vals,
                   int64_t* nnz_out, void* stream);

/* ── conversion-time CSR operations (device arrays) ─────────────────────
 * What the reference's conversion path does in torch / numpy on the host:
 * prune_to_csr     to_sparse_csr (sili/conversion/sparse_prune.py:466-482):
 *                  w [rows, cols] -> row-major CSR of the entries with
 *                  |w| >= min_abs and w != 0; two-phase (idx / vals NULL ->
 *                  ptrs and *nnz_out only)
 * csr_transpose    csr.t().to_sparse_csr() (sili/sparse_rnn.py:1002): rows
 *                  of the result ascend in column order
 * csr_stack_vertical  stack_csr_vertical (sili/conversion/rnn_fold.py:259-320):
 *                  parts [rows_p, cols] -> [sum rows_p, cols]; out_ptrs has
 *                  sum rows_p + 1 entries
 * fit_rank1_envelope  fit_rank1_scale_envelope (sili/sparse_rnn.py:854-882) on
 *                  the |vals| of a CSR, n_iters alternating max-fits
 * fp4_row_rescale  FoldedLayer.from_descriptor's FP4 preparation
 *                  (sili/sparse_rnn.py:1005-1037): mode 0 per_row (row_scale
 *                  out = max|row| / 6, 1 for empty / zero rows), mode 1 rank1
 *                  (row_scale in = the envelope's rows, out = them / 6);
 *                  vals divided in place */
int sili_prune_to_csr(const float* w, int64_t rows, int64_t cols, float min_abs, int* ptrs, int* idx, float* vals,
                      int64_t* nnz_out, void* stream);
int sili_csr_transpose(const int* ptrs, const int* idx, const float* vals, int n_rows, int n_cols, int* out_ptrs,
                       int* out_idx, float* out_vals, void* stream);
int sili_csr_stack_vertical(int n_parts, const int* const* ptrs, const int* const* idx, const float* const* vals,
                            const int* rows, int* out_ptrs, int* out_idx, float* out_vals, void* stream);
int sili_fit_rank1_envelope(const int* ptrs, const int* idx, const float* vals, int n_rows, int n_cols, int n_iters,
                            float* row_scale, float* col_scale, void* stream);
int sili_fp4_row_rescale(const int* ptrs, const int* idx, float* vals, int n_rows, int mode, const float* col_scale,
                         float* row_scale, void* stream);

/* ── attention (sili/lib/headers/attention.hpp) ────────────────────────── */
/* banded_attention_forward (:39-96) and, for inner_k > 0,
 * sparse_banded_attention_forward (:121-197; the inner_k band keys of largest
 * L2 norm, ties to the lower key) over `groups` query matrices [T, d] and
 * `kv_groups` key / value matrices [K, d] (query group g reads key group
 * g / (groups / kv_groups)); out [groups, T, d].  Host or device arrays.
 * The bindings banded_attention / sparse_banded_attention of
 * cpu_backend.cpp:3404-3443 are groups = kv_groups = 1.  d <= 256. */
int sili_banded_attention(const float* q, const float* k, const float* v, float* out, int64_t groups,
                          int64_t kv_groups, int64_t T, int64_t K, int64_t d, int64_t half_bandwidth,
                          int64_t inner_k, int causal, void* stream);
/* sparse_attention_forward (:228-333, binding cpu_backend.cpp:3384-3402):
 * q, k, v, out [T, d]; top_k = 0 -> floor(sqrt(T)); rows of unselected
 * queries are zero. */
int sili_sparse_attention(const float* q, const float* k, const float* v, float* out, int64_t T, int64_t d,
                          int64_t top_k, int causal, void* stream);
/* banded_attention_backward (:354-442, binding cpu_backend.cpp:3445-3468):
 * dQ [groups, T, d], dK / dV [kv_groups, K, d] (written, not accumulated). */
int sili_banded_attention_backward(const float* q, const float* k, const float* v, const float* dO, float* dQ,
                                   float* dK, float* dV, int64_t groups, int64_t kv_groups, int64_t T, int64_t K,
                                   int64_t d, int64_t half_bandwidth, int causal, void* stream);

#ifdef __cplusplus
}
#endif
#endif
