/* CPU restatement of sili's FP4 delta-CSR sparse-layer path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path, never the
 * product.  See sili_oracle.h for the contract.  Reference citations are
 * file:line within the reference project (sili/...).
 *
 * The restatement follows the reference's num_cpus == 1 evaluation order
 * (rows ascending, synapses in stored order, batch samples ascending), so its
 * float sums are the reference's single-thread sums.
 */
#include "sili_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ── small vectors with the reference's lazy-resize semantics ───────────── */
typedef struct { float* d; int64_t n; } fvec;
typedef struct { uint32_t* d; int64_t n; } uvec;

static void fvec_resize(fvec* v, int64_t n, float fill) {
    if (n <= v->n) { v->n = n; return; }
    v->d = (float*)realloc(v->d, (size_t)n * sizeof(float));
    for (int64_t i = v->n; i < n; ++i) v->d[i] = fill;
    v->n = n;
}
static void uvec_resize(uvec* v, int64_t n, uint32_t fill) {
    if (n <= v->n) { v->n = n; return; }
    v->d = (uint32_t*)realloc(v->d, (size_t)n * sizeof(uint32_t));
    for (int64_t i = v->n; i < n; ++i) v->d[i] = fill;
    v->n = n;
}

struct OLayer {
    int64_t rows, cols;
    /* DeltaCSRLayout, delta_csr_types.hpp:763-797 */
    int64_t *byte_start, *byte_end, *elem_start, *elem_end;
    uint8_t* idx; int64_t idx_n;      /* indices_buf, size = byte_start[rows] */
    uint8_t* val; int64_t val_n;      /* FP4BiPacked bytes, size = elem_start[rows] */
    int64_t total_nnz;
    int64_t max_idx_bytes, max_val_bytes;   /* DeltaCSRWeights::set_limits */
    int64_t idx_budget, val_budget;         /* cpu_backend.cpp:372-378 */
    int rank;
    fvec value_scale, value_scale_importance, value_scale_momentum;
    fvec output_scale, output_scale_importance;
    fvec importance_scale, output_importance_scale;
    uvec value_scale_step, output_scale_step;
    int output_scale_trainable;
    float *in_acc, *grad_acc;
    int* out_degree;
    int64_t n_probes; int *prow, *pcol; float* pval;
    double importance_l1, importance_l2_sq, value_l1, value_l2_sq;
    float importance_max_abs, value_max_abs, max_abs_decay;
    int stochastic; uint64_t seed; uint64_t call;
    int scale_noop;   /* NoScalePolicy (delta_csr_types.hpp:528-537): ScalePolicy::update does nothing */
    int resync;       /* DeferredScaleWrite = true (SparseLinearLayerResync{,Deterministic}) */
    /* block4 store (block4.hpp:1016-1490): per block-row tile lists plus the
     * reference's per-block-row allocations (index bytes, tile bytes, tile
     * slots), which decide headroom growth, eviction and budget errors. */
    int64_t b4_rows, b4_cols;
    struct OTileRow* b4;
    int64_t *b4_idx_alloc, *b4_tile_alloc, *b4_elem_alloc;
    int64_t b4_max_idx, b4_max_tile;
    uint32_t b4_switch;
    uint64_t b4_dropped, b4_ovf_events, b4_ovf_bytes;
    /* stochastic draws of the sparse-gradient block4 update: 0 = counter
     * draws (o_rng_draw, the CUDA path's), 1 = the reference's xorshift64*
     * stream (fp4quant.hpp:170-190) for pinning against its build */
    int ref_stream; uint64_t ref_state;
    /* column-sharded rows (a layer holding some of the columns of every
     * row): global synapse count per row and the global column count; during
     * o_backward_dense_shard the row-scale sums go to shard_part instead of
     * being applied */
    int* shard_nnz; int64_t shard_n_out; double* shard_part;
};

#define NO_LIMIT INT64_MAX

/* block4 store, defined with the block4 section near the end of the file */
static void b4_init(OLayer* L);
static void b4_free(OLayer* L);
static void b4_forward(const OLayer* L, const float* x, int batch, float* y);
static void b4_backward(OLayer* L, const float* x, const float* dy, int batch, float lr, int lr_per_row_nnz,
                        int damp, float beta2, float eps, float* dx, float* colg, float* colc, uint64_t call);
static int64_t b4_row_live(const OLayer* L, int64_t row);
typedef int (*o_less_fn)(int64_t a, int64_t b, const void* ctx);
void o_std_sort(int64_t* a, int64_t n, o_less_fn lt, const void* c);
int64_t o_b4_ntiles(const OLayer* L);
/* a block4 tile: block-column, 16 slot bytes (slot = lj*4 + li,
 * Block4Tile::slot_index, block4.hpp:309), sparse-packed flag */
typedef struct OTile { int32_t bc; uint8_t s[16]; uint8_t sparse; } OTile;
struct OTileRow { OTile* t; int64_t n, cap; };
#define B4_SLOT(li, lj) ((lj) * 4 + (li))

/* ── codec: fp4quant.hpp ─────────────────────────────────────────────────── */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp4_decode_bits, fp4quant.hpp:68-84; equals FP4_TABLE (code 8 = NaN). */
float o_fp4_decode(uint8_t code) {
    const uint32_t s = (code >> 3) & 1u, e = (code >> 1) & 3u, m = code & 1u;
    uint32_t bits;
    if (e == 0) bits = m ? (0x3F000000u | (s << 31)) : (s ? 0x7FC00000u : 0u);
    else bits = (s << 31) | ((e + 126u) << 23) | (m << 22);
    return u2f(bits);
}

/* fp4_encode_bits, fp4quant.hpp:86-121. */
uint8_t o_fp4_encode(float v) {
    const uint32_t bits = f2u(v), sign = bits & 0x80000000u, a = bits & 0x7FFFFFFFu;
    uint32_t mag;
    if (a > 0x7F800000u) return 0;
    else if (a < 0x3E800000u) mag = 0;
    else if (a < 0x3F400000u) mag = 1;
    else if (a < 0x3F800000u) mag = 2;
    else {
        uint32_t r = a + (1u << 21);
        if (r > 0x40C00000u) r = 0x40C00000u;
        mag = ((((r >> 23) & 0xFFu) - 126u) << 1) | ((r >> 22) & 1u);
    }
    if (mag == 0) return 0;
    return (uint8_t)(((sign ? 1u : 0u) << 3) | mag);
}

/* fp4_quantize_stochastic, fp4quant.hpp:238-273, with the 64-bit draw passed in
 * (the reference takes it from its thread-local xorshift64*). */
uint8_t o_fp4_quantize_stochastic_r(float v, uint64_t r) {
    const uint32_t bits = f2u(v), sign = bits & 0x80000000u, a = bits & 0x7FFFFFFFu;
    uint32_t mag;
    if (a > 0x7F800000u) return 0;
    if (a >= 0x40C00000u) mag = 7;
    else if (a < 0x3F000000u) {
        const float p = u2f(a) * 2.0f;
        const float u = (float)((double)(r >> 40) * (1.0 / 16777216.0));
        mag = (u < p) ? 1u : 0u;
    } else if (a < 0x3F800000u) {
        const float p = u2f(a) * 2.0f - 1.0f;
        const float u = (float)((double)(r >> 40) * (1.0 / 16777216.0));
        mag = (u < p) ? 2u : 1u;
    } else {
        uint32_t rr = a + (uint32_t)(r & 0x3FFFFFu);
        if (rr > 0x40C00000u) rr = 0x40C00000u;
        mag = ((((rr >> 23) & 0xFFu) - 126u) << 1) | ((rr >> 22) & 1u);
    }
    if (mag == 0) return 0;
    return (uint8_t)(((sign ? 1u : 0u) << 3) | mag);
}

/* The reference's stream generator (xorshift64*, fp4quant.hpp:196-200). */
uint64_t o_xorshift_next(uint64_t* s) {
    *s ^= *s >> 12; *s ^= *s << 25; *s ^= *s >> 27;
    return *s * 0x2545F4914F6CDD1DULL;
}

/* Counter-based draw used by this build's stochastic rounding (GPU and this
 * oracle alike): splitmix64's finaliser applied twice over (seed, call,
 * element, lane).  The reference draws from a per-thread xorshift64* stream
 * instead, so stochastic parity with the reference is statistical. */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
uint64_t o_rng_draw(uint64_t seed, uint64_t call, uint64_t elem, uint32_t lane) {
    uint64_t k = mix64(seed ^ (call * 0x9E3779B97F4A7C15ULL));
    return mix64(k ^ (elem * 2u + lane) * 0xD1B54A32D192ED03ULL);
}

/* ── ULEB128, delta_csr_types.hpp:211-241 ───────────────────────────────── */
static int uleb_len(uint32_t v) { int n = 0; do { v >>= 7; ++n; } while (v); return n; }
static int uleb_put(uint32_t v, uint8_t* buf) {
    int n = 0;
    do { uint8_t b = (uint8_t)(v & 0x7Fu); v >>= 7; if (v) b |= 0x80u; buf[n++] = b; } while (v);
    return n;
}
static uint32_t uleb_get(const uint8_t* buf, int64_t* pos) {
    uint32_t r = 0; int sh = 0; uint8_t b;
    do { b = buf[(*pos)++]; r |= (uint32_t)(b & 0x7Fu) << sh; sh += 7; } while (b & 0x80u);
    return r;
}

/* ── lazy scale accessors, delta_csr_types.hpp:1006-1240 ────────────────── */
float o_get_importance_scale(const OLayer* L, int row) {
    return row < L->importance_scale.n ? L->importance_scale.d[row] : 1.0f;
}
float o_get_output_importance_scale(const OLayer* L, int col) {
    return col < L->output_importance_scale.n ? L->output_importance_scale.d[col] : 1.0f;
}
float o_get_value_scale_k(const OLayer* L, int row, int k) {
    const int64_t i = (int64_t)row * L->rank + k;
    if (i < L->value_scale.n) return L->value_scale.d[i];
    return k == 0 ? 1.0f : 0.0f;
}
float o_get_output_scale_k(const OLayer* L, int col, int k) {
    const int64_t i = (int64_t)col * L->rank + k;
    if (i < L->output_scale.n) return L->output_scale.d[i];
    return k == 0 ? 1.0f : 0.0f;
}
float o_get_value_scale_importance_k(const OLayer* L, int row, int k) {
    const int64_t i = (int64_t)row * L->rank + k;
    return i < L->value_scale_importance.n ? L->value_scale_importance.d[i] : 0.0f;
}
float o_get_output_scale_importance_k(const OLayer* L, int col, int k) {
    const int64_t i = (int64_t)col * L->rank + k;
    return i < L->output_scale_importance.n ? L->output_scale_importance.d[i] : 0.0f;
}
float o_get_value_scale_momentum_k(const OLayer* L, int row, int k) {
    const int64_t i = (int64_t)row * L->rank + k;
    return i < L->value_scale_momentum.n ? L->value_scale_momentum.d[i] : 0.0f;
}
uint32_t o_get_value_scale_step_k(const OLayer* L, int row, int k) {
    const int64_t i = (int64_t)row * L->rank + k;
    return i < L->value_scale_step.n ? L->value_scale_step.d[i] : 0u;
}
uint32_t o_get_output_scale_step_k(const OLayer* L, int col, int k) {
    const int64_t i = (int64_t)col * L->rank + k;
    return i < L->output_scale_step.n ? L->output_scale_step.d[i] : 0u;
}
/* get_scale, delta_csr_types.hpp:1235-1240 */
float o_get_scale(const OLayer* L, int row, int col) {
    float s = 0.0f;
    for (int k = 0; k < L->rank; ++k) s = fmaf(o_get_value_scale_k(L, row, k), o_get_output_scale_k(L, col, k), s);
    return s;
}
void o_set_value_scale_raw_k(OLayer* L, int row, int k, float v) {
    const int64_t i = (int64_t)row * L->rank + k;
    if (i >= L->value_scale.n) fvec_resize(&L->value_scale, i + 1, 1.0f);
    L->value_scale.d[i] = v;
}
void o_set_output_scale_raw_k(OLayer* L, int col, int k, float v) {
    const int64_t i = (int64_t)col * L->rank + k;
    if (i >= L->output_scale.n) fvec_resize(&L->output_scale, i + 1, 1.0f);
    L->output_scale.d[i] = v;
    L->output_scale_trainable = 1;
}
void o_set_importance_scale_raw(OLayer* L, int row, float v) {
    if (row >= L->importance_scale.n) fvec_resize(&L->importance_scale, row + 1, 1.0f);
    L->importance_scale.d[row] = v;
}
void o_set_output_importance_scale_raw(OLayer* L, int col, float v) {
    if (col >= L->output_importance_scale.n) fvec_resize(&L->output_importance_scale, col + 1, 1.0f);
    L->output_importance_scale.d[col] = v;
}
/* cpu_backend.cpp:466-471 */
int o_set_scale_rank(OLayer* L, int rank) {
    if (rank < 1 || rank > 4) return O_EINVAL;
    L->rank = rank;
    return O_OK;
}
int o_get_scale_rank(const OLayer* L) { return L->rank; }
int o_output_scale_trainable(const OLayer* L) { return L->output_scale_trainable; }

/* ── layout helpers ──────────────────────────────────────────────────────── */
static inline int64_t row_nnz(const OLayer* L, int64_t r) { return L->elem_end[r] - L->elem_start[r]; }
static inline float get_w(const OLayer* L, int64_t vb) { return o_fp4_decode((uint8_t)(L->val[vb] >> 4)); }
static inline float get_imp(const OLayer* L, int64_t vb) { return o_fp4_decode((uint8_t)(L->val[vb] & 0xF)); }
/* ValueAccessor<FP4BiPacked>::set, delta_csr_types.hpp:252-255 */
static inline void set_wi(OLayer* L, int64_t vb, float w, float imp) {
    L->val[vb] = (uint8_t)((o_fp4_encode(w) << 4) | o_fp4_encode(imp));
}

static void free_layout(OLayer* L) {
    free(L->byte_start); free(L->byte_end); free(L->elem_start); free(L->elem_end);
    free(L->idx); free(L->val);
    L->byte_start = L->byte_end = L->elem_start = L->elem_end = NULL;
    L->idx = L->val = NULL;
}

/* delta_csr_from_absolute, delta_csr_memory.hpp:16-93.  Builds a fresh layout
 * into L (replacing the old one).  index_bytes/values_bytes are the reserve
 * requests, checked against the hard limits like reserve_indices/values. */
static int from_absolute(OLayer* L, const int* ptrs, const int* idx, const float* w, const float* imp,
                         int64_t rows, int64_t cols, int64_t index_bytes, int64_t values_bytes,
                         float bf, int64_t hard_idx, int64_t hard_val) {
    if (values_bytes > hard_val) return O_ENOMEM;
    if (index_bytes > hard_idx) return O_ENOMEM;
    int64_t* bs = (int64_t*)calloc((size_t)rows + 1, 8);
    int64_t* be = (int64_t*)calloc((size_t)rows + 1, 8);
    int64_t* es = (int64_t*)calloc((size_t)rows + 1, 8);
    int64_t* ee = (int64_t*)calloc((size_t)rows + 1, 8);
    for (int64_t r = 0; r < rows; ++r) {
        int64_t nb = 0; uint32_t prev = 0;
        for (int i = ptrs[r]; i < ptrs[r + 1]; ++i) { nb += uleb_len((uint32_t)idx[i] - prev); prev = (uint32_t)idx[i]; }
        const int64_t n = ptrs[r + 1] - ptrs[r];
        be[r] = bs[r] + nb;
        const int64_t byte_blank = (int64_t)((float)nb * bf) + 5;
        bs[r + 1] = be[r] + byte_blank;
        ee[r] = es[r] + n;
        int64_t eb = (int64_t)((float)n * bf) + 1;
        if (eb < 1) eb = 1;
        es[r + 1] = ee[r] + eb;
    }
    uint8_t* ib = (uint8_t*)calloc((size_t)bs[rows] + 16, 1);
    uint8_t* vb = (uint8_t*)calloc((size_t)es[rows] + 16, 1);
    for (int64_t r = 0; r < rows; ++r) {
        int64_t bp = bs[r], ep = es[r]; uint32_t prev = 0;
        for (int i = ptrs[r]; i < ptrs[r + 1]; ++i) {
            bp += uleb_put((uint32_t)idx[i] - prev, ib + bp);
            prev = (uint32_t)idx[i];
            vb[ep++] = (uint8_t)((o_fp4_encode(w[i]) << 4) | o_fp4_encode(imp[i]));
        }
    }
    free_layout(L);
    L->rows = rows; L->cols = cols;
    L->byte_start = bs; L->byte_end = be; L->elem_start = es; L->elem_end = ee;
    L->idx = ib; L->idx_n = bs[rows];
    L->val = vb; L->val_n = es[rows];
    L->total_nnz = ptrs[rows];
    L->max_idx_bytes = hard_idx; L->max_val_bytes = hard_val;
    return O_OK;
}

/* recompute_stats, delta_csr_types.hpp:1350-1364 (update_*_stats :1306-1315) */
void o_recompute_stats(OLayer* L) {
    L->importance_l1 = L->importance_l2_sq = L->value_l1 = L->value_l2_sq = 0.0;
    L->importance_max_abs = L->value_max_abs = 0.0f;
    for (int64_t r = 0; r < L->rows; ++r)
        for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
            const float w = get_w(L, vb), im = get_imp(L, vb);
            L->value_l1 += fabs((double)w) - 0.0;
            L->value_l2_sq += (double)w * w - 0.0;
            L->value_max_abs = fmaxf(L->value_max_abs * L->max_abs_decay, fabsf(w));
            L->importance_l1 += fabs((double)im) - 0.0;
            L->importance_l2_sq += (double)im * im - 0.0;
            L->importance_max_abs = fmaxf(L->importance_max_abs * L->max_abs_decay, fabsf(im));
        }
}

/* SparseLinearLayerImpl constructor, cpu_backend.cpp:375-447 */
OLayer* o_create(int n_in, int n_out, int max_weights) {
    OLayer* L = (OLayer*)calloc(1, sizeof(OLayer));
    L->rank = 1; L->max_abs_decay = 1.0f;
    L->idx_budget = (int64_t)max_weights * 8 + 4096;
    L->val_budget = (int64_t)max_weights + 64;
    int* p = (int*)calloc((size_t)n_in + 1, sizeof(int));
    from_absolute(L, p, NULL, NULL, NULL, n_in, n_out, L->idx_budget, L->val_budget, 0.2f, NO_LIMIT, NO_LIMIT);
    free(p);
    L->max_idx_bytes = L->idx_budget; L->max_val_bytes = L->val_budget;
    o_recompute_stats(L);
    L->in_acc = (float*)calloc((size_t)n_in + 1, sizeof(float));
    L->grad_acc = (float*)calloc((size_t)n_out + 1, sizeof(float));
    L->out_degree = (int*)calloc((size_t)n_out + 1, sizeof(int));
    b4_init(L);
    L->b4_max_idx = (int64_t)max_weights * 8 + 4096;
    L->b4_max_tile = ((int64_t)max_weights / 16 > 4 ? (int64_t)max_weights / 16 : 4) * 16;
    L->b4_switch = 10;
    return L;
}

void o_destroy(OLayer* L) {
    if (!L) return;
    free_layout(L);
    free(L->value_scale.d); free(L->value_scale_importance.d); free(L->value_scale_momentum.d);
    free(L->output_scale.d); free(L->output_scale_importance.d);
    free(L->importance_scale.d); free(L->output_importance_scale.d);
    free(L->value_scale_step.d); free(L->output_scale_step.d);
    free(L->in_acc); free(L->grad_acc); free(L->out_degree);
    free(L->prow); free(L->pcol); free(L->pval);
    free(L->shard_nnz);
    b4_free(L);
    free(L);
}

/* load_weights, cpu_backend.cpp:859-901 */
int o_load_weights(OLayer* L, const int* ptrs, const int* idx, const float* vals, int nnz) {
    float* imp = (float*)calloc((size_t)nnz + 1, sizeof(float));
    int64_t ib = (int64_t)nnz * 8 + 4096, vb = (int64_t)nnz + 64;
    if (ib < L->idx_budget) ib = L->idx_budget;
    if (vb < L->val_budget) vb = L->val_budget;
    const int rc = from_absolute(L, ptrs, idx, vals, imp, L->rows, L->cols, ib, vb, 0.2f, NO_LIMIT, NO_LIMIT);
    free(imp);
    if (rc) return rc;
    L->idx_budget = ib; L->val_budget = vb;
    L->max_idx_bytes = ib; L->max_val_bytes = vb;
    o_recompute_stats(L);
    memset(L->out_degree, 0, (size_t)L->cols * sizeof(int));
    for (int i = 0; i < nnz; ++i) L->out_degree[idx[i]]++;
    return O_OK;
}

void o_set_value_bytes(OLayer* L, const uint8_t* bytes, int64_t n) {
    for (int64_t i = 0; i < n && i < L->val_n; ++i) L->val[i] = bytes[i];
}
void o_set_stochastic(OLayer* L, int stochastic, uint64_t seed) { L->stochastic = stochastic; L->seed = seed; L->call = 0; }
/* 0: RMSpropScalePolicy (SparseLinearLayer{,Deterministic}), 1: NoScalePolicy
 * (SparseLinearLayerNoScale{,Deterministic}, cpu_backend.cpp:998, 1013),
 * 2: RMSpropScalePolicy with DeferredScaleWrite (SparseLinearLayerResync
 * {,Deterministic}, :993, :1012) */
void o_set_scale_policy(OLayer* L, int policy) { L->scale_noop = policy == 1; L->resync = policy == 2; }

/* ── forward, linear_disldo.hpp:68-126 (scattered part) ─────────────────── */
void o_forward_dense(OLayer* L, const float* x, int batch, float* y) {
    const int64_t n_out = L->cols, n_in = L->rows;
    memset(y, 0, (size_t)batch * n_out * sizeof(float));
    for (int64_t r = 0; r < n_in; ++r) {
        int64_t pos = L->byte_start[r]; uint32_t col = 0;
        for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
            col += uleb_get(L->idx, &pos);
            const float w = get_w(L, vb) * o_get_scale(L, (int)r, (int)col);
            for (int b = 0; b < batch; ++b) {
                const float iv = x[(int64_t)b * n_in + r];
                if (iv == 0.0f) continue;
                float* o = &y[(int64_t)b * n_out + col];
                *o = fmaf(w, iv, *o);
            }
        }
    }
    b4_forward(L, x, batch, y);
}

/* ── scale policy, delta_csr_types.hpp:445-466 (RMSpropScalePolicy) ────── */
static void rmsprop_scale_update(float* scale, float* state, float g, float lr, float beta2, float eps,
                                 float contrib, uint32_t* step) {
    if (!isfinite(g) || !isfinite(contrib)) return;
    const float ns = fmaf(beta2, *state, (1.0f - beta2) * fmaf(g, g, contrib * contrib));
    if (!isfinite(ns)) return;
    float hat = ns;
    if (step) {
        ++(*step);
        const float bc = 1.0f - powf(beta2, (float)(*step));
        if (bc > 0.0f) hat = ns / bc;
    }
    if (!isfinite(hat)) return;
    const float nsc = *scale - lr * g / (sqrtf(hat) + eps);
    if (!isfinite(nsc)) return;
    *state = ns;
    *scale = nsc;
}

/* Per-(synapse, sample) recurrence of the non-deferred scattered backward,
 * linear_disldo.hpp:811-885 with BoundedRMSpropSynapsePolicy
 * (delta_csr_types.hpp:707-758) at the production arguments
 * min_decay_frac = 0, max_abs_delta = 2, max_ci = 100 (cpu_backend.cpp:518-525). */
static inline float bounded_ci(float ci, float g, float contrib, float beta2) {
    const float ema = fmaf(beta2, ci, (1.0f - beta2) * fmaf(g, g, contrib * contrib));
    const float floor_ = 0.0f * ci;
    float r = (ema < floor_) ? floor_ : ema;  /* std::max(ema, floor) */
    r = 100.0f < r ? 100.0f : r;              /* std::min(.., max_ci) */
    return r;
}
/* update_cw's clipped raw step (before the eff_lr multiply) */
static inline float bounded_raw(float g, float ci, float S, float eps, int damp) {
    float raw = damp ? (-g * S) / (sqrtf(ci) + eps) : (-g * S);
    if (raw > 2.0f) raw = 2.0f;
    if (raw < -2.0f) raw = -2.0f;
    return raw;
}

static void presize_scales(OLayer* L) {
    const int64_t nr = L->rows * L->rank, nc = L->cols * L->rank;
    if (L->value_scale.n < nr) fvec_resize(&L->value_scale, nr, 1.0f);
    if (L->output_scale.n < nc) fvec_resize(&L->output_scale, nc, 1.0f);
    if (L->value_scale_importance.n < nr) fvec_resize(&L->value_scale_importance, nr, 0.0f);
    if (L->output_scale_importance.n < nc) fvec_resize(&L->output_scale_importance, nc, 0.0f);
    if (L->value_scale_momentum.n < nr) fvec_resize(&L->value_scale_momentum, nr, 0.0f);
    if (L->value_scale_step.n < nr) uvec_resize(&L->value_scale_step, nr, 0u);
}

/* disldo_backward, linear_disldo.hpp:462-2113, non-deferred scattered path
 * (block4 empty), num_cpus = 1. */
void o_backward_dense(OLayer* L, const float* x, const float* dy, int batch, float lr,
                      int lr_per_row_nnz, int damp, float beta2, float eps, float* dx) {
    const int64_t n_in = L->rows, n_out = L->cols, rank = L->rank;
    /* accumulators, :515-520 */
    for (int b = 0; b < batch; ++b) {
        for (int64_t r = 0; r < n_in; ++r) L->in_acc[r] += fabsf(x[(int64_t)b * n_in + r]);
        for (int64_t c = 0; c < n_out; ++c) L->grad_acc[c] += fabsf(dy[(int64_t)b * n_out + c]);
    }
    memset(dx, 0, (size_t)batch * n_in * sizeof(float));
    float* colg = (float*)calloc((size_t)(n_out * rank) + 1, sizeof(float));
    float* colc = (float*)calloc((size_t)(n_out * rank) + 1, sizeof(float));
    const int os_train = L->output_scale_trainable;
    presize_scales(L);
    const uint64_t call = L->call++;
    double sa_new = 0, sa_old = 0, sq_new = 0, sq_old = 0; float mx_new = 0.0f;
    /* DeferredScaleWrite's buffered stores: (value position, cw, ci, row, col) */
    int64_t n_def = 0;
    int64_t* def_vb = NULL; float* def_cw = NULL; float* def_ci = NULL; int64_t* def_r = NULL; int64_t* def_c = NULL;
    if (L->resync && lr != 0.0f && L->total_nnz > 0) {
        def_vb = (int64_t*)malloc((size_t)L->total_nnz * 8); def_r = (int64_t*)malloc((size_t)L->total_nnz * 8);
        def_c = (int64_t*)malloc((size_t)L->total_nnz * 8);
        def_cw = (float*)malloc((size_t)L->total_nnz * 4); def_ci = (float*)malloc((size_t)L->total_nnz * 4);
    }
    if (L->total_nnz > 0) {
        for (int64_t r = 0; r < n_in; ++r) {
            const int64_t nnz = row_nnz(L, r);
            if (nnz == 0) continue;
            /* a column shard divides by the row's global synapse count */
            const int64_t gnnz = L->shard_part ? (int64_t)L->shard_nnz[r] : nnz;
            const float eff_lr = lr_per_row_nnz ? lr / (float)gnnz : lr;
            const float scale_eff_lr = lr / (float)gnnz;
            const float imp_scale = o_get_importance_scale(L, (int)r);
            double sgs[4] = {0, 0, 0, 0}, sgc[4] = {0, 0, 0, 0};
            int64_t pos = L->byte_start[r]; uint32_t col = 0;
            for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
                col += uleb_get(L->idx, &pos);
                const float cw_orig = get_w(L, vb), ci_orig = get_imp(L, vb);
                const float cis = imp_scale * o_get_output_importance_scale(L, (int)col);
                float ci = ci_orig * cis;
                if (L->resync) {
                    /* the DeferredScaleWrite branch, linear_disldo.hpp:686-790: the
                     * old true-units step (cw += update_cw(g, ci, 1, ...)),
                     * component-0 scale sums from the stored code, the store
                     * buffered until the scales are final */
                    const float vs0 = o_get_value_scale_k(L, (int)r, 0), os0 = o_get_output_scale_k(L, (int)col, 0);
                    float cw = (cw_orig * vs0) * os0;
                    for (int b = 0; b < batch; ++b) {
                        const float iv = x[(int64_t)b * n_in + r];
                        const float dyv = dy[(int64_t)b * n_out + col];
                        const float g = dyv * iv;
                        if (lr != 0.0f) {
                            const float contrib = iv * cw_orig;
                            ci = bounded_ci(ci, g, contrib, beta2);
                            cw = fmaf(eff_lr, bounded_raw(g, ci, 1.0f, eps, damp), cw);
                            sgs[0] = fma((double)cw_orig * (double)os0, (double)g, sgs[0]);
                            sgc[0] = fma((double)cw_orig * (double)os0, (double)contrib, sgc[0]);
                            if (os_train) {
                                colg[col * rank] = fmaf(cw_orig * vs0, g, colg[col * rank]);
                                colc[col * rank] = fmaf(cw_orig * vs0, contrib, colc[col * rank]);
                            }
                        }
                        float* d = &dx[(int64_t)b * n_in + r];
                        *d = fmaf(cw, dyv, *d);
                    }
                    if (lr != 0.0f) {
                        def_vb[n_def] = vb; def_cw[n_def] = cw; def_ci[n_def] = ci;
                        def_r[n_def] = r; def_c[n_def] = col; ++n_def;
                        /* stats from the true-units ci, as the reference's stand-in */
                        sa_new += fabs((double)ci); sa_old += fabs((double)ci_orig);
                        sq_new += (double)ci * ci; sq_old += (double)ci_orig * ci_orig;
                        if (fabsf(ci) > mx_new) mx_new = fabsf(ci);
                    }
                    continue;
                }
                const float S = o_get_scale(L, (int)r, (int)col);
                float quant = cw_orig, cw = quant * S;
                for (int b = 0; b < batch; ++b) {
                    const float iv = x[(int64_t)b * n_in + r];
                    const float dyv = dy[(int64_t)b * n_out + col];
                    const float g = dyv * iv;
                    if (lr != 0.0f) {
                        const float contrib = iv * cw_orig;
                        ci = bounded_ci(ci, g, contrib, beta2);
                        quant = fmaf(eff_lr, bounded_raw(g, ci, S, eps, damp), quant);
                        cw = quant * S;
                        const float qf = (quant == 0.0f) ? 0.1f : quant;
                        for (int64_t k = 0; k < rank; ++k) {
                            const float os_k = o_get_output_scale_k(L, (int)col, (int)k);
                            const float vs_k = o_get_value_scale_k(L, (int)r, (int)k);
                            sgs[k] = fma((double)qf * (double)os_k, (double)g, sgs[k]);
                            sgc[k] = fma((double)qf * (double)os_k, (double)contrib, sgc[k]);
                            if (os_train) {
                                colg[col * rank + k] = fmaf(qf * vs_k, g, colg[col * rank + k]);
                                colc[col * rank + k] = fmaf(qf * vs_k, contrib, colc[col * rank + k]);
                            }
                        }
                    }
                    float* d = &dx[(int64_t)b * n_in + r];
                    *d = fmaf(cw, dyv, *d);
                }
                if (lr != 0.0f) {
                    const float imp_st = ci / cis;
                    if (L->stochastic) {
                        const uint8_t wq = o_fp4_quantize_stochastic_r(quant, o_rng_draw(L->seed, call, (uint64_t)vb, 0));
                        const uint8_t iq = o_fp4_quantize_stochastic_r(imp_st, o_rng_draw(L->seed, call, (uint64_t)vb, 1));
                        L->val[vb] = (uint8_t)((wq << 4) | iq);
                    } else {
                        set_wi(L, vb, quant, imp_st);
                    }
                    const float ai = get_imp(L, vb);
                    sa_new += fabs((double)ai); sa_old += fabs((double)ci_orig);
                    sq_new += (double)ai * ai; sq_old += (double)ci_orig * ci_orig;
                    if (fabsf(ai) > mx_new) mx_new = fabsf(ai);
                }
            }
            if (lr != 0.0f && L->resync) {
                /* component 0 only, through value_scale[r] / value_scale_importance[r]
                 * (flat index r) and the step counter of (r, 0),
                 * linear_disldo.hpp:918-923 */
                rmsprop_scale_update(&L->value_scale.d[r], &L->value_scale_importance.d[r], (float)sgs[0],
                                     scale_eff_lr, beta2, eps, (float)sgc[0], &L->value_scale_step.d[r * rank]);
            } else if (lr != 0.0f) {
                for (int64_t k = 0; k < rank; ++k) {
                    const int64_t i = r * rank + k;
                    if (L->shard_part) {   /* this shard's part of the row sums */
                        L->shard_part[2 * i] = sgs[k];
                        L->shard_part[2 * i + 1] = sgc[k];
                        continue;
                    }
                    if (L->scale_noop) continue;   /* ScalePolicy::update, linear_disldo.hpp:914-925 */
                    rmsprop_scale_update(&L->value_scale.d[i], &L->value_scale_importance.d[i],
                                         (float)sgs[k], scale_eff_lr, beta2, eps, (float)sgc[k],
                                         &L->value_scale_step.d[i]);
                }
            }
        }
        if (lr != 0.0f) {
            /* update_importance_stats_aggregate, delta_csr_types.hpp:1327-1335 */
            L->importance_l1 += sa_new - sa_old;
            L->importance_l2_sq += sq_new - sq_old;
            L->importance_max_abs = fmaxf(L->importance_max_abs * L->max_abs_decay, mx_new);
        }
    }
    b4_backward(L, x, dy, batch, lr, lr_per_row_nnz, damp, beta2, eps, dx, colg, colc, call);
    /* dead-row bootstrap, linear_disldo.hpp:1985-2042; a column shard only
     * sums its columns' part of S (rows dead on every shard take the step in
     * o_apply_row_part) */
    if (lr != 0.0f && L->shard_part) {
        int any_dead = 0;
        for (int64_t r = 0; r < n_in; ++r) if (L->shard_nnz[r] == 0) { any_dead = 1; break; }
        double* S = L->shard_part + 2 * n_in * rank;
        for (int b = 0; b < batch && any_dead; ++b)
            for (int64_t k = 0; k < rank; ++k) {
                double sum = 0.0;
                for (int64_t c = 0; c < n_out; ++c)
                    sum += (double)o_get_output_scale_k(L, (int)c, (int)k) * (double)dy[(int64_t)b * n_out + c];
                S[b * rank + k] = sum;
            }
    } else if (lr != 0.0f) {
        int any_dead = 0;
        for (int64_t r = 0; r < n_in; ++r) if (row_nnz(L, r) == 0 && b4_row_live(L, r) == 0) { any_dead = 1; break; }
        if (any_dead) {
            double* S = (double*)calloc((size_t)(batch * rank) + 1, sizeof(double));
            for (int b = 0; b < batch; ++b)
                for (int64_t k = 0; k < rank; ++k) {
                    double s = 0.0;
                    for (int64_t c = 0; c < n_out; ++c)
                        s += (double)o_get_output_scale_k(L, (int)c, (int)k) * (double)dy[(int64_t)b * n_out + c];
                    S[b * rank + k] = s;
                }
            const float dead_lr = lr / (float)n_out;
            for (int64_t r = 0; r < n_in; ++r) {
                if (row_nnz(L, r) != 0 || b4_row_live(L, r) != 0) continue;
                for (int64_t k = 0; k < rank; ++k) {
                    double sum = 0.0;
                    for (int b = 0; b < batch; ++b) {
                        const float iv = x[(int64_t)b * n_in + r];
                        if (iv == 0.0f) continue;
                        sum += (double)iv * S[b * rank + k];
                    }
                    if (sum == 0.0) continue;
                    const float g = (float)sum;
                    if (!isfinite(g)) continue;
                    const int64_t i = r * rank + k;
                    float* m = &L->value_scale_momentum.d[i];
                    float* v = &L->value_scale_importance.d[i];
                    const float nm = fmaf(0.9f, *m, (1.0f - 0.9f) * g);
                    const float nv = fmaf(1.0f - beta2, g * g, beta2 * *v);
                    if (!isfinite(nm) || !isfinite(nv)) continue;
                    const float nvs = L->value_scale.d[i] - dead_lr * nm / (sqrtf(nv) + eps);
                    if (!isfinite(nvs)) continue;
                    *m = nm; *v = nv;
                    L->value_scale.d[i] = nvs;
                }
            }
            free(S);
        }
    }
    /* output_scale update, linear_disldo.hpp:2051-2080 (ScalePolicy::update at :2075) */
    if (lr != 0.0f && os_train && !L->scale_noop) {
        if (L->output_scale_step.n < n_out * rank) uvec_resize(&L->output_scale_step, n_out * rank, 0u);
        for (int64_t c = 0; c < n_out; ++c) {
            const int deg = L->out_degree[c];
            if (deg == 0) continue;
            const float col_lr = lr / (float)deg;
            for (int64_t k = 0; k < rank; ++k) {
                const float g = (float)(0.0 + (double)colg[c * rank + k]);
                const float cc = (float)(0.0 + (double)colc[c * rank + k]);
                rmsprop_scale_update(&L->output_scale.d[c * rank + k], &L->output_scale_importance.d[c * rank + k],
                                     g, col_lr, beta2, eps, cc, &L->output_scale_step.d[c * rank + k]);
            }
        }
    }
    /* the deferred stores under the final scales, linear_disldo.hpp:2090-2112 */
    for (int64_t q = 0; q < n_def; ++q) {
        const int r = (int)def_r[q], c = (int)def_c[q];
        const float comb = o_get_value_scale_k(L, r, 0) * o_get_output_scale_k(L, c, 0);
        const float combi = o_get_importance_scale(L, r) * o_get_output_importance_scale(L, c);
        const float w = def_cw[q] / comb, imp = def_ci[q] / combi;
        if (L->stochastic) {
            const uint8_t wq = o_fp4_quantize_stochastic_r(w, o_rng_draw(L->seed, call, (uint64_t)def_vb[q], 0));
            const uint8_t iq = o_fp4_quantize_stochastic_r(imp, o_rng_draw(L->seed, call, (uint64_t)def_vb[q], 1));
            L->val[def_vb[q]] = (uint8_t)((wq << 4) | iq);
        } else {
            set_wi(L, def_vb[q], w, imp);
        }
    }
    free(def_vb); free(def_cw); free(def_ci); free(def_r); free(def_c);
    free(colg); free(colc);
}

/* ── column shards of one layer (a folded stack split by output column) ──
 * Every synapse update of disldo_backward is local to its (row, column); what
 * couples the columns of a row is (a) lr / nnz_row, (b) the row's value_scale
 * step from sums over all its synapses (linear_disldo.hpp:901-925) and (c) the
 * dead-row bootstrap's S over all columns (:1985-2042).  A shard takes the
 * global row counts for (a), returns its part of (b) and (c), and after the
 * parts are summed over the shards applies the row steps with the totals. */
int o_set_row_shard(OLayer* L, const int* global_row_nnz, int64_t n, int64_t global_n_out) {
    free(L->shard_nnz);
    L->shard_nnz = NULL;
    if (n == 0) return 0;
    if (n != L->rows) return 1;
    L->shard_nnz = (int*)malloc((size_t)n * sizeof(int));
    memcpy(L->shard_nnz, global_row_nnz, (size_t)n * sizeof(int));
    L->shard_n_out = global_n_out;
    return 0;
}
int64_t o_row_part_len(const OLayer* L, int batch) { return 2 * L->rows * L->rank + (int64_t)batch * L->rank; }

int o_backward_dense_shard(OLayer* L, const float* x, const float* dy, int batch, float lr, int lr_per_row_nnz,
                           int damp, float beta2, float eps, float* dx, double* part) {
    if (!L->shard_nnz || o_b4_ntiles(L) > 0) return 1;   /* block4 tiles: not sharded */
    memset(part, 0, (size_t)o_row_part_len(L, batch) * sizeof(double));
    L->shard_part = part;
    o_backward_dense(L, x, dy, batch, lr, lr_per_row_nnz, damp, beta2, eps, dx);
    L->shard_part = NULL;
    return 0;
}

void o_apply_row_part(OLayer* L, const float* x, int batch, float lr, float beta2, float eps, const double* part) {
    const int64_t n_in = L->rows, rank = L->rank;
    if (lr == 0.0f || !L->shard_nnz) return;
    const double* S = part + 2 * n_in * rank;
    const float dead_lr = lr / (float)L->shard_n_out;
    for (int64_t r = 0; r < n_in; ++r) {
        const int64_t gnnz = L->shard_nnz[r];
        for (int64_t k = 0; k < rank; ++k) {
            const int64_t i = r * rank + k;
            if (gnnz > 0) {
                if (!L->scale_noop)
                    rmsprop_scale_update(&L->value_scale.d[i], &L->value_scale_importance.d[i], (float)part[2 * i],
                                         lr / (float)gnnz, beta2, eps, (float)part[2 * i + 1],
                                         &L->value_scale_step.d[i]);
                continue;
            }
            double sum = 0.0;
            for (int b = 0; b < batch; ++b) {
                const float iv = x[(int64_t)b * n_in + r];
                if (iv == 0.0f) continue;
                sum += (double)iv * S[b * rank + k];
            }
            if (sum == 0.0) continue;
            const float g = (float)sum;
            if (!isfinite(g)) continue;
            float* m = &L->value_scale_momentum.d[i];
            float* v = &L->value_scale_importance.d[i];
            const float nm = fmaf(0.9f, *m, (1.0f - 0.9f) * g);
            const float nv = fmaf(1.0f - beta2, g * g, beta2 * *v);
            if (!isfinite(nm) || !isfinite(nv)) continue;
            const float nvs = L->value_scale.d[i] - dead_lr * nm / (sqrtf(nv) + eps);
            if (!isfinite(nvs)) continue;
            *m = nm; *v = nv;
            L->value_scale.d[i] = nvs;
        }
    }
}

/* ── sisldo_forward, sisldo_ops.hpp:198-340 (scattered part, num_cpus = 1) ─ */
static void b4_forward_sparse(const OLayer* L, const int* ptrs, const int* idx, const float* vals, int batch,
                              float* y);
static void b4_backward_sparse(OLayer* L, const float* x, const int* dptrs, const int* didx, const float* dvals,
                               int batch, float lr, int lr_per_row_nnz, int damp, float beta2, float eps, float* dx,
                               uint64_t call);
void o_forward_sparse(OLayer* L, const int* ptrs, const int* idx, const float* vals, int batch, float* y) {
    const int64_t n_out = L->cols;
    memset(y, 0, (size_t)batch * n_out * sizeof(float));
    if (L->total_nnz > 0) for (int b = 0; b < batch; ++b) {
        for (int i = ptrs[b]; i < ptrs[b + 1]; ++i) {
            const int r = idx[i];
            const float iv = vals[i];
            int64_t pos = L->byte_start[r]; uint32_t col = 0;
            const float vs = o_get_value_scale_k(L, r, 0);
            for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
                col += uleb_get(L->idx, &pos);
                /* wval_stored * (vs*os) * in_val, as the reference's build
                 * evaluates it: (wval_stored * in_val) * (vs*os), then += */
                const float cs = vs * o_get_output_scale_k(L, (int)col, 0);
                float* o = &y[(int64_t)b * n_out + col];
                *o = *o + (get_w(L, vb) * iv) * cs;
            }
        }
    }
    b4_forward_sparse(L, ptrs, idx, vals, batch, y);
}

/* ── disldo_backward_sparse_grad, sisldo_ops.hpp:589-799 (scattered, num_cpus = 1) */
void o_backward_sparse(OLayer* L, const float* x, const int* dptrs, const int* didx, const float* dvals,
                       int batch, float lr, int lr_per_row_nnz, int damp, float beta2, float eps, float* dx) {
    const int64_t n_in = L->rows;
    for (int b = 0; b < batch; ++b)
        for (int64_t r = 0; r < n_in; ++r) L->in_acc[r] += fabsf(x[(int64_t)b * n_in + r]);
    for (int b = 0; b < batch; ++b)
        for (int j = dptrs[b]; j < dptrs[b + 1]; ++j) L->grad_acc[didx[j]] += fabsf(dvals[j]);
    if (L->value_scale.n < n_in) fvec_resize(&L->value_scale, n_in, 1.0f);
    if (L->value_scale_importance.n < n_in) fvec_resize(&L->value_scale_importance, n_in, 0.0f);
    memset(dx, 0, (size_t)batch * n_in * sizeof(float));
    const uint64_t call = L->call++;
    if (L->total_nnz == 0) {
        b4_backward_sparse(L, x, dptrs, didx, dvals, batch, lr, lr_per_row_nnz, damp, beta2, eps, dx, call);
        return;
    }
    double* sgs = (double*)calloc((size_t)n_in + 1, sizeof(double));
    double* sgc = (double*)calloc((size_t)n_in + 1, sizeof(double));
    double sa_new = 0, sa_old = 0, sq_new = 0, sq_old = 0; float mx_new = 0.0f;
    for (int b = 0; b < batch; ++b) {
        const int og0 = dptrs[b], og1 = dptrs[b + 1];
        for (int64_t r = 0; r < n_in; ++r) {
            const int64_t nnz = row_nnz(L, r);
            if (nnz == 0) continue;
            const float in_val = x[(int64_t)b * n_in + r];
            const float eff_lr = lr_per_row_nnz ? lr / (float)nnz : lr;
            int64_t pos = L->byte_start[r]; uint32_t col = 0;
            int og = og0;
            float dxa = 0.0f;
            const float imp_scale = o_get_importance_scale(L, (int)r);
            const float val_scale = o_get_value_scale_k(L, (int)r, 0);
            for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
                col += uleb_get(L->idx, &pos);
                const float w_stored = get_w(L, vb);
                const float out_scale = o_get_output_scale_k(L, (int)col, 0);
                const float cs = val_scale * out_scale;
                const float w = w_stored * cs;
                while (og < og1 && didx[og] < (int)col) ++og;
                if (og >= og1 || didx[og] != (int)col) continue;
                const float dyv = dvals[og];
                dxa = fmaf(w, dyv, dxa);
                if (lr != 0.0f) {
                    const float cis = imp_scale * o_get_output_importance_scale(L, (int)col);
                    const float grad = dyv * in_val;
                    const float stored_imp = get_imp(L, vb);
                    float imp = stored_imp * cis;
                    const float contrib = in_val * w;
                    imp = fmaf(beta2, imp, (1.0f - beta2) * fmaf(grad, grad, contrib * contrib));
                    const float step = damp ? (-eff_lr * grad) / (sqrtf(imp) + eps) : (-eff_lr * grad);
                    const float new_w = w + step;
                    set_wi(L, vb, new_w / cs, imp / cis);
                    const float ai = get_imp(L, vb);
                    sa_new += fabs((double)ai); sa_old += fabs((double)stored_imp);
                    sq_new += (double)ai * ai; sq_old += (double)stored_imp * stored_imp;
                    if (fabsf(ai) > mx_new) mx_new = fabsf(ai);
                    sgs[r] += (double)w_stored * (double)out_scale * (double)(dyv * in_val);
                    sgc[r] += (double)w_stored * (double)out_scale * (double)contrib;
                }
            }
            dx[(int64_t)b * n_in + r] += dxa;
        }
    }
    if (lr != 0.0f) {
        L->importance_l1 += sa_new - sa_old;
        L->importance_l2_sq += sq_new - sq_old;
        L->importance_max_abs = fmaxf(L->importance_max_abs * L->max_abs_decay, mx_new);
        if (L->value_scale_step.n < n_in * L->rank) uvec_resize(&L->value_scale_step, n_in * L->rank, 0u);
        for (int64_t r = 0; r < n_in; ++r) {
            if (sgs[r] == 0.0 && sgc[r] == 0.0) continue;
            const int64_t nnz = row_nnz(L, r);
            if (nnz == 0) continue;
            const float se = lr / (float)nnz;
            const float g = (float)sgs[r], cg = (float)sgc[r];
            float* vsi = &L->value_scale_importance.d[r];
            const float nv = fmaf(beta2, *vsi, (1.0f - beta2) * fmaf(g, g, cg * cg));
            uint32_t* st = &L->value_scale_step.d[r * L->rank];
            ++(*st);
            const float bc = 1.0f - powf(beta2, (float)(*st));
            const float hat = bc > 0.0f ? nv / bc : nv;
            *vsi = nv;
            L->value_scale.d[r] -= se * g / (sqrtf(hat) + eps);
        }
    }
    free(sgs); free(sgc);
    b4_backward_sparse(L, x, dptrs, didx, dvals, batch, lr, lr_per_row_nnz, damp, beta2, eps, dx, call);
}

/* ── synaptogenesis candidates, delta_csr_memory.hpp:1308-1427 ──────────── */
/* Strict descending order with ascending index on ties (the reference's
 * partial_sort leaves tie order unspecified). */
static const float* g_keys;
static int cmp_desc_idx(const void* a, const void* b) {
    const int64_t ia = *(const int64_t*)a, ib = *(const int64_t*)b;
    const float ka = g_keys[ia], kb = g_keys[ib];
    if (ka > kb) return -1;
    if (ka < kb) return 1;
    return ia < ib ? -1 : (ia > ib);
}
static int64_t* top_k_desc(const float* keys, int64_t n, int64_t k, const uint8_t* excl) {
    int64_t m = 0;
    int64_t* ix = (int64_t*)malloc((size_t)(n + 1) * sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) if (!excl || !excl[i]) ix[m++] = i;
    g_keys = keys;
    qsort(ix, (size_t)m, sizeof(int64_t), cmp_desc_idx);
    (void)k;
    return ix;
}

static void decode_row(const OLayer* L, int64_t r, uint32_t* cols) {
    int64_t pos = L->byte_start[r]; uint32_t c = 0; int64_t n = row_nnz(L, r);
    for (int64_t i = 0; i < n; ++i) { c += uleb_get(L->idx, &pos); cols[i] = c; }
}

void o_build_probes(OLayer* L, int k, int per_row) {
    const int64_t n_in = L->rows, n_out = L->cols;
    free(L->prow); free(L->pcol); free(L->pval);
    L->prow = NULL; L->pcol = NULL; L->pval = NULL; L->n_probes = 0;
    if (n_in == 0 || n_out == 0 || k <= 0) return;
    const int64_t kin = k < n_in ? k : n_in;
    int64_t* in_idx = top_k_desc(L->in_acc, n_in, kin, NULL);
    int64_t cap = kin * (int64_t)k + 1, np = 0;
    L->prow = (int*)malloc((size_t)cap * sizeof(int));
    L->pcol = (int*)malloc((size_t)cap * sizeof(int));
    L->pval = (float*)malloc((size_t)cap * sizeof(float));
    uint32_t* cols = (uint32_t*)malloc((size_t)(n_out + 1) * sizeof(uint32_t));
    uint8_t* ex = (uint8_t*)calloc((size_t)n_out + 1, 1);
    if (!per_row) {
        const int64_t kout = k < n_out ? k : n_out;
        int64_t* out_idx = top_k_desc(L->grad_acc, n_out, kout, NULL);
        for (int64_t a = 0; a < kin; ++a) {
            const int64_t r = in_idx[a];
            const int64_t n = row_nnz(L, r);
            decode_row(L, r, cols);
            for (int64_t i = 0; i < n; ++i) ex[cols[i]] = 1;
            for (int64_t b = 0; b < kout; ++b) {
                const int64_t c = out_idx[b];
                if (ex[c]) continue;
                L->prow[np] = (int)r; L->pcol[np] = (int)c;
                L->pval[np] = L->in_acc[r] * L->grad_acc[c];
                ++np;
            }
            for (int64_t i = 0; i < n; ++i) ex[cols[i]] = 0;
        }
        free(out_idx);
    } else {
        for (int64_t a = 0; a < kin; ++a) {
            const int64_t r = in_idx[a];
            const int64_t n = row_nnz(L, r);
            decode_row(L, r, cols);
            for (int64_t i = 0; i < n; ++i) ex[cols[i]] = 1;
            int64_t* cand = top_k_desc(L->grad_acc, n_out, k, ex);
            int64_t navail = n_out - 0;
            for (int64_t i = 0; i < n; ++i) navail -= 1;
            /* n counts distinct existing cols (rows are strictly increasing) */
            const int64_t kr = k < navail ? k : navail;
            for (int64_t i = 0; i < kr; ++i) {
                const int64_t c = cand[i];
                L->prow[np] = (int)r; L->pcol[np] = (int)c;
                L->pval[np] = L->in_acc[r] * L->grad_acc[c];
                ++np;
            }
            free(cand);
            for (int64_t i = 0; i < n; ++i) ex[cols[i]] = 0;
        }
    }
    L->n_probes = np;
    free(in_idx); free(cols); free(ex);
}

int64_t o_num_probes(const OLayer* L) { return L->n_probes; }
void o_get_probes(const OLayer* L, int* rows, int* cols, float* scores) {
    for (int64_t i = 0; i < L->n_probes; ++i) { rows[i] = L->prow[i]; cols[i] = L->pcol[i]; scores[i] = L->pval[i]; }
}
void o_set_probes(OLayer* L, const int* rows, const int* cols, const float* scores, int64_t n) {
    free(L->prow); free(L->pcol); free(L->pval);
    L->prow = (int*)malloc((size_t)(n + 1) * sizeof(int));
    L->pcol = (int*)malloc((size_t)(n + 1) * sizeof(int));
    L->pval = (float*)malloc((size_t)(n + 1) * sizeof(float));
    for (int64_t i = 0; i < n; ++i) { L->prow[i] = rows[i]; L->pcol[i] = cols[i]; L->pval[i] = scores[i]; }
    L->n_probes = n;
}

/* ── row rebuild (canonical re-encode of one row within its allocation) ─── */
/* delta_csr_row_remove_col (:429-492) and delta_csr_row_insert_col
 * (:500-585) both leave the row's live bytes equal to the ULEB128 encoding of
 * its sorted column list, written from byte_start[row], and its value bytes
 * in column order from elem_start[row]; only the blank tail differs.  The
 * restatement therefore rewrites the live part of the row. */
static int row_write(OLayer* L, int64_t r, const uint32_t* cols, const uint8_t* vals, int64_t n) {
    int64_t nb = 0; uint32_t prev = 0;
    for (int64_t i = 0; i < n; ++i) { nb += uleb_len(cols[i] - prev); prev = cols[i]; }
    if (nb > L->byte_start[r + 1] - L->byte_start[r]) return O_EHEADROOM;
    if (n > L->elem_start[r + 1] - L->elem_start[r]) return O_EHEADROOM;
    int64_t bp = L->byte_start[r]; prev = 0;
    for (int64_t i = 0; i < n; ++i) { bp += uleb_put(cols[i] - prev, L->idx + bp); prev = cols[i]; }
    L->byte_end[r] = bp;
    memcpy(L->val + L->elem_start[r], vals, (size_t)n);
    L->total_nnz += n - row_nnz(L, r);
    L->elem_end[r] = L->elem_start[r] + n;
    return O_OK;
}

/* Byte cost of inserting col into a sorted row (delta_csr_row_insert_col's
 * idx_delta, :541-551) and its headroom test (:553-559). */
static int insert_fits(const OLayer* L, int64_t r, const uint32_t* cols, int64_t n, uint32_t c) {
    int64_t i = 0; uint32_t prev = 0;
    while (i < n && cols[i] < c) { prev = cols[i]; ++i; }
    const int64_t nd = uleb_len(c - prev);
    int64_t upd = 0, old = 0;
    if (i < n) { upd = uleb_len(cols[i] - c); old = uleb_len(cols[i] - prev); }
    const int64_t delta = nd + upd - old;
    const int64_t used = L->byte_end[r] - L->byte_start[r];
    if (delta > 0 && delta > (L->byte_start[r + 1] - L->byte_start[r]) - used) return 0;
    if (n >= L->elem_start[r + 1] - L->elem_start[r]) return 0;
    return 1;
}

/* o_synap_row_step: after the block4 section below */

/* ── headroom management ─────────────────────────────────────────────────── */
/* delta_csr_shift_row, delta_csr_memory.hpp:225-293 */
static int shift_row(OLayer* L, int64_t row, int64_t tb, int64_t te) {
    const int64_t R = L->rows;
    const int64_t cb = L->byte_start[row + 1] - L->byte_start[row];
    if (cb != tb && row + 1 < R) {
        const int64_t src = L->byte_start[row + 1];
        const int64_t len = L->byte_start[R] - src;
        const int64_t dst = L->byte_start[row] + tb;
        int64_t nt = L->idx_n;
        if (tb > cb) {
            nt = L->idx_n + (tb - cb);
            if (nt > L->max_idx_bytes) return O_ENOMEM;
            L->idx = (uint8_t*)realloc(L->idx, (size_t)nt + 16);
            memset(L->idx + L->idx_n, 0, (size_t)(nt - L->idx_n));
        }
        if (len > 0) memmove(L->idx + dst, L->idx + src, (size_t)len);
        if (tb < cb) nt = L->idx_n - (cb - tb);
        L->idx_n = nt;
        const int64_t d = tb - cb;
        for (int64_t r = row + 1; r <= R; ++r) L->byte_start[r] += d;
        for (int64_t r = row + 1; r < R; ++r) L->byte_end[r] += d;
    }
    const int64_t ce = L->elem_start[row + 1] - L->elem_start[row];
    if (ce != te && row + 1 < R) {
        const int64_t src = L->elem_start[row + 1];
        const int64_t len = L->elem_start[R] - src;
        const int64_t dst = L->elem_start[row] + te;
        const int64_t cur = L->elem_start[R];
        if (te > ce) {
            const int64_t nt = cur + (te - ce);
            if (nt > L->max_val_bytes) return O_ENOMEM;
            L->val = (uint8_t*)realloc(L->val, (size_t)nt + 16);
            memset(L->val + L->val_n, 0, (size_t)(nt - L->val_n));
            L->val_n = nt;
        }
        if (len > 0) memmove(L->val + dst, L->val + src, (size_t)len);
        if (te < ce) L->val_n = cur - (ce - te);
        const int64_t d = te - ce;
        for (int64_t r = row + 1; r <= R; ++r) L->elem_start[r] += d;
        for (int64_t r = row + 1; r < R; ++r) L->elem_end[r] += d;
    }
    return O_OK;
}

/* delta_csr_equalize_step, delta_csr_memory.hpp:296-306 (row passed in) */
int o_equalizer_step(OLayer* L, int row_in) {
    if (L->rows == 0) return O_OK;
    const int64_t row = (int64_t)row_in % L->rows;
    const int64_t tb = (L->byte_start[L->rows] + L->rows - 1) / L->rows;
    const int64_t te = (L->elem_start[L->rows] + L->rows - 1) / L->rows;
    return shift_row(L, row, tb, te);
}

/* equalize_to_capacity, cpu_backend.cpp:684-729 */
int o_equalize_to_capacity(OLayer* L, int target_elems, int target_bytes) {
    const int64_t te = target_elems;
    const int64_t tb = target_bytes > 0 ? target_bytes : te * 5 + 4;
    const int64_t R = L->rows;
    for (int64_t r = 0; r + 1 < R; ++r) {
        const int64_t cb = L->byte_start[r + 1] - L->byte_start[r];
        const int64_t ce = L->elem_start[r + 1] - L->elem_start[r];
        const int64_t ub = cb > tb ? cb : tb, ue = ce > te ? ce : te;
        if (ub == cb && ue == ce) continue;
        const int rc = shift_row(L, r, ub, ue);
        if (rc) return rc;
    }
    if (R > 0) {
        const int64_t r = R - 1;
        const int64_t cb = L->byte_start[R] - L->byte_start[r];
        const int64_t ce = L->elem_start[R] - L->elem_start[r];
        const int64_t ub = cb > tb ? cb : tb, ue = ce > te ? ce : te;
        if (ub > cb) {
            const int64_t nt = L->idx_n + (ub - cb);
            L->idx = (uint8_t*)realloc(L->idx, (size_t)nt + 16);
            memset(L->idx + L->idx_n, 0, (size_t)(nt - L->idx_n));
            L->idx_n = nt;
            L->byte_start[R] = L->byte_start[r] + ub;
        }
        if (ue > ce) {
            const int64_t nt = L->elem_start[R] + (ue - ce);
            L->val = (uint8_t*)realloc(L->val, (size_t)nt + 16);
            memset(L->val + L->val_n, 0, (size_t)(nt - L->val_n));
            L->val_n = nt;
            L->elem_start[R] = nt;
        }
    }
    return O_OK;
}

/* compact, sisldo_ops.hpp:44-96 */
void o_compact(OLayer* L) {
    const int64_t R = L->rows;
    int64_t tb = 0, te = 0;
    for (int64_t r = 0; r < R; ++r) { tb += L->byte_end[r] - L->byte_start[r]; te += row_nnz(L, r); }
    uint8_t* ib = (uint8_t*)calloc((size_t)tb + 16, 1);
    uint8_t* vb = (uint8_t*)calloc((size_t)te + 16, 1);
    int64_t bc = 0, ec = 0;
    for (int64_t r = 0; r < R; ++r) {
        const int64_t bl = L->byte_end[r] - L->byte_start[r], n = row_nnz(L, r);
        memcpy(ib + bc, L->idx + L->byte_start[r], (size_t)bl);
        /* values are re-set through the quantizer: decode -> encode is the identity
         * on codes the encoder produces; code 8 (NaN) re-encodes to 0 */
        for (int64_t k = 0; k < n; ++k) {
            const uint8_t v = L->val[L->elem_start[r] + k];
            vb[ec + k] = (uint8_t)((o_fp4_encode(o_fp4_decode(v >> 4)) << 4) | o_fp4_encode(o_fp4_decode(v & 0xF)));
        }
        L->byte_start[r] = bc; L->byte_end[r] = bc + bl; bc += bl;
        L->elem_start[r] = ec; L->elem_end[r] = ec + n; ec += n;
    }
    L->byte_start[R] = bc; L->elem_start[R] = ec;
    free(L->idx); free(L->val);
    L->idx = ib; L->idx_n = tb; L->val = vb; L->val_n = te;
}

static void to_absolute(const OLayer* L, int* ptrs, int* idx, float* w, float* imp) {
    int64_t f = 0; ptrs[0] = 0;
    for (int64_t r = 0; r < L->rows; ++r) {
        int64_t pos = L->byte_start[r]; uint32_t c = 0;
        for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb, ++f) {
            c += uleb_get(L->idx, &pos);
            idx[f] = (int)c; w[f] = get_w(L, vb); imp[f] = get_imp(L, vb);
        }
        ptrs[r + 1] = (int)f;
    }
}

/* expand_headroom / expand_headroom_to, sisldo_ops.hpp:127-186 */
static int rebuild(OLayer* L, int64_t budget, float bf) {
    const int64_t n = L->total_nnz;
    int* p = (int*)malloc((size_t)(L->rows + 1) * sizeof(int));
    int* ix = (int*)malloc((size_t)(n + 1) * sizeof(int));
    float* w = (float*)malloc((size_t)(n + 1) * sizeof(float));
    float* im = (float*)malloc((size_t)(n + 1) * sizeof(float));
    to_absolute(L, p, ix, w, im);
    const double f = 1.0 + (double)bf;
    const int64_t ibytes = (int64_t)((double)budget * f * 6.0 + 4096.0);
    const int64_t vbytes = (int64_t)((double)budget * f) + 64;
    const int rc = from_absolute(L, p, ix, w, im, L->rows, L->cols, ibytes, vbytes, bf,
                                 L->max_idx_bytes, L->max_val_bytes);
    free(p); free(ix); free(w); free(im);
    if (rc == O_OK) { L->max_idx_bytes = L->idx_budget; L->max_val_bytes = L->val_budget; }
    return rc;
}
int o_expand_headroom(OLayer* L, float bf) { return rebuild(L, L->total_nnz, bf); }
int o_expand_headroom_to(OLayer* L, int min_nnz_per_row, float bf) {
    int64_t b = L->rows * (int64_t)min_nnz_per_row;
    if (b < L->total_nnz) b = L->total_nnz;
    return rebuild(L, b, bf);
}

/* rescale_value_row / rescale_importance_row, delta_csr_types.hpp:1389-1431 */
void o_rescale_value_row(OLayer* L, int row, float ns) {
    const float os = o_get_value_scale_k(L, row, 0);
    if (ns == os) return;
    if (row >= L->rows) return;
    for (int64_t vb = L->elem_start[row]; vb < L->elem_end[row]; ++vb)
        set_wi(L, vb, get_w(L, vb) * os / ns, get_imp(L, vb));
    o_set_value_scale_raw_k(L, row, 0, ns);
}
void o_rescale_importance_row(OLayer* L, int row, float ns) {
    const float os = o_get_importance_scale(L, row);
    if (ns == os) return;
    if (row >= L->rows) return;
    for (int64_t vb = L->elem_start[row]; vb < L->elem_end[row]; ++vb)
        set_wi(L, vb, get_w(L, vb), get_imp(L, vb) * os / ns);
    o_set_importance_scale_raw(L, row, ns);
}

/* ── export ──────────────────────────────────────────────────────────────── */
void o_sizes(const OLayer* L, int64_t* s) {
    s[0] = L->rows; s[1] = L->cols; s[2] = L->total_nnz; s[3] = L->idx_n; s[4] = L->val_n; s[5] = 0;
}
void o_layout(const OLayer* L, int64_t* bs, int64_t* be, int64_t* es, int64_t* ee) {
    for (int64_t r = 0; r <= L->rows; ++r) { bs[r] = L->byte_start[r]; es[r] = L->elem_start[r]; }
    for (int64_t r = 0; r < L->rows; ++r) { be[r] = L->byte_end[r]; ee[r] = L->elem_end[r]; }
}
void o_indices_buf(const OLayer* L, uint8_t* out) { memcpy(out, L->idx, (size_t)L->idx_n); }
void o_value_bytes(const OLayer* L, uint8_t* out) { memcpy(out, L->val, (size_t)L->val_n); }
void o_accums(const OLayer* L, float* a, float* g) {
    memcpy(a, L->in_acc, (size_t)L->rows * sizeof(float));
    memcpy(g, L->grad_acc, (size_t)L->cols * sizeof(float));
}
void o_set_accums(OLayer* L, const float* a, const float* g) {
    memcpy(L->in_acc, a, (size_t)L->rows * sizeof(float));
    memcpy(L->grad_acc, g, (size_t)L->cols * sizeof(float));
}
void o_zero_accum(OLayer* L) {
    memset(L->in_acc, 0, (size_t)L->rows * sizeof(float));
    memset(L->grad_acc, 0, (size_t)L->cols * sizeof(float));
}
void o_out_degree(const OLayer* L, int* out) { memcpy(out, L->out_degree, (size_t)L->cols * sizeof(int)); }
void o_stats(const OLayer* L, double* s) {
    s[0] = L->value_l1; s[1] = L->value_l2_sq; s[2] = L->value_max_abs;
    s[3] = L->importance_l1; s[4] = L->importance_l2_sq; s[5] = L->importance_max_abs;
}
/* delta_csr_combined_to_absolute, delta_csr_memory.hpp:127-213: per row the
 * scattered synapses then the row's live block4 slots, std::sort by column */
static int lt_i32_asc(int64_t a, int64_t b, const void* c) { const int* k = (const int*)c; return k[a] < k[b]; }
static int64_t b4_live_slots(const OLayer* L) {
    int64_t n = 0;
    for (int64_t br = 0; br < L->b4_rows; ++br)
        for (int64_t e = 0; e < L->b4[br].n; ++e)
            for (int li = 0; li < 4; ++li)
                for (int lj = 0; lj < 4; ++lj)
                    if (L->b4[br].t[e].s[B4_SLOT(li, lj)] && br * 4 + li < L->rows && (int64_t)L->b4[br].t[e].bc * 4 + lj < L->cols) ++n;
    return n;
}
int64_t o_export_nnz(const OLayer* L) { return L->total_nnz + (o_b4_ntiles(L) ? b4_live_slots(L) : 0); }
void o_export(const OLayer* L, int* ptrs, int* idx, float* w, float* imp) {
    if (o_b4_ntiles(L) == 0) { to_absolute(L, ptrs, idx, w, imp); return; }
    ptrs[0] = 0;
    int64_t o = 0;
    for (int64_t r = 0; r < L->rows; ++r) {
        const int64_t n = row_nnz(L, r), br = r / 4, li = r % 4;
        const int64_t cap = n + 4 * L->b4[br].n + 1;
        int* cc = (int*)malloc((size_t)cap * sizeof(int));
        float* ww = (float*)malloc((size_t)cap * sizeof(float));
        float* ii = (float*)malloc((size_t)cap * sizeof(float));
        int64_t* pm = (int64_t*)malloc((size_t)cap * sizeof(int64_t));
        uint32_t* cols = (uint32_t*)malloc((size_t)n * 4 + 4);
        decode_row(L, r, cols);
        int64_t m = 0;
        for (int64_t k = 0; k < n; ++k) {
            cc[m] = (int)cols[k]; ww[m] = get_w(L, L->elem_start[r] + k); ii[m] = get_imp(L, L->elem_start[r] + k); ++m;
        }
        for (int64_t e = 0; e < L->b4[br].n; ++e)
            for (int lj = 0; lj < 4; ++lj) {
                const uint8_t byte = L->b4[br].t[e].s[B4_SLOT(li, lj)];
                const int64_t col = (int64_t)L->b4[br].t[e].bc * 4 + lj;
                if (byte == 0 || col >= L->cols) continue;
                cc[m] = (int)col; ww[m] = o_fp4_decode(byte & 0xF); ii[m] = o_fp4_decode((uint8_t)(byte >> 4)); ++m;
            }
        for (int64_t q = 0; q < m; ++q) pm[q] = q;
        o_std_sort(pm, m, lt_i32_asc, cc);
        for (int64_t q = 0; q < m; ++q) { idx[o] = cc[pm[q]]; w[o] = ww[pm[q]]; imp[o] = ii[pm[q]]; ++o; }
        ptrs[r + 1] = (int)o;
        free(cc); free(ww); free(ii); free(pm); free(cols);
    }
}

/* ── activation sparsifiers ─────────────────────────────────────────────── */
/* dense_to_csr, cpu_backend.cpp:3075-3116 */
int64_t o_dense_to_csr(const float* x, int rows, int cols, float thr, int* ptrs, int* idx, float* vals) {
    int64_t n = 0;
    for (int b = 0; b < rows; ++b) {
        ptrs[b] = (int)n;
        for (int c = 0; c < cols; ++c) {
            const float v = x[(int64_t)b * cols + c];
            if (v > thr || v < -thr) { if (idx) { idx[n] = c; vals[n] = v; } ++n; }
        }
    }
    ptrs[rows] = (int)n;
    return n;
}

/* top_k_csr, csr.hpp:404-503: global exact top-k by |v|, emitted row-major
 * with ascending columns.  Ties at the k-th magnitude are resolved toward
 * the lower flat index (the reference's partial_sort leaves them unspecified). */
static const float* g_absx;
static int cmp_abs_desc(const void* a, const void* b) {
    const int64_t ia = *(const int64_t*)a, ib = *(const int64_t*)b;
    const float ka = fabsf(g_absx[ia]), kb = fabsf(g_absx[ib]);
    if (ka > kb) return -1;
    if (ka < kb) return 1;
    return (ia > ib) - (ia < ib);
}
static int cmp_i64(const void* a, const void* b) {
    const int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
    return (x > y) - (x < y);
}
int64_t o_top_k_csr(const float* x, int rows, int cols, int64_t k, int* ptrs, int* idx, float* vals) {
    const int64_t n = (int64_t)rows * cols;
    if (k > n) k = n;
    int64_t* ix = (int64_t*)malloc((size_t)(n + 1) * sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) ix[i] = i;
    g_absx = x;
    qsort(ix, (size_t)n, sizeof(int64_t), cmp_abs_desc);
    qsort(ix, (size_t)k, sizeof(int64_t), cmp_i64);
    for (int b = 0; b <= rows; ++b) ptrs[b] = 0;
    for (int64_t i = 0; i < k; ++i) {
        idx[i] = (int)(ix[i] % cols); vals[i] = x[ix[i]];
        ptrs[ix[i] / cols + 1]++;
    }
    for (int b = 0; b < rows; ++b) ptrs[b + 1] += ptrs[b];
    free(ix);
    return k;
}

/* ── the top-k growth rule: exact top-k of |sum_b x[b,r] dy[b,c]| ─────── */
/* Defined here (no reference function exists): score[r,c] = |s| with
 * s = fmaf(x[b,r], dy[b,c], s) for b = 0..B-1 in order from s = 0; candidates
 * are the non-existing (r,c) with the k largest scores, ties toward lower
 * (r, c); returned row-major. */
typedef struct { float s; int32_t r, c; } Cand;
static int cmp_cand(const void* a, const void* b) {
    const Cand* x = (const Cand*)a; const Cand* y = (const Cand*)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    if (x->r != y->r) return x->r < y->r ? -1 : 1;
    return (x->c > y->c) - (x->c < y->c);
}
static int cmp_cand_rc(const void* a, const void* b) {
    const Cand* x = (const Cand*)a; const Cand* y = (const Cand*)b;
    if (x->r != y->r) return x->r < y->r ? -1 : 1;
    return (x->c > y->c) - (x->c < y->c);
}
int64_t o_topk_dyx_candidates(const OLayer* L, const float* x, const float* dy, int batch, int64_t k,
                              int* rows, int* cols, float* scores) {
    const int64_t n_in = L->rows, n_out = L->cols;
    const int64_t total = n_in * n_out - L->total_nnz;
    if (k > total) k = total;
    if (k <= 0) return 0;
    Cand* heap = (Cand*)malloc((size_t)(n_in * n_out - L->total_nnz + 1) * sizeof(Cand));
    uint8_t* ex = (uint8_t*)calloc((size_t)n_out + 1, 1);
    uint32_t* rc = (uint32_t*)malloc((size_t)(n_out + 1) * sizeof(uint32_t));
    int64_t m = 0;
    for (int64_t r = 0; r < n_in; ++r) {
        const int64_t n = row_nnz(L, r);
        decode_row(L, r, rc);
        for (int64_t i = 0; i < n; ++i) ex[rc[i]] = 1;
        for (int64_t c = 0; c < n_out; ++c) {
            if (ex[c]) continue;
            float s = 0.0f;
            for (int b = 0; b < batch; ++b) s = fmaf(x[(int64_t)b * n_in + r], dy[(int64_t)b * n_out + c], s);
            heap[m].s = fabsf(s); heap[m].r = (int32_t)r; heap[m].c = (int32_t)c; ++m;
        }
        for (int64_t i = 0; i < n; ++i) ex[rc[i]] = 0;
    }
    qsort(heap, (size_t)m, sizeof(Cand), cmp_cand);
    qsort(heap, (size_t)k, sizeof(Cand), cmp_cand_rc);
    for (int64_t i = 0; i < k; ++i) { rows[i] = heap[i].r; cols[i] = heap[i].c; scores[i] = heap[i].s; }
    free(heap); free(ex); free(rc);
    return k;
}

/* Applies the rule: prune the k existing synapses of smallest |FP4(w)*S(r,c)|
 * (ties toward lower (r, c)), add the k candidates with weight 0 and
 * importance fp4(score) (as delta_csr_synap_row_step stores new synapses),
 * and rebuild the arrays with delta_csr_from_absolute's headroom rules. */
typedef struct { float a; int32_t r, c; int64_t f; } Ex;
static int cmp_ex(const void* a, const void* b) {
    const Ex* x = (const Ex*)a; const Ex* y = (const Ex*)b;
    if (x->a < y->a) return -1;
    if (x->a > y->a) return 1;
    if (x->r != y->r) return x->r < y->r ? -1 : 1;
    return (x->c > y->c) - (x->c < y->c);
}
int o_topk_dyx_step(OLayer* L, const float* x, const float* dy, int batch, int64_t k) {
    if (o_b4_ntiles(L) > 0) return O_EINVAL;   /* defined on the scattered store */
    int* cr = (int*)malloc((size_t)(k + 1) * sizeof(int));
    int* cc = (int*)malloc((size_t)(k + 1) * sizeof(int));
    float* cs = (float*)malloc((size_t)(k + 1) * sizeof(float));
    const int64_t nc = o_topk_dyx_candidates(L, x, dy, batch, k, cr, cc, cs);
    const int rc = o_topk_apply(L, cr, cc, cs, nc);
    free(cr); free(cc); free(cs);
    return rc;
}

/* |sum_b x[b,r] * dy[b,c]| by the rule's ascending-b fma chain, at n given
 * positions: the scores o_topk_dyx_candidates ranks, for checking a chosen
 * set without scoring every position. */
void o_dyx_scores_at(const float* x, const float* dy, int batch, int64_t n_in, int64_t n_out, const int* rows,
                     const int* cols, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        float s = 0.0f;
        for (int b = 0; b < batch; ++b)
            s = fmaf(x[(int64_t)b * n_in + rows[i]], dy[(int64_t)b * n_out + cols[i]], s);
        out[i] = fabsf(s);
    }
}

/* The rule's second half for a given candidate list (rows / cols ascending by
 * (row, col), scores = their |dy^T x|): prune as many smallest |FP4(w) S|,
 * add the candidates, rebuild (o_topk_dyx_step = candidates + this). */
int o_topk_apply(OLayer* L, const int* cr, const int* cc, const float* cs, int64_t nc) {
    const int64_t nnz = L->total_nnz;
    if (o_b4_ntiles(L) > 0) return O_EINVAL;
    {   /* the rebuild's reserve requests against the hard limits, before any change */
        const int64_t nn0 = nnz - (nc < nnz ? nc : nnz) + nc;
        if (nn0 + 64 > L->max_val_bytes || nn0 * 8 + 4096 > L->max_idx_bytes) return O_ENOMEM;
    }
    int* p = (int*)malloc((size_t)(L->rows + 1) * sizeof(int));
    int* ix = (int*)malloc((size_t)(nnz + 1) * sizeof(int));
    float* w = (float*)malloc((size_t)(nnz + 1) * sizeof(float));
    float* im = (float*)malloc((size_t)(nnz + 1) * sizeof(float));
    to_absolute(L, p, ix, w, im);
    Ex* e = (Ex*)malloc((size_t)(nnz + 1) * sizeof(Ex));
    for (int64_t r = 0; r < L->rows; ++r)
        for (int64_t f = p[r]; f < p[r + 1]; ++f) {
            e[f].a = fabsf(w[f] * o_get_scale(L, (int)r, ix[f]));
            e[f].r = (int32_t)r; e[f].c = ix[f]; e[f].f = f;
        }
    qsort(e, (size_t)nnz, sizeof(Ex), cmp_ex);
    const int64_t npr = nc < nnz ? nc : nnz;
    uint8_t* drop = (uint8_t*)calloc((size_t)nnz + 1, 1);
    for (int64_t i = 0; i < npr; ++i) { drop[e[i].f] = 1; L->out_degree[e[i].c]--; }
    const int64_t nn = nnz - npr + nc;
    int* np_ = (int*)calloc((size_t)L->rows + 1, sizeof(int));
    int* nix = (int*)malloc((size_t)(nn + 1) * sizeof(int));
    float* nw = (float*)malloc((size_t)(nn + 1) * sizeof(float));
    float* nim = (float*)malloc((size_t)(nn + 1) * sizeof(float));
    int64_t o = 0, a = 0;
    for (int64_t r = 0; r < L->rows; ++r) {
        int64_t f = p[r];
        while (f < p[r + 1] || (a < nc && cr[a] == r)) {
            const int take_old = f < p[r + 1] && !(a < nc && cr[a] == r && cc[a] < ix[f]);
            if (take_old) {
                if (!drop[f]) { nix[o] = ix[f]; nw[o] = w[f]; nim[o] = im[f]; ++o; }
                ++f;
            } else {
                nix[o] = cc[a]; nw[o] = 0.0f; nim[o] = o_fp4_decode(o_fp4_encode(cs[a])); ++o;
                L->out_degree[cc[a]]++;
                ++a;
            }
        }
        np_[r + 1] = (int)o;
    }
    const int rc = from_absolute(L, np_, nix, nw, nim, L->rows, L->cols,
                                 (int64_t)nn * 8 + 4096, (int64_t)nn + 64, 0.2f, L->max_idx_bytes, L->max_val_bytes);
    free(p); free(ix); free(w); free(im); free(e); free(drop);
    free(np_); free(nix); free(nw); free(nim);
    return rc;
}

/* ══ std::sort restatement ══════════════════════════════════════════════════
 * The reference orders synapses by stored importance and probes by score with
 * std::sort (delta_csr_memory.hpp:1149-1152, :1182-1185), which is not stable;
 * stored importances take only 15 values, so which tied synapses are pruned is
 * decided by the sort's own permutation.  This is the introsort of GCC's
 * libstdc++ (the reference's toolchain): median-of-three pivot moved to the
 * front, unguarded Hoare partition, depth limit 2*floor(log2 n) with heapsort
 * fallback, final insertion sort with threshold 16.  Restated from the
 * algorithm so the same permutation can be produced here and on the GPU. */

static void ss_adjust_heap(int64_t* f, int64_t hole, int64_t len, int64_t val, o_less_fn lt, const void* c) {
    const int64_t top = hole;
    int64_t child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (lt(f[child], f[child - 1], c)) child--;
        f[hole] = f[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        f[hole] = f[child - 1];
        hole = child - 1;
    }
    int64_t parent = (hole - 1) / 2;
    while (hole > top && lt(f[parent], val, c)) {
        f[hole] = f[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    f[hole] = val;
}
static void ss_heapsort(int64_t* f, int64_t n, o_less_fn lt, const void* c) {
    if (n >= 2)
        for (int64_t parent = (n - 2) / 2;; --parent) {
            ss_adjust_heap(f, parent, n, f[parent], lt, c);
            if (parent == 0) break;
        }
    for (int64_t last = n; last > 1;) {
        --last;
        const int64_t v = f[last];
        f[last] = f[0];
        ss_adjust_heap(f, 0, last, v, lt, c);
    }
}
static void ss_swap(int64_t* a, int64_t* b) { const int64_t t = *a; *a = *b; *b = t; }
static void ss_introsort(int64_t* f, int64_t* l, int64_t depth, o_less_fn lt, const void* c) {
    while (l - f > 16) {
        if (depth == 0) { ss_heapsort(f, l - f, lt, c); return; }
        --depth;
        int64_t *a = f + 1, *b = f + (l - f) / 2, *z = l - 1;
        if (lt(*a, *b, c)) {
            if (lt(*b, *z, c)) ss_swap(f, b);
            else if (lt(*a, *z, c)) ss_swap(f, z);
            else ss_swap(f, a);
        } else if (lt(*a, *z, c)) ss_swap(f, a);
        else if (lt(*b, *z, c)) ss_swap(f, z);
        else ss_swap(f, b);
        int64_t *lo = f + 1, *hi = l;
        for (;;) {
            while (lt(*lo, *f, c)) ++lo;
            --hi;
            while (lt(*f, *hi, c)) --hi;
            if (!(lo < hi)) break;
            ss_swap(lo, hi);
            ++lo;
        }
        ss_introsort(lo, l, depth, lt, c);
        l = lo;
    }
}
static void ss_linear_insert(int64_t* p, o_less_fn lt, const void* c) {
    const int64_t v = *p;
    int64_t* q = p - 1;
    while (lt(v, *q, c)) { *p = *q; p = q; --q; }
    *p = v;
}
static void ss_insertion(int64_t* f, int64_t* l, o_less_fn lt, const void* c) {
    if (f == l) return;
    for (int64_t* i = f + 1; i != l; ++i) {
        if (lt(*i, *f, c)) {
            const int64_t v = *i;
            memmove(f + 1, f, (size_t)(i - f) * sizeof(int64_t));
            *f = v;
        } else ss_linear_insert(i, lt, c);
    }
}
void o_std_sort(int64_t* a, int64_t n, o_less_fn lt, const void* c) {
    if (n <= 1) return;
    int lg = 0;
    while (((int64_t)1 << (lg + 1)) <= n) ++lg;
    ss_introsort(a, a + n, 2 * (int64_t)lg, lt, c);
    if (n > 16) {
        ss_insertion(a, a + 16, lt, c);
        for (int64_t* i = a + 16; i != a + n; ++i) ss_linear_insert(i, lt, c);
    } else ss_insertion(a, a + n, lt, c);
}

/* test hook: sort indices 0..n-1 by keys ascending (desc != 0: descending) */
static int lt_f_asc(int64_t a, int64_t b, const void* c) { const float* k = (const float*)c; return k[a] < k[b]; }
static int lt_f_desc(int64_t a, int64_t b, const void* c) { const float* k = (const float*)c; return k[a] > k[b]; }
void o_std_sort_keys(const float* keys, int64_t n, int desc, int64_t* perm) {
    for (int64_t i = 0; i < n; ++i) perm[i] = i;
    o_std_sort(perm, n, desc ? lt_f_desc : lt_f_asc, keys);
}

/* ══ block4: 4x4 dense FP4 tiles ════════════════════════════════════════════
 * Logical content of the reference's Block4Store (block4.hpp:1016-1490): per
 * block-row br (input rows 4br..4br+3) the tiles in ascending block-column bc,
 * 16 slot bytes each, slot = lj*4 + li (Block4Tile::slot_index,
 * block4.hpp:309), byte = importance code << 4 | weight code.  The sparse
 * packing of tiles with <= switch_point live slots is represented by a flag
 * and its byte length (block4_sparse_packed_len, :340-343), which is all the
 * reference's accounting needs: per block-row allocations of index bytes,
 * tile bytes and tile slots, grown and shifted exactly as the reference does,
 * because they decide headroom growth, budget errors and the eviction in
 * merge_row_workspace. */

static int b4_live(const uint8_t* s) { int n = 0; for (int i = 0; i < 16; ++i) n += s[i] != 0; return n; }
static int64_t b4_sparse_len(int n) { return 1 + (n + 1) / 2 + n; }
static int64_t b4_tlen(const OTile* t) { return t->sparse ? b4_sparse_len(b4_live(t->s)) : 16; }
static int64_t b4_tile_used(const OLayer* L, int64_t br) {
    int64_t u = 0;
    for (int64_t e = 0; e < L->b4[br].n; ++e) u += b4_tlen(&L->b4[br].t[e]);
    return u;
}
static int64_t b4_idx_used(const OLayer* L, int64_t br) {
    int64_t u = 0; uint32_t prev = 0;
    for (int64_t e = 0; e < L->b4[br].n; ++e) { u += uleb_len((uint32_t)L->b4[br].t[e].bc - prev); prev = (uint32_t)L->b4[br].t[e].bc; }
    return u;
}
static int64_t b4_sum(const int64_t* a, int64_t n) { int64_t s = 0; for (int64_t i = 0; i < n; ++i) s += a[i]; return s; }
int64_t o_b4_ntiles(const OLayer* L) {
    int64_t n = 0;
    for (int64_t br = 0; br < L->b4_rows; ++br) n += L->b4[br].n;
    return n;
}

static void b4_free(OLayer* L) {
    if (L->b4) for (int64_t br = 0; br < L->b4_rows; ++br) free(L->b4[br].t);
    free(L->b4); free(L->b4_idx_alloc); free(L->b4_tile_alloc); free(L->b4_elem_alloc);
    L->b4 = NULL; L->b4_idx_alloc = L->b4_tile_alloc = L->b4_elem_alloc = NULL;
}
/* Block4Store::init, block4.hpp:1103-1117 */
static void b4_init(OLayer* L) {
    b4_free(L);
    L->b4_rows = (L->rows + 3) / 4;
    L->b4_cols = (L->cols + 3) / 4;
    L->b4 = (struct OTileRow*)calloc((size_t)L->b4_rows + 1, sizeof(struct OTileRow));
    L->b4_idx_alloc = (int64_t*)calloc((size_t)L->b4_rows + 1, 8);
    L->b4_tile_alloc = (int64_t*)calloc((size_t)L->b4_rows + 1, 8);
    L->b4_elem_alloc = (int64_t*)calloc((size_t)L->b4_rows + 1, 8);
}
static int64_t b4_find(const OLayer* L, int64_t br, int32_t bc) {
    const struct OTileRow* R = &L->b4[br];
    for (int64_t e = 0; e < R->n; ++e) {
        if (R->t[e].bc == bc) return e;
        if (R->t[e].bc > bc) break;
    }
    return -1;
}

/* block4_row_shift, block4.hpp:497-609: set one block-row's allocations to
 * the targets, never below what it uses; the last block-row never moves. */
static int b4_row_shift(OLayer* L, int64_t br, int64_t ti, int64_t tt, int64_t te) {
    const int64_t ui = b4_idx_used(L, br), ut = b4_tile_used(L, br), ue = L->b4[br].n;
    if (ti < ui) ti = ui;
    if (tt < ut) tt = ut;
    if (te < ue) te = ue;
    if (br + 1 >= L->b4_rows) return O_OK;
    if (L->b4_idx_alloc[br] != ti) {
        if (ti > L->b4_idx_alloc[br] && b4_sum(L->b4_idx_alloc, L->b4_rows) + (ti - L->b4_idx_alloc[br]) > L->b4_max_idx)
            return O_ENOMEM;
        L->b4_idx_alloc[br] = ti;
    }
    if (L->b4_tile_alloc[br] != tt) {
        if (tt > L->b4_tile_alloc[br] && b4_sum(L->b4_tile_alloc, L->b4_rows) + (tt - L->b4_tile_alloc[br]) > L->b4_max_tile)
            return O_ENOMEM;
        L->b4_tile_alloc[br] = tt;
    }
    L->b4_elem_alloc[br] = te;
    return O_OK;
}
/* block4_grow_last_row, block4.hpp:611-646 */
static int b4_grow_last(OLayer* L, int64_t ti, int64_t tt, int64_t te) {
    const int64_t r = L->b4_rows - 1;
    if (r < 0) return O_OK;
    if (ti > L->b4_idx_alloc[r]) {
        if (b4_sum(L->b4_idx_alloc, L->b4_rows) + (ti - L->b4_idx_alloc[r]) > L->b4_max_idx) return O_ENOMEM;
        L->b4_idx_alloc[r] = ti;
    }
    if (tt > L->b4_tile_alloc[r]) {
        if (b4_sum(L->b4_tile_alloc, L->b4_rows) + (tt - L->b4_tile_alloc[r]) > L->b4_max_tile) return O_ENOMEM;
        L->b4_tile_alloc[r] = tt;
    }
    if (te > L->b4_elem_alloc[r]) L->b4_elem_alloc[r] = te;
    return O_OK;
}
/* block4_ensure_row_headroom, block4.hpp:648-668: room for one more tile */
static int b4_ensure_headroom(OLayer* L, int64_t br) {
    const int64_t ti = L->b4_idx_alloc[br] + 5, tt = L->b4_tile_alloc[br] + 1, te = L->b4_elem_alloc[br] + 1;
    return br + 1 < L->b4_rows ? b4_row_shift(L, br, ti, tt, te) : b4_grow_last(L, ti, tt, te);
}
/* block4_row_insert_tile, block4.hpp:670-771: an empty sparse tile (1 byte) */
static int b4_insert_tile(OLayer* L, int64_t br, int32_t bc) {
    struct OTileRow* R = &L->b4[br];
    int64_t p = 0;
    while (p < R->n && R->t[p].bc < bc) ++p;
    if (p < R->n && R->t[p].bc == bc) return 0;
    const uint32_t prev = p > 0 ? (uint32_t)R->t[p - 1].bc : 0u;
    int64_t delta = uleb_len((uint32_t)bc - prev);
    if (p < R->n) delta += uleb_len((uint32_t)R->t[p].bc - (uint32_t)bc) - uleb_len((uint32_t)R->t[p].bc - prev);
    if (delta > 0 && delta > L->b4_idx_alloc[br] - b4_idx_used(L, br)) return 0;
    if (R->n >= L->b4_elem_alloc[br]) return 0;
    if (1 > L->b4_tile_alloc[br] - b4_tile_used(L, br)) return 0;
    if (R->n + 1 > R->cap) {
        R->cap = R->cap ? R->cap * 2 : 8;
        R->t = (OTile*)realloc(R->t, (size_t)R->cap * sizeof(OTile));
    }
    memmove(R->t + p + 1, R->t + p, (size_t)(R->n - p) * sizeof(OTile));
    memset(&R->t[p], 0, sizeof(OTile));
    R->t[p].bc = bc;
    R->t[p].sparse = 1;
    R->n++;
    return 1;
}
/* Block4Store::get_or_create, block4.hpp:1168-1184 */
static int b4_get_or_create(OLayer* L, int64_t br, int32_t bc, int64_t* e) {
    *e = b4_find(L, br, bc);
    if (*e >= 0) return O_OK;
    if (!b4_insert_tile(L, br, bc)) {
        const int rc = b4_ensure_headroom(L, br);
        if (rc) return rc;
        b4_insert_tile(L, br, bc);
    }
    *e = b4_find(L, br, bc);
    return O_OK;
}
/* commit_dirty_sparse_tile, block4.hpp:1223-1268: repack, sparse iff live <=
 * switch_point; growth past the row's headroom takes the shortfall from the
 * buffer (block4_resize_tile_in_row, :906-957) or, over budget, is dropped. */
static void b4_commit(OLayer* L, int64_t br, int64_t e, const uint8_t* s) {
    OTile* t = &L->b4[br].t[e];
    const int n = b4_live(s);
    const int sp = (uint32_t)n <= L->b4_switch;
    const int64_t nl = sp ? b4_sparse_len(n) : 16, cl = b4_tlen(t);
    if (nl > cl) {
        const int64_t head = L->b4_tile_alloc[br] - b4_tile_used(L, br);
        if (nl - cl > head) {
            const int64_t sf = nl - cl - head;
            if (b4_sum(L->b4_tile_alloc, L->b4_rows) + sf > L->b4_max_tile) { L->b4_dropped++; return; }
            L->b4_tile_alloc[br] += sf;
        }
    }
    memcpy(t->s, s, 16);
    t->sparse = (uint8_t)sp;
}
/* a write through a Block4TileHandle: sparse tiles are unpacked to scratch
 * and committed when the handle dies; dense tiles are written in place */
static void b4_write(OLayer* L, int64_t br, int64_t e, const uint8_t* s) {
    OTile* t = &L->b4[br].t[e];
    if (t->sparse) b4_commit(L, br, e, s);
    else memcpy(t->s, s, 16);
}
/* Block4Store::maybe_compress, block4.hpp:1193-1206 */
static void b4_maybe_compress(OLayer* L, int64_t br, int64_t e) {
    OTile* t = &L->b4[br].t[e];
    if (t->sparse || (uint32_t)b4_live(t->s) > L->b4_switch) return;
    t->sparse = 1;
}
/* Block4Store::erase -> block4_row_remove_tile, block4.hpp:773-888 */
static void b4_erase(OLayer* L, int64_t br, int32_t bc) {
    const int64_t e = b4_find(L, br, bc);
    if (e < 0) return;
    struct OTileRow* R = &L->b4[br];
    memmove(R->t + e, R->t + e + 1, (size_t)(R->n - e - 1) * sizeof(OTile));
    R->n--;
}

/* block4_expand_headroom, delta_csr_memory.hpp:769-823 (compact_block4 is
 * blank_fraction 0, min_slack 0) */
int o_b4_expand_headroom(OLayer* L, float bf, int64_t min_slack) {
    if (L->b4_rows == 0) return O_OK;
    int64_t total = 0;
    int64_t* na = (int64_t*)malloc((size_t)L->b4_rows * 8);
    for (int64_t br = 0; br < L->b4_rows; ++br) {
        const int64_t rb = b4_tile_used(L, br);
        na[br] = rb + (int64_t)((float)rb * bf) + min_slack;
        total += na[br];
    }
    if (total > L->b4_max_tile) { free(na); return O_ENOMEM; }
    memcpy(L->b4_tile_alloc, na, (size_t)L->b4_rows * 8);
    free(na);
    return O_OK;
}
/* Block4Store::equalize_step, block4.hpp:1208-1221 */
int o_b4_equalize_step(OLayer* L, int64_t row) {
    const int64_t R = L->b4_rows;
    if (R == 0) return O_OK;
    row %= R;
    const int64_t ti = (b4_sum(L->b4_idx_alloc, R) + R - 1) / R;
    const int64_t tt = (b4_sum(L->b4_tile_alloc, R) + R - 1) / R;
    const int64_t te = (b4_sum(L->b4_elem_alloc, R) + R - 1) / R;
    return b4_row_shift(L, row, ti, tt, te);
}
void o_b4_set_switch_point(OLayer* L, uint32_t v) { L->b4_switch = v; }

/* block4_load_dense, delta_csr_memory.hpp:843-945, via load_dense_codes
 * (cpu_backend.cpp:910-921): every (br, bc) tile is created, codes written
 * raw (weight | importance << 4), then block4_expand_headroom(0.2, 16);
 * out_degree = n_in for every column.  The scattered CSR is left as is. */
int o_load_dense_codes(OLayer* L, const uint8_t* wc, const uint8_t* ic) {
    const int64_t n_in = L->rows, n_out = L->cols;
    b4_init(L);
    const int64_t BR = L->b4_rows, BC = L->b4_cols;
    const int64_t dense = BR * BC * 16;
    L->b4_max_idx = BR * BC * 16;
    L->b4_max_tile = (int64_t)((double)dense * (1.0 + (double)0.2f)) + BR * 16;
    for (int64_t br = 0; br < BR; ++br) {
        for (int64_t bc = 0; bc < BC; ++bc) {
            int64_t e;
            const int rc = b4_get_or_create(L, br, (int32_t)bc, &e);
            if (rc) return rc;
            uint8_t s[16];
            memcpy(s, L->b4[br].t[e].s, 16);
            for (int64_t row = br * 4; row < br * 4 + 4 && row < n_in; ++row)
                for (int64_t col = bc * 4; col < bc * 4 + 4 && col < n_out; ++col) {
                    const int64_t i = row * n_out + col;
                    s[B4_SLOT(row - br * 4, col - bc * 4)] = (uint8_t)(wc[i] | (ic[i] << 4));
                }
            b4_write(L, br, e, s);
        }
    }
    const int rc = o_b4_expand_headroom(L, 0.2f, 16);
    for (int64_t c = 0; c < n_out; ++c) L->out_degree[c] = (int)n_in;
    return rc;
}

/* ── block4 state export ─────────────────────────────────────────────────── */
void o_b4_export(const OLayer* L, int* br_out, int* bc_out, uint8_t* slots, uint8_t* sparse) {
    int64_t t = 0;
    for (int64_t br = 0; br < L->b4_rows; ++br)
        for (int64_t e = 0; e < L->b4[br].n; ++e, ++t) {
            br_out[t] = (int)br; bc_out[t] = L->b4[br].t[e].bc;
            memcpy(slots + 16 * t, L->b4[br].t[e].s, 16);
            if (sparse) sparse[t] = L->b4[br].t[e].sparse;
        }
}
/* per block-row: idx alloc, idx used, tile alloc, tile used, elem alloc, tiles */
void o_b4_rows(const OLayer* L, int64_t* out) {
    for (int64_t br = 0; br < L->b4_rows; ++br) {
        out[6 * br + 0] = L->b4_idx_alloc[br]; out[6 * br + 1] = b4_idx_used(L, br);
        out[6 * br + 2] = L->b4_tile_alloc[br]; out[6 * br + 3] = b4_tile_used(L, br);
        out[6 * br + 4] = L->b4_elem_alloc[br]; out[6 * br + 5] = L->b4[br].n;
    }
}
/* Block4View counters (cpu_backend.cpp:51-98): tiles, live synapses,
 * switch_point, dropped_growth_events, row_merge_overflow_events,
 * row_merge_overflow_bytes_dropped, used_bytes, alloc_bytes */
void o_b4_view(const OLayer* L, int64_t* v) {
    int64_t live = 0, used = 0;
    for (int64_t br = 0; br < L->b4_rows; ++br) {
        for (int64_t e = 0; e < L->b4[br].n; ++e) live += b4_live(L->b4[br].t[e].s);
        used += b4_tile_used(L, br);
    }
    v[0] = o_b4_ntiles(L); v[1] = live; v[2] = L->b4_switch; v[3] = (int64_t)L->b4_dropped;
    v[4] = (int64_t)L->b4_ovf_events; v[5] = (int64_t)L->b4_ovf_bytes; v[6] = used;
    v[7] = b4_sum(L->b4_tile_alloc, L->b4_rows);
}

/* ── block4 forward, linear_disldo.hpp:128-339 (num_cpus = 1) ───────────── */
static void b4_forward(const OLayer* L, const float* x, int batch, float* y) {
    const int64_t n_in = L->rows, n_out = L->cols;
    if (o_b4_ntiles(L) == 0) return;
    float* mo = (float*)calloc((size_t)batch * n_out + 1, sizeof(float));
    for (int64_t br = 0; br < L->b4_rows; ++br)
        for (int64_t e = 0; e < L->b4[br].n; ++e) {
            const OTile* t = &L->b4[br].t[e];
            for (int lj = 0; lj < 4; ++lj) {
                const int64_t col = (int64_t)t->bc * 4 + lj;
                if (col >= n_out) continue;
                float w4[4]; int64_t ri[4];
                for (int li = 0; li < 4; ++li) {
                    const int64_t row = br * 4 + li;
                    if (row < n_in) { w4[li] = o_fp4_decode(t->s[B4_SLOT(li, lj)] & 0xF) * o_get_scale(L, (int)row, (int)col); ri[li] = row; }
                    else { w4[li] = 0.0f; ri[li] = 0; }
                }
                for (int b = 0; b < batch; ++b) {
                    const float* xr = x + (int64_t)b * n_in;
                    /* the reference build's evaluation of acc += w4[li]*x (li = 0..3) */
                    const float acc = fmaf(w4[0], xr[ri[0]], w4[1] * xr[ri[1]]) + fmaf(w4[2], xr[ri[2]], w4[3] * xr[ri[3]]);
                    mo[(int64_t)b * n_out + col] += acc;
                }
            }
        }
    for (int64_t i = 0; i < (int64_t)batch * n_out; ++i) y[i] += mo[i];
    free(mo);
}

/* ── block4 backward, linear_disldo.hpp:939-1951 (num_cpus = 1) ─────────── */
/* Block4Vec horizontal sum of the per-row scale-gradient terms
 * (block4_vec_hsum, block4.hpp:75-77) as the reference's build evaluates it:
 * lanes 0+2 and 1+3 first (pinned against the reference build) */
static inline float b4_hsum(const float* p) { return (p[0] + p[2]) + (p[1] + p[3]); }

static void b4_true_importance_evict(OLayer* L, int64_t br, OTile* ws, int64_t n) {
    /* Block4Store::merge_row_workspace, block4.hpp:1368-1465: while the row's
     * packed bytes exceed its allocation, zero the live slot of smallest
     * |decoded importance * importance_scale(row) * output_importance_scale(col)|
     * (first in tile, li, lj order on ties) and repack that tile. */
    const int64_t cap = L->b4_tile_alloc[br];
    for (;;) {
        int64_t used = 0;
        for (int64_t e = 0; e < n; ++e) used += b4_tlen(&ws[e]);
        if (used <= cap) break;
        double best = -1.0; int64_t be = 0; int bli = 0, blj = 0;
        for (int64_t e = 0; e < n; ++e)
            for (int li = 0; li < 4; ++li)
                for (int lj = 0; lj < 4; ++lj) {
                    const uint8_t byte = ws[e].s[B4_SLOT(li, lj)];
                    if (byte == 0) continue;
                    const int64_t row = br * 4 + li, col = (int64_t)ws[e].bc * 4 + lj;
                    const double ti = (double)o_fp4_decode((uint8_t)((byte >> 4) & 0xF)) *
                                      (double)o_get_importance_scale(L, (int)row) *
                                      (double)o_get_output_importance_scale(L, (int)col);
                    const double a = fabs(ti);
                    if (best < 0.0 || a < best) { best = a; be = e; bli = li; blj = lj; }
                }
        if (best < 0.0) break;
        ws[be].s[B4_SLOT(bli, blj)] = 0;
        ws[be].sparse = (uint32_t)b4_live(ws[be].s) <= L->b4_switch;
    }
    int64_t used = 0, fit = 0, ft = 0;
    for (int64_t e = 0; e < n; ++e) used += b4_tlen(&ws[e]);
    for (int64_t e = 0; e < n; ++e) {
        const int64_t tl = b4_tlen(&ws[e]);
        if (fit + tl > cap) break;
        fit += tl; ++ft;
    }
    if (ft < n) { L->b4_ovf_events++; L->b4_ovf_bytes += (uint64_t)(used - fit); }
}

static void b4_backward(OLayer* L, const float* x, const float* dy, int batch, float lr, int lr_per_row_nnz,
                        int damp, float beta2, float eps, float* dx, float* colg, float* colc, uint64_t call) {
    const int64_t n_in = L->rows, n_out = L->cols, rank = L->rank;
    if (o_b4_ntiles(L) == 0) return;
    uint32_t* rlc = (uint32_t*)calloc((size_t)n_in + 1, sizeof(uint32_t));
    for (int64_t br = 0; br < L->b4_rows; ++br) {
        if (L->b4[br].n == 0) continue;
        for (int li = 0; li < 4; ++li)
            if (br * 4 + li < n_in) rlc[br * 4 + li] = (uint32_t)L->b4[br].n * 4u;
    }
    double* trg = (double*)calloc((size_t)(n_in * rank) + 1, sizeof(double));
    double* trc = (double*)calloc((size_t)(n_in * rank) + 1, sizeof(double));
    const int training = lr != 0.0f;
    for (int64_t br = 0; br < L->b4_rows; ++br) {
        struct OTileRow* R = &L->b4[br];
        if (R->n == 0) continue;
        OTile* ws = (OTile*)malloc((size_t)R->n * sizeof(OTile));
        memcpy(ws, R->t, (size_t)R->n * sizeof(OTile));
        for (int64_t e = 0; e < R->n; ++e) {
            uint8_t* td = ws[e].s;
            const int64_t bc = ws[e].bc;
            int dirty = 0;
            for (int li = 0; li < 4; ++li) {
                const int64_t row = br * 4 + li;
                if (row >= n_in) continue;
                const uint32_t nnz_row = rlc[row];
                if (nnz_row == 0) continue;
                const float imp_scale = o_get_importance_scale(L, (int)row);
                const float eff_lr = lr_per_row_nnz ? lr / (float)nnz_row : lr;
                float vsk[4];
                for (int64_t k = 0; k < rank; ++k) vsk[k] = o_get_value_scale_k(L, (int)row, (int)k);
                int64_t col4[4]; int valid[4];
                float S4[4], cis4[4], quant[4], ci[4], qorig[4], osk[4][4];
                for (int lj = 0; lj < 4; ++lj) {
                    const int64_t col = bc * 4 + lj;
                    valid[lj] = col < n_out;
                    if (!valid[lj]) {
                        col4[lj] = 0; S4[lj] = cis4[lj] = quant[lj] = ci[lj] = qorig[lj] = 0.0f;
                        for (int64_t k = 0; k < rank; ++k) osk[k][lj] = 0.0f;
                        continue;
                    }
                    col4[lj] = col;
                    const uint8_t byte = td[B4_SLOT(li, lj)];
                    const float ois = o_get_output_importance_scale(L, (int)col);
                    S4[lj] = o_get_scale(L, (int)row, (int)col);
                    cis4[lj] = imp_scale * ois;
                    quant[lj] = qorig[lj] = o_fp4_decode(byte & 0xF);
                    ci[lj] = o_fp4_decode((uint8_t)(byte >> 4)) * cis4[lj];
                    for (int64_t k = 0; k < rank; ++k) osk[k][lj] = o_get_output_scale_k(L, (int)col, (int)k);
                }
                float mcol[4][4] = {{0}}, mcolc[4][4] = {{0}};
                double mrow[4] = {0, 0, 0, 0}, mrowc[4] = {0, 0, 0, 0};
                const int full = bc * 4 + 4 <= n_out;
                for (int b = 0; b < batch; ++b) {
                    const float iv = x[(int64_t)b * n_in + row];
                    float* d = &dx[(int64_t)b * n_in + row];
                    if (full) {
                        float dyv[4], g[4], qf[4], cb[4];
                        for (int lj = 0; lj < 4; ++lj) { dyv[lj] = dy[(int64_t)b * n_out + col4[lj]]; g[lj] = dyv[lj] * iv; }
                        if (training) {
                            for (int lj = 0; lj < 4; ++lj) {
                                cb[lj] = qorig[lj] * iv;
                                ci[lj] = bounded_ci(ci[lj], g[lj], cb[lj], beta2);
                                quant[lj] = fmaf(eff_lr, bounded_raw(g[lj], ci[lj], S4[lj], eps, damp), quant[lj]);
                                qf[lj] = (quant[lj] == 0.0f) ? 0.1f : quant[lj];
                            }
                            for (int64_t k = 0; k < rank; ++k) {
                                float p[4], pc[4];
                                for (int lj = 0; lj < 4; ++lj) { p[lj] = (qf[lj] * osk[k][lj]) * g[lj]; pc[lj] = (qf[lj] * osk[k][lj]) * cb[lj]; }
                                mrow[k] += (double)b4_hsum(p);
                                for (int lj = 0; lj < 4; ++lj) mcol[k][lj] = fmaf(qf[lj] * vsk[k], g[lj], mcol[k][lj]);
                                mrowc[k] += (double)b4_hsum(pc);
                                for (int lj = 0; lj < 4; ++lj) mcolc[k][lj] = fmaf(qf[lj] * vsk[k], cb[lj], mcolc[k][lj]);
                            }
                        }
                        /* hsum(quant*S*dy): the reference build forms quant*(S*dy) per lane
                         * and sums the lanes pairwise */
                        float p[4];
                        for (int lj = 0; lj < 4; ++lj) p[lj] = quant[lj] * (S4[lj] * dyv[lj]);
                        *d += (p[0] + p[1]) + (p[2] + p[3]);
                    } else {
                        for (int lj = 0; lj < 4; ++lj) {
                            if (!valid[lj]) continue;
                            const float dyv = dy[(int64_t)b * n_out + col4[lj]];
                            const float g = dyv * iv, S = S4[lj];
                            if (training) {
                                const float cb = iv * qorig[lj];
                                ci[lj] = bounded_ci(ci[lj], g, cb, beta2);
                                quant[lj] = fmaf(eff_lr, bounded_raw(g, ci[lj], S, eps, damp), quant[lj]);
                                const float qf = (quant[lj] == 0.0f) ? 0.1f : quant[lj];
                                for (int64_t k = 0; k < rank; ++k) {
                                    mrow[k] = fma((double)qf * (double)osk[k][lj], (double)g, mrow[k]);
                                    mcol[k][lj] = fmaf(qf * vsk[k], g, mcol[k][lj]);
                                    mrowc[k] = fma((double)qf * (double)osk[k][lj], (double)cb, mrowc[k]);
                                    mcolc[k][lj] = fmaf(qf * vsk[k], cb, mcolc[k][lj]);
                                }
                            }
                            *d = fmaf(quant[lj], S * dyv, *d);   /* quant*(S*dy), fused */
                        }
                    }
                }
                if (training) {
                    for (int64_t k = 0; k < rank; ++k) { trg[row * rank + k] += mrow[k]; trc[row * rank + k] += mrowc[k]; }
                    for (int lj = 0; lj < 4; ++lj) {
                        if (!valid[lj]) continue;
                        for (int64_t k = 0; k < rank; ++k) {
                            colg[col4[lj] * rank + k] += mcol[k][lj];
                            colc[col4[lj] * rank + k] += mcolc[k][lj];
                        }
                        const float imp_ratio = ci[lj] / cis4[lj];
                        uint8_t wq, iq;
                        if (L->stochastic) {
                            /* block4 draws use their own element space: bit 61 | row*n_out + col */
                            const uint64_t el = (1ULL << 61) | ((uint64_t)row * (uint64_t)n_out + (uint64_t)col4[lj]);
                            wq = o_fp4_quantize_stochastic_r(quant[lj], o_rng_draw(L->seed, call, el, 0));
                            iq = o_fp4_quantize_stochastic_r(imp_ratio, o_rng_draw(L->seed, call, el, 1));
                        } else {
                            wq = o_fp4_encode(quant[lj]);
                            iq = o_fp4_encode(imp_ratio);
                        }
                        td[B4_SLOT(li, lj)] = (uint8_t)((iq << 4) | wq);
                        dirty = 1;
                    }
                }
            }
            if (training && dirty) ws[e].sparse = (uint32_t)b4_live(td) <= L->b4_switch;
        }
        if (training) {
            b4_true_importance_evict(L, br, ws, R->n);
            memcpy(R->t, ws, (size_t)R->n * sizeof(OTile));
        }
        free(ws);
    }
    /* block4 value_scale step, linear_disldo.hpp:1882-1950 */
    if (training) {
        for (int64_t row = 0; row < n_in; ++row) {
            const uint32_t nnz_row = rlc[row];
            if (nnz_row == 0) continue;
            const float scale_eff_lr = lr / (float)nnz_row;
            for (int64_t k = 0; k < rank; ++k) {
                const double s = trg[row * rank + k], sc = trc[row * rank + k];
                if (s == 0.0 && sc == 0.0) continue;
                const int64_t i = row * rank + k;
                const float g = (float)s, c = (float)sc;
                if (!isfinite(g) || !isfinite(c)) continue;
                float* vi = &L->value_scale_importance.d[i];
                const float nv = fmaf(beta2, *vi, (1.0f - beta2) * fmaf(g, g, c * c));
                if (!isfinite(nv)) continue;
                uint32_t* st = &L->value_scale_step.d[i];
                ++(*st);
                const float bcor = 1.0f - powf(beta2, (float)(*st));
                const float hat = bcor > 0.0f ? nv / bcor : nv;
                if (!isfinite(hat)) continue;
                const float nvs = L->value_scale.d[i] - scale_eff_lr * g / (sqrtf(hat) + eps);
                if (!isfinite(nvs)) continue;
                *vi = nv;
                L->value_scale.d[i] = nvs;
            }
        }
    }
    free(rlc); free(trg); free(trc);
}

/* live block4 slots of input row r (for the dead-row test, :1961-1967) */
static int64_t b4_row_live(const OLayer* L, int64_t row) {
    if (L->b4_rows == 0) return 0;
    const int64_t br = row / 4;
    if (br >= L->b4_rows) return 0;
    return L->b4[br].n * 4;
}

/* ── scattered row edits ─────────────────────────────────────────────────── */
/* delta_csr_row_remove_col, delta_csr_memory.hpp:429-492 */
static int sc_remove_col(OLayer* L, int64_t r, uint32_t c) {
    const int64_t n = row_nnz(L, r);
    uint32_t* cols = (uint32_t*)malloc((size_t)n * 4 + 4);
    uint8_t* vals = (uint8_t*)malloc((size_t)n + 1);
    decode_row(L, r, cols);
    memcpy(vals, L->val + L->elem_start[r], (size_t)n);
    int64_t i = 0;
    while (i < n && cols[i] != c) ++i;
    int found = i < n;
    if (found) {
        memmove(cols + i, cols + i + 1, (size_t)(n - i - 1) * 4);
        memmove(vals + i, vals + i + 1, (size_t)(n - i - 1));
        row_write(L, r, cols, vals, n - 1);
    }
    free(cols); free(vals);
    return found;
}
/* delta_csr_row_insert_col, delta_csr_memory.hpp:500-585, storing
 * ValueAccessor::set(w, imp) (deterministic codes) */
static int sc_insert_col(OLayer* L, int64_t r, uint32_t c, float w, float imp) {
    const int64_t n = row_nnz(L, r);
    uint32_t* cols = (uint32_t*)malloc((size_t)n * 4 + 8);
    uint8_t* vals = (uint8_t*)malloc((size_t)n + 2);
    decode_row(L, r, cols);
    memcpy(vals, L->val + L->elem_start[r], (size_t)n);
    int64_t i = 0;
    while (i < n && cols[i] < c) ++i;
    int ok = !(i < n && cols[i] == c) && insert_fits(L, r, cols, n, c);
    if (ok) {
        memmove(cols + i + 1, cols + i, (size_t)(n - i) * 4);
        memmove(vals + i + 1, vals + i, (size_t)(n - i));
        cols[i] = c;
        vals[i] = (uint8_t)((o_fp4_encode(w) << 4) | o_fp4_encode(imp));
        row_write(L, r, cols, vals, n + 1);
    }
    free(cols); free(vals);
    return ok;
}

/* block4_demote_tile, delta_csr_memory.hpp:946-1003 */
static int b4_demote(OLayer* L, int64_t br, int32_t bc) {
    const int64_t e = b4_find(L, br, bc);
    if (e < 0) return O_OK;
    uint8_t s[16];
    memcpy(s, L->b4[br].t[e].s, 16);
    for (int li = 0; li < 4; ++li) {
        const int64_t row = br * 4 + li;
        if (row >= L->rows) continue;
        for (int lj = 0; lj < 4; ++lj) {
            const uint8_t byte = s[B4_SLOT(li, lj)];
            if (byte == 0) continue;
            const int64_t col = (int64_t)bc * 4 + lj;
            if (col >= L->cols) continue;
            if (!sc_insert_col(L, row, (uint32_t)col, o_fp4_decode(byte & 0xF), o_fp4_decode((uint8_t)(byte >> 4))))
                return O_EHEADROOM;
        }
    }
    b4_erase(L, br, bc);
    return O_OK;
}

/* block4_maybe_promote, delta_csr_memory.hpp:593-702 */
static int b4_maybe_promote(OLayer* L, int64_t row, uint32_t col) {
    const int64_t br = row / 4, bc = col / 4, li = row % 4, lj = col % 4;
    int64_t e = b4_find(L, br, (int32_t)bc);
    if (e >= 0) {
        const int64_t n = row_nnz(L, row);
        uint32_t* cols = (uint32_t*)malloc((size_t)n * 4 + 4);
        decode_row(L, row, cols);
        int64_t k = 0;
        while (k < n && cols[k] != col) ++k;
        free(cols);
        if (k == n) return O_OK;
        const uint8_t v = L->val[L->elem_start[row] + k];
        uint8_t s[16];
        memcpy(s, L->b4[br].t[e].s, 16);
        s[B4_SLOT(li, lj)] = (uint8_t)(o_fp4_encode(o_fp4_decode(v >> 4)) | (o_fp4_encode(o_fp4_decode(v & 0xF)) << 4));
        b4_write(L, br, e, s);
        b4_maybe_compress(L, br, e);
        sc_remove_col(L, row, col);
        return O_OK;
    }
    const int64_t row_lo = br * 4, row_hi = row_lo + 4 < L->rows ? row_lo + 4 : L->rows;
    const int64_t col_lo = bc * 4, col_hi = col_lo + 4 < L->cols ? col_lo + 4 : L->cols;
    int64_t fr[16], fc[16], fv[16], nf = 0;
    for (int64_t r = row_lo; r < row_hi; ++r) {
        const int64_t n = row_nnz(L, r);
        if (n == 0) continue;
        uint32_t* cols = (uint32_t*)malloc((size_t)n * 4 + 4);
        decode_row(L, r, cols);
        for (int64_t k = 0; k < n; ++k)
            if ((int64_t)cols[k] >= col_lo && (int64_t)cols[k] < col_hi && nf < 16) {
                fr[nf] = r; fc[nf] = cols[k]; fv[nf] = L->elem_start[r] + k; ++nf;
            }
        free(cols);
    }
    if (nf < 2) return O_OK;
    const int rc = b4_get_or_create(L, br, (int32_t)bc, &e);
    if (rc) return rc;
    uint8_t s[16];
    memcpy(s, L->b4[br].t[e].s, 16);
    for (int64_t f = 0; f < nf; ++f) {
        const uint8_t v = L->val[fv[f]];
        s[B4_SLOT(fr[f] - row_lo, fc[f] - col_lo)] =
            (uint8_t)(o_fp4_encode(o_fp4_decode(v >> 4)) | (o_fp4_encode(o_fp4_decode(v & 0xF)) << 4));
    }
    b4_write(L, br, e, s);
    b4_maybe_compress(L, br, e);
    for (int64_t f = 0; f < nf; ++f) sc_remove_col(L, fr[f], (uint32_t)fc[f]);
    return O_OK;
}

/* delta_csr_synap_row_step, delta_csr_memory.hpp:1019-1258, scattered and
 * block4 synapses, with the reference's std::sort orderings (o_std_sort). */
static int lt_u32_desc(int64_t a, int64_t b, const void* c) { const uint32_t* k = (const uint32_t*)c; return k[a] > k[b]; }

int o_synap_row_step(OLayer* L, int row_in, float cutoff, int max_rw, int max_prune, float imp_eps, int* did) {
    *did = 0;
    if (L->rows == 0) return O_OK;
    const int64_t r = (int64_t)row_in % L->rows;
    const int64_t n_sc = row_nnz(L, r);
    const int has_probes = L->n_probes > 0;
    const int64_t br = r / 4, li = r % 4;
    const int64_t nt = (br < L->b4_rows) ? L->b4[br].n : 0;
    const int64_t cap = n_sc + 4 * nt + 1;
    uint32_t* cols = (uint32_t*)malloc((size_t)cap * 4);
    float* imp = (float*)malloc((size_t)cap * 4);
    uint8_t* isb4 = (uint8_t*)calloc((size_t)cap, 1);
    decode_row(L, r, cols);
    for (int64_t k = 0; k < n_sc; ++k) imp[k] = o_fp4_decode(L->val[L->elem_start[r] + k] & 0xF);
    int64_t n_exist = n_sc;
    for (int64_t e = 0; e < nt; ++e)
        for (int lj = 0; lj < 4; ++lj) {
            const uint8_t byte = L->b4[br].t[e].s[B4_SLOT(li, lj)];
            if (byte == 0) continue;
            const int64_t col = (int64_t)L->b4[br].t[e].bc * 4 + lj;
            if (col >= L->cols) continue;
            cols[n_exist] = (uint32_t)col;
            imp[n_exist] = o_fp4_decode((uint8_t)(byte >> 4));
            isb4[n_exist] = 1;
            ++n_exist;
        }
    if (n_exist == 0 && !has_probes) { free(cols); free(imp); free(isb4); return O_OK; }
    /* probes of this row in COO order (:1133-1144) */
    uint32_t* pc = (uint32_t*)malloc((size_t)(L->n_probes + 1) * 4);
    float* ps = (float*)malloc((size_t)(L->n_probes + 1) * 4);
    int64_t np = 0;
    for (int64_t p = 0; p < L->n_probes; ++p)
        if (L->prow[p] == r) { pc[np] = (uint32_t)L->pcol[p]; ps[np] = L->pval[p]; ++np; }
    /* removals by stored importance ascending (:1147-1167) */
    int64_t* by = (int64_t*)malloc((size_t)(n_exist + 1) * 8);
    for (int64_t i = 0; i < n_exist; ++i) by[i] = i;
    o_std_sort(by, n_exist, lt_f_asc, imp);
    uint32_t* rmc = (uint32_t*)malloc((size_t)(n_exist + 1) * 4);
    uint8_t* rmb = (uint8_t*)malloc((size_t)(n_exist + 1));
    int64_t nrm = 0;
    for (int64_t a = 0; a < n_exist && nrm < max_prune; ++a) {
        const int64_t k = by[a];
        const int64_t keep = n_exist - nrm;
        const float fl = (imp[k] < imp_eps) ? imp_eps : imp[k];   /* std::max(imp, eps) */
        if (fl < cutoff || keep > max_rw) { rmc[nrm] = cols[k]; rmb[nrm] = isb4[k]; ++nrm; }
    }
    int64_t* rperm = (int64_t*)malloc((size_t)(nrm + 1) * 8);
    for (int64_t i = 0; i < nrm; ++i) rperm[i] = i;
    o_std_sort(rperm, nrm, lt_u32_desc, rmc);
    /* adds by score descending (:1171-1201) */
    int64_t* pidx = (int64_t*)malloc((size_t)(np + 1) * 8);
    for (int64_t i = 0; i < np; ++i) pidx[i] = i;
    o_std_sort(pidx, np, lt_f_desc, ps);
    const uint64_t slots = (uint64_t)((int64_t)max_rw - (n_exist - nrm));
    uint32_t* add_c = (uint32_t*)malloc((size_t)(np + 1) * 4);
    float* add_s = (float*)malloc((size_t)(np + 1) * 4);
    int64_t nadd = 0;
    for (int64_t a = 0; a < np; ++a) {
        if ((uint64_t)nadd >= slots) break;
        const uint32_t c = pc[pidx[a]];
        int exists = 0;
        for (int64_t i = 0; i < n_exist; ++i) if (cols[i] == c) { exists = 1; break; }
        if (!exists) { add_c[nadd] = c; add_s[nadd] = ps[pidx[a]]; ++nadd; }
    }
    int rc = O_OK;
    /* removals, highest column first (:1203-1233) */
    for (int64_t q = 0; q < nrm && rc == O_OK; ++q) {
        const uint32_t c = rmc[rperm[q]];
        if (rmb[rperm[q]]) {
            const int32_t bc = (int32_t)(c / 4);
            const int lj = (int)(c % 4);
            const int64_t e = b4_find(L, br, bc);
            int demote = 0;
            if (e >= 0 && L->b4[br].t[e].s[B4_SLOT(li, lj)] != 0) {
                uint8_t s[16];
                memcpy(s, L->b4[br].t[e].s, 16);
                s[B4_SLOT(li, lj)] = 0;
                demote = b4_live(s) < 2;
                b4_write(L, br, e, s);
            }
            if (demote) rc = b4_demote(L, br, bc);
        } else {
            sc_remove_col(L, r, c);
        }
        if (rc == O_OK && L->out_degree[c] > 0) L->out_degree[c]--;
    }
    /* inserts in score order, each followed by the block4 promotion (:1235-1255) */
    for (int64_t a = 0; a < nadd && rc == O_OK; ++a) {
        if (!sc_insert_col(L, r, add_c[a], 0.0f, add_s[a])) { rc = O_EHEADROOM; break; }
        L->out_degree[add_c[a]]++;
        rc = b4_maybe_promote(L, r, add_c[a]);
    }
    free(cols); free(imp); free(isb4); free(pc); free(ps); free(by); free(rmc); free(rmb);
    free(rperm); free(pidx); free(add_c); free(add_s);
    if (rc == O_OK) *did = 1;
    return rc;
}

/* ── sisldo_forward block4 windows, sisldo_ops.hpp:379-549 (num_cpus = 1) ──
 * Per sample, each run of input indices inside one block-row forms a window
 * of 4 input values; every tile of that block-row adds, per column, the sum
 * over its live slots of (w * value_scale(row) * output_scale(col)) * x. */
static void b4_forward_sparse(const OLayer* L, const int* ptrs, const int* idx, const float* vals, int batch,
                              float* y) {
    const int64_t n_in = L->rows, n_out = L->cols;
    if (o_b4_ntiles(L) == 0) return;
    float* mo = (float*)calloc((size_t)batch * n_out + 1, sizeof(float));
    for (int b = 0; b < batch; ++b) {
        int i = ptrs[b];
        while (i < ptrs[b + 1]) {
            const int64_t br = idx[i] / 4, lo = br * 4, hi = lo + 4;
            float local[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            int j = i;
            while (j < ptrs[b + 1] && idx[j] < hi) { local[idx[j] - lo] = vals[j]; ++j; }
            if (br < L->b4_rows && L->b4[br].n > 0) {
                for (int64_t e = 0; e < L->b4[br].n; ++e) {
                    const OTile* t = &L->b4[br].t[e];
                    for (int lj = 0; lj < 4; ++lj) {
                        const int64_t col = (int64_t)t->bc * 4 + lj;
                        if (col >= n_out) continue;
                        const float os = o_get_output_scale_k(L, (int)col, 0);
                        float acc = 0.0f;
                        for (int li = 0; li < 4; ++li) {
                            const int64_t row = br * 4 + li;
                            if (row >= n_in) continue;
                            const uint8_t byte = t->s[B4_SLOT(li, lj)];
                            if (byte == 0) continue;
                            /* acc += w * value_scale * out_scale * x as the reference's build
                             * evaluates it: fma(os*vs, x*w, acc) */
                            const float vsr = o_get_value_scale_k(L, (int)row, 0);
                            acc = fmaf(os * vsr, local[li] * o_fp4_decode(byte & 0xF), acc);
                        }
                        mo[(int64_t)b * n_out + col] += acc;
                    }
                }
            }
            i = j;
        }
    }
    for (int64_t q = 0; q < (int64_t)batch * n_out; ++q) y[q] += mo[q];
    free(mo);
}

/* ── disldo_backward_sparse_grad block4 part, sisldo_ops.hpp:835-1104 ─────
 * Per sample, per block-row: every tile whose 4-column window holds gradient
 * entries takes them; dx adds w*dy over the window; at lr != 0 each touched
 * slot gets the plain RMSprop step (no clip) and a stochastic requantize,
 * then the row's workspace merge evicts down to its allocation.  After all
 * samples: importance statistics and the rank-1 value_scale step. */
void o_set_ref_stream(OLayer* L, int on, uint64_t seed) {
    L->ref_stream = on;
    L->ref_state = (seed ^ 0x9E3779B97F4A7C15ULL) | 1ULL;
}
static uint8_t b4_qstoch(OLayer* L, float v, uint64_t call, uint64_t el, uint32_t lane) {
    if (L->ref_stream) {
        const uint32_t a = f2u(v) & 0x7FFFFFFFu;
        const uint64_t r = (a > 0x7F800000u || a >= 0x40C00000u) ? 0 : o_xorshift_next(&L->ref_state);
        return o_fp4_quantize_stochastic_r(v, r);
    }
    return o_fp4_quantize_stochastic_r(v, o_rng_draw(L->seed, call, el, lane));
}
static void b4_backward_sparse(OLayer* L, const float* x, const int* dptrs, const int* didx, const float* dvals,
                               int batch, float lr, int lr_per_row_nnz, int damp, float beta2, float eps, float* dx,
                               uint64_t call) {
    const int64_t n_in = L->rows, n_out = L->cols;
    if (o_b4_ntiles(L) == 0) return;
    double* rs = (double*)calloc((size_t)n_in + 1, sizeof(double));
    double* rc = (double*)calloc((size_t)n_in + 1, sizeof(double));
    double t_an = 0, t_ao = 0, t_sn = 0, t_so = 0; float t_mx = 0.0f;
    for (int b = 0; b < batch; ++b) {
        const int og0 = dptrs[b], og1 = dptrs[b + 1];
        double an = 0, ao = 0, sn = 0, so = 0; float mx = 0.0f;
        for (int64_t br = 0; br < L->b4_rows; ++br) {
            struct OTileRow* R = &L->b4[br];
            const int64_t nt = R->n;
            if (nt == 0) continue;
            const int64_t nnz_row = nt * 4;
            float dxa[4] = {0, 0, 0, 0};
            double rgl[4] = {0, 0, 0, 0}, rglc[4] = {0, 0, 0, 0};
            OTile* ws = (OTile*)malloc((size_t)nt * sizeof(OTile));
            memcpy(ws, R->t, (size_t)nt * sizeof(OTile));
            int og = og0;
            for (int64_t e = 0; e < nt; ++e) {
                const int64_t lo = (int64_t)ws[e].bc * 4, hi = lo + 4;
                while (og < og1 && didx[og] < lo) ++og;
                float dyl[4] = {0, 0, 0, 0};
                int any = 0;
                for (int p = og; p < og1 && didx[p] < hi; ++p) { dyl[didx[p] - lo] = dvals[p]; any = 1; }
                if (!any) continue;
                uint8_t* td = ws[e].s;
                int dirty = 0;
                for (int li = 0; li < 4; ++li) {
                    const int64_t row = br * 4 + li;
                    if (row >= n_in) continue;
                    const float in_val = x[(int64_t)b * n_in + row];
                    const float vs = o_get_value_scale_k(L, (int)row, 0);
                    const float imp_scale = o_get_importance_scale(L, (int)row);
                    const float eff_lr = lr_per_row_nnz ? lr / (float)nnz_row : lr;
                    for (int lj = 0; lj < 4; ++lj) {
                        if (dyl[lj] == 0.0f) continue;
                        const int64_t col = lo + lj;
                        if (col >= n_out) continue;
                        const uint8_t byte = td[B4_SLOT(li, lj)];
                        const float wd = o_fp4_decode(byte & 0xF);
                        const float os = o_get_output_scale_k(L, (int)col, 0);
                        const float cs = vs * os;
                        const float w = wd * cs;
                        const float dyv = dyl[lj];
                        if (lr == 0.0f) {
                            /* w*dy with w = w_dec*vs*os, as the reference's build
                             * evaluates it at lr = 0: fma(os*vs, dy*w_dec, acc) */
                            dxa[li] = fmaf(os * vs, dyv * wd, dxa[li]);
                            continue;
                        }
                        dxa[li] = fmaf(w, dyv, dxa[li]);
                        const float cis = imp_scale * o_get_output_importance_scale(L, (int)col);
                        const float imp_dec = o_fp4_decode((uint8_t)(byte >> 4));
                        const float grad = dyv * in_val;
                        float imp = imp_dec * cis;
                        const float contrib = in_val * w;
                        imp = fmaf(beta2, imp, (1.0f - beta2) * fmaf(grad, grad, contrib * contrib));
                        const float step = damp ? (-eff_lr * grad) / (sqrtf(imp) + eps) : (-eff_lr * grad);
                        const float new_w = w + step;
                        /* counter key: bit 61 | (sample, row, col) -- a slot can be
                         * updated once per sample within one call */
                        const uint64_t el = (1ULL << 61) |
                                            (((uint64_t)b * (uint64_t)n_in + (uint64_t)row) * (uint64_t)n_out + (uint64_t)col);
                        const uint8_t wq = b4_qstoch(L, new_w / cs, call, el, 0);
                        const uint8_t iq = b4_qstoch(L, imp / cis, call, el, 1);
                        td[B4_SLOT(li, lj)] = (uint8_t)((iq << 4) | wq);
                        dirty = 1;
                        const float actual = o_fp4_decode(iq) * cis, stored = imp_dec * cis;
                        an += fabs((double)actual); ao += fabs((double)stored);
                        sn += (double)actual * actual; so += (double)stored * stored;
                        if (fabsf(actual) > mx) mx = fabsf(actual);
                        rgl[li] += (double)wd * (double)os * (double)(dyv * in_val);
                        rglc[li] += (double)wd * (double)os * (double)contrib;
                    }
                }
                if (dirty) ws[e].sparse = (uint32_t)b4_live(td) <= L->b4_switch;
            }
            if (lr != 0.0f) {
                b4_true_importance_evict(L, br, ws, nt);
                memcpy(R->t, ws, (size_t)nt * sizeof(OTile));
            }
            free(ws);
            for (int li = 0; li < 4; ++li) {
                const int64_t row = br * 4 + li;
                if (row >= n_in) continue;
                dx[(int64_t)b * n_in + row] += dxa[li];
                if (lr != 0.0f) { rs[row] += rgl[li]; rc[row] += rglc[li]; }
            }
        }
        t_an += an; t_ao += ao; t_sn += sn; t_so += so;
        if (mx > t_mx) t_mx = mx;
    }
    if (lr != 0.0f) {
        L->importance_l1 += t_an - t_ao;
        L->importance_l2_sq += t_sn - t_so;
        L->importance_max_abs = fmaxf(L->importance_max_abs * L->max_abs_decay, t_mx);
        if (L->value_scale_step.n < n_in * L->rank) uvec_resize(&L->value_scale_step, n_in * L->rank, 0u);
        for (int64_t r = 0; r < n_in; ++r) {
            if (rs[r] == 0.0 && rc[r] == 0.0) continue;
            const int64_t br = r / 4;
            const int64_t nnz_row = (br < L->b4_rows ? L->b4[br].n : 0) * 4;
            if (nnz_row == 0) continue;
            const float se = lr / (float)nnz_row;
            const float g = (float)rs[r], cg = (float)rc[r];
            float* vsi = &L->value_scale_importance.d[r];
            const float nv = fmaf(beta2, *vsi, (1.0f - beta2) * fmaf(g, g, cg * cg));
            uint32_t* st = &L->value_scale_step.d[r * L->rank];
            ++(*st);
            const float bcor = 1.0f - powf(beta2, (float)(*st));
            const float hat = bcor > 0.0f ? nv / bcor : nv;
            *vsi = nv;
            L->value_scale.d[r] -= se * g / (sqrtf(hat) + eps);
        }
    }
    free(rs); free(rc);
}
