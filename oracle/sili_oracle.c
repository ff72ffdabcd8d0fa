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
};

#define NO_LIMIT INT64_MAX

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
    if (L->total_nnz > 0) {
        for (int64_t r = 0; r < n_in; ++r) {
            const int64_t nnz = row_nnz(L, r);
            if (nnz == 0) continue;
            const float eff_lr = lr_per_row_nnz ? lr / (float)nnz : lr;
            const float scale_eff_lr = lr / (float)nnz;
            const float imp_scale = o_get_importance_scale(L, (int)r);
            double sgs[4] = {0, 0, 0, 0}, sgc[4] = {0, 0, 0, 0};
            int64_t pos = L->byte_start[r]; uint32_t col = 0;
            for (int64_t vb = L->elem_start[r]; vb < L->elem_end[r]; ++vb) {
                col += uleb_get(L->idx, &pos);
                const float cw_orig = get_w(L, vb), ci_orig = get_imp(L, vb);
                const float cis = imp_scale * o_get_output_importance_scale(L, (int)col);
                float ci = ci_orig * cis;
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
            if (lr != 0.0f) {
                for (int64_t k = 0; k < rank; ++k) {
                    const int64_t i = r * rank + k;
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
    /* dead-row bootstrap, linear_disldo.hpp:1985-2042 (block4 empty) */
    if (lr != 0.0f) {
        int any_dead = 0;
        for (int64_t r = 0; r < n_in; ++r) if (row_nnz(L, r) == 0) { any_dead = 1; break; }
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
                if (row_nnz(L, r) != 0) continue;
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
                    const float nv = fmaf(beta2, *v, (1.0f - beta2) * (g * g));
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
    /* output_scale update, linear_disldo.hpp:2051-2080 */
    if (lr != 0.0f && os_train) {
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
    free(colg); free(colc);
}

/* ── sisldo_forward, sisldo_ops.hpp:198-340 (scattered part, num_cpus = 1) ─ */
void o_forward_sparse(OLayer* L, const int* ptrs, const int* idx, const float* vals, int batch, float* y) {
    const int64_t n_out = L->cols;
    memset(y, 0, (size_t)batch * n_out * sizeof(float));
    if (L->total_nnz == 0) return;
    for (int b = 0; b < batch; ++b) {
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
    L->call++;
    if (L->total_nnz == 0) return;
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

/* delta_csr_synap_row_step, delta_csr_memory.hpp:1019-1258, scattered storage.
 * Sort ties: the reference uses std::sort (unstable); this restatement breaks
 * importance ties by stored position and score ties by probe order, which is
 * what std::sort yields for rows of at most 16 entries (insertion sort). */
typedef struct { float key; int64_t pos; } KP;
static int cmp_kp_asc(const void* a, const void* b) {
    const KP* x = (const KP*)a; const KP* y = (const KP*)b;
    if (x->key < y->key) return -1;
    if (x->key > y->key) return 1;
    return (x->pos > y->pos) - (x->pos < y->pos);
}
static int cmp_kp_desc(const void* a, const void* b) {
    const KP* x = (const KP*)a; const KP* y = (const KP*)b;
    if (x->key > y->key) return -1;
    if (x->key < y->key) return 1;
    return (x->pos > y->pos) - (x->pos < y->pos);
}
static int cmp_u32_desc(const void* a, const void* b) {
    const uint32_t x = *(const uint32_t*)a, y = *(const uint32_t*)b;
    return (x < y) - (x > y);
}

int o_synap_row_step(OLayer* L, int row_in, float cutoff, int max_rw, int max_prune, float imp_eps, int* did) {
    *did = 0;
    if (L->rows == 0) return O_OK;
    const int64_t r = (int64_t)row_in % L->rows;
    const int64_t n = row_nnz(L, r);
    const int has_probes = L->n_probes > 0;
    if (n == 0 && !has_probes) return O_OK;
    uint32_t* cols = (uint32_t*)malloc((size_t)(n + L->n_probes + 1) * sizeof(uint32_t));
    uint8_t* vals = (uint8_t*)malloc((size_t)(n + L->n_probes + 1));
    decode_row(L, r, cols);
    memcpy(vals, L->val + L->elem_start[r], (size_t)n);
    /* step 2: probes of this row, in COO order (:1133-1144) */
    KP* pr = (KP*)malloc((size_t)(L->n_probes + 1) * sizeof(KP));
    int64_t np = 0;
    for (int64_t p = 0; p < L->n_probes; ++p)
        if (L->prow[p] == r) { pr[np].key = L->pval[p]; pr[np].pos = p; ++np; }
    /* step 3: removals (:1147-1167) */
    KP* bi = (KP*)malloc((size_t)(n + 1) * sizeof(KP));
    for (int64_t i = 0; i < n; ++i) { bi[i].key = o_fp4_decode(vals[i] & 0xF); bi[i].pos = i; }
    qsort(bi, (size_t)n, sizeof(KP), cmp_kp_asc);
    uint8_t* rm = (uint8_t*)calloc((size_t)n + 1, 1);
    int64_t nrm = 0;
    for (int64_t a = 0; a < n && nrm < max_prune; ++a) {
        const int64_t k = bi[a].pos;
        const int64_t keep = n - nrm;
        const float imp = bi[a].key;
        const float fl = (imp < imp_eps) ? imp_eps : imp;   /* std::max(imp, eps) */
        if (fl < cutoff || keep > max_rw) { rm[k] = 1; ++nrm; }
    }
    /* step 4: adds (:1171-1201) */
    qsort(pr, (size_t)np, sizeof(KP), cmp_kp_desc);
    const int64_t slots = (int64_t)max_rw - (n - nrm);
    uint32_t* add_c = (uint32_t*)malloc((size_t)(np + 1) * sizeof(uint32_t));
    float* add_s = (float*)malloc((size_t)(np + 1) * sizeof(float));
    int64_t nadd = 0;
    for (int64_t a = 0; a < np; ++a) {
        if ((uint64_t)nadd >= (uint64_t)slots) break;
        const uint32_t c = (uint32_t)L->pcol[pr[a].pos];
        int exists = 0;
        for (int64_t i = 0; i < n; ++i) if (cols[i] == c) { exists = 1; break; }
        if (!exists) { add_c[nadd] = c; add_s[nadd] = pr[a].key; ++nadd; }
    }
    /* step 5: apply removes high col first (:1203-1233) */
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i) {
        if (rm[i]) { if (L->out_degree[cols[i]] > 0) L->out_degree[cols[i]]--; continue; }
        cols[m] = cols[i]; vals[m] = vals[i]; ++m;
    }
    int rc = row_write(L, r, cols, vals, m);
    /* step 6: inserts in score order (:1235-1255) */
    for (int64_t a = 0; a < nadd && rc == O_OK; ++a) {
        const uint32_t c = add_c[a];
        int64_t i = 0;
        while (i < m && cols[i] < c) ++i;
        if (i < m && cols[i] == c) { rc = O_EHEADROOM; break; }   /* insert_col false -> throw */
        if (!insert_fits(L, r, cols, m, c)) { rc = O_EHEADROOM; break; }
        memmove(cols + i + 1, cols + i, (size_t)(m - i) * sizeof(uint32_t));
        memmove(vals + i + 1, vals + i, (size_t)(m - i));
        cols[i] = c;
        vals[i] = (uint8_t)((o_fp4_encode(0.0f) << 4) | o_fp4_encode(add_s[a]));
        ++m;
        rc = row_write(L, r, cols, vals, m);
        if (rc == O_OK) L->out_degree[c]++;
    }
    (void)cmp_u32_desc;
    free(cols); free(vals); free(pr); free(bi); free(rm); free(add_c); free(add_s);
    if (rc == O_OK) *did = 1;
    return rc;
}

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
int64_t o_export_nnz(const OLayer* L) { return L->total_nnz; }
void o_export(const OLayer* L, int* ptrs, int* idx, float* w, float* imp) { to_absolute(L, ptrs, idx, w, imp); }

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

/* ── BASELINE config-3 rule: exact top-k of |sum_b x[b,r] dy[b,c]| ─────── */
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
    const int64_t nnz = L->total_nnz;
    int* cr = (int*)malloc((size_t)(k + 1) * sizeof(int));
    int* cc = (int*)malloc((size_t)(k + 1) * sizeof(int));
    float* cs = (float*)malloc((size_t)(k + 1) * sizeof(float));
    const int64_t nc = o_topk_dyx_candidates(L, x, dy, batch, k, cr, cc, cs);
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
    free(cr); free(cc); free(cs); free(p); free(ix); free(w); free(im); free(e); free(drop);
    free(np_); free(nix); free(nw); free(nim);
    return rc;
}
