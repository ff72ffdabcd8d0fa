// Host side of sili_b200: per-layer device state and the C ABI declared in
// include/sili_b200.h.  Mirrors sili._cpu.SparseLinearLayerImpl
// (sili/cpu_backend.cpp:349-1013); every compute path runs CUDA kernels.
#include "../../include/sili_b200.h"
#include "common.cuh"
#include "kernels.cuh"

#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

using namespace sili;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define CK(x)                                                                                   \
    do {                                                                                        \
        cudaError_t e_ = (x);                                                                   \
        if (e_ != cudaSuccess) return fail(SILI_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define RC(x)                   \
    do {                        \
        int r_ = (x);           \
        if (r_) return r_;      \
    } while (0)

// Grow-only device buffer.
template <typename T>
struct DBuf {
    T* p = nullptr;
    int64_t cap = 0;
    DBuf() = default;
    DBuf(const DBuf&) = delete;
    DBuf& operator=(const DBuf&) = delete;
    ~DBuf() { if (p) cudaFree(p); }
    int reserve(int64_t n) {            // contents not preserved
        if (n <= cap) return SILI_OK;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        const int64_t want = std::max<int64_t>(n, 1);
        cudaError_t e = cudaMalloc((void**)&p, (size_t)want * sizeof(T));
        if (e != cudaSuccess) return fail(SILI_ECUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        cap = want;
        return SILI_OK;
    }
    int grow(int64_t n, int64_t keep, cudaStream_t s) {   // preserves [0, keep)
        if (n <= cap) return SILI_OK;
        T* q = nullptr;
        const int64_t want = std::max<int64_t>(n, cap + cap / 2);
        cudaError_t e = cudaMalloc((void**)&q, (size_t)want * sizeof(T));
        if (e != cudaSuccess) return fail(SILI_ECUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        if (p && keep > 0) {
            e = cudaMemcpyAsync(q, p, (size_t)keep * sizeof(T), cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return fail(SILI_ECUDA, cudaGetErrorString(e));
            cudaStreamSynchronize(s);
        }
        if (p) cudaFree(p);
        p = q;
        cap = want;
        return SILI_OK;
    }
    void swap(DBuf& o) { std::swap(p, o.p); std::swap(cap, o.cap); }
    void release() {                    // frees the memory (waits for its users, as cudaFree does)
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
};

// FP4_TABLE (fp4quant.hpp:16-33), code 8 = NaN
float fp4_decode_host(uint32_t code) {
    static const float t[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f, NAN,
                                -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
    return t[code & 15u];
}

bool is_device_ptr(const void* ptr) {
    if (!ptr) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

struct sili_layer {
    int dev = 0;
    cudaStream_t stream = nullptr;
    int64_t rows = 0, cols = 0;
    int rank = 1;
    bool stochastic = true;
    uint64_t seed = 0x5EEDu, call = 0;
    // delta-CSR (DeltaCSRWeights, delta_csr_types.hpp:898-939)
    DBuf<uint8_t> idx, val;
    int64_t idx_n = 0, val_n = 0;
    DBuf<int64_t> bs, be, es, ee;
    int64_t total_nnz = 0;
    int64_t max_idx_bytes = INT64_MAX, max_val_bytes = INT64_MAX;
    int64_t idx_budget = 4096, val_budget = 64;
    // scales (SparseLinearWeightsDelta, delta_csr_types.hpp:1004-1240).  The
    // device arrays are full size and hold the reference's default read value
    // where the reference's lazily-sized vector has no entry yet; n_vs / n_os
    // track that vector's logical size, because growing it fills with 1.0 even
    // at components k >= 1 (set_value_scale_raw_k, :1105-1110).
    DBuf<float> vs, os, vsi, osi, vsm, is, ois;
    DBuf<uint32_t> vstep, ostep;
    int64_t n_vs = 0, n_os = 0;
    bool os_trainable = false;
    int scale_policy = SILI_SCALE_POLICY_RMSPROP;   // the class's ScalePolicy (cpu_backend.cpp:993-1013)
    DBuf<float> def_cw, def_ci;   // a Resync update's deferred true-units state, by value position
    DBuf<float> in_acc, grad_acc;
    DBuf<int> out_degree;
    DBuf<int> prow, pcol;
    DBuf<float> pval;
    // build_probes' scratch, kept between calls (allocating it per call cost
    // more than the probe kernels)
    DBuf<float> pb_keys;
    DBuf<int> pb_iota, pb_in, pb_out, pb_flags, pb_pos, pb_tr, pb_tc, pb_counts;
    DBuf<float> pb_tv;
    int64_t n_probes = 0;
    // running stats (delta_csr_types.hpp:1265-1281)
    double st[4] = {0, 0, 0, 0};   // value_l1, value_l2_sq, importance_l1, importance_l2_sq
    float st_vmax = 0.f, st_imax = 0.f, max_abs_decay = 1.f;
    DBuf<double> d_st;             // pending importance l1/l2 deltas
    DBuf<float> d_stmax;
    DBuf<unsigned long long> d_dyflag;   // = call tag when that call's dy held an inf or NaN
    bool st_pending = false;
    // derived index
    bool aux_dirty = true;
    DBuf<int> rowptr, abs_cols, frow, fvpos, colcount, colptr, crow, cvpos, sort_k, sort_ko, sort_v, sort_vo;
    DBuf<int> colptr_x, padcnt;   // exact column offsets, padded counts
    DBuf<int> fcpos;              // padded CSC position of each synapse (row-major order)
    DBuf<int> cpack;              // packed CSC (row << 4 | weight code) for the row-tiled forward
    bool pack_valid = false;      // cpack matches the current weight codes
    DBuf<uint8_t> cub_tmp;
    // scratch
    DBuf<float> xT, dyT, dxT, colg, colc, ytmp, x_stage, dy_stage, dx_stage;
    DBuf<float> xsT;              // the last forward_sparse input, densified and transposed
    DBuf<float> fold_raw;         // sili_folded_forward's per-suffix outputs before the sums
    int sparse_batch = 0;
    bool has_dead_rows = false;
    // column shard (sili_layer_set_row_shard): global synapse count per row,
    // global column count, whether some row has none anywhere; the
    // arguments of the last shard backward, which its row steps reuse
    DBuf<int> shard_nnz;
    int64_t shard_n_out = 0;
    bool shard_on = false, shard_any_dead = false;
    DBuf<double> rpart;
    float sh_lr = 0.f, sh_beta2 = 0.f, sh_eps = 0.f;
    unsigned sh_flags = 0;
    int sh_batch = -1;
    DBuf<uint8_t> presT, presX;
    DBuf<double> dS, sgs, sgc;
    DBuf<int> i_tmp0, i_tmp1, i_tmp2;
    DBuf<float> f_tmp0;
    int last_batch = 0;
    DBuf<float> pow_tab;
    float pow_beta2 = NAN;
    int pow_n = 0;
    // block4 store (Block4Store, block4.hpp:1016-1490); device layout in B4View
    int64_t b4_BR = 0, b4_BC = 0;
    DBuf<int64_t> b4_es, b4_alloc, b4_used;
    DBuf<int> b4_nt, b4_bc;
    DBuf<uint4> b4_tile;
    DBuf<uint8_t> b4_sparse;
    DBuf<unsigned long long> b4_cnt;
    DBuf<float> b4_hs;       // per-tile dx sums of the tile-parallel update
    DBuf<double> b4_mr;      // per-tile value_scale sums of the tile-parallel update
    DBuf<float> b4_mc;       // per-slot output_scale sums of the tile-parallel update
    DBuf<int> b4_cptr, b4_ctile, b4_cbr, b4_keys, b4_keys_o, b4_perm, b4_perm_o, b4_slots, b4_brs, b4_off;
    int64_t b4_ntiles = 0;                 // live tiles (host mirror)
    int64_t b4_max_idx = INT64_MAX, b4_max_tile = INT64_MAX;
    uint32_t b4_switch = 10;
    bool b4_dirty = true;                  // tile column index stale
    bool b4_tc = false;                    // block4 forward on the tensor cores (tolerance contract)
    DBuf<uint16_t> b4_xs;                  // its split activations
    DBuf<float> b4_part;                   // its per-slice partial sums
    DBuf<unsigned int> tc_err;             // set by a kernel whose bounded device-side wait gave up
    DBuf<int> b4_pmap;                     // its panel map (tile slot per 32 x 16 block cell)
    bool b4_pmap_dirty = true;             // the tile layout changed since the map was built
    DBuf<int> b4_pmapT;                    // the lr = 0 dx's panel map (block-rows along the panel)
    bool b4_pmapT_dirty = true;
    // synaptogenesis working set (probe-by-row index, scratch, snapshot)
    struct SynStateT {
        DBuf<int> pr_ptr, keys, keys_o, ids, ids_o, od0, od_decs;
        DBuf<uint8_t> scratch, did;
        DBuf<long long> res;
        DBuf<uint8_t> s_idx, s_val, s_be, s_ee, s_od, s_nt, s_bc, s_tile, s_sp, s_alloc, s_cnt;
        int64_t m = 0, p = 0, stride = 0;
    } syn;
    // top-k |dy^T x| working set
    struct TopkStateT {
        DBuf<uint32_t> bits, keys, pk, pk_o;
        DBuf<unsigned int> hist;
        DBuf<int64_t> cand, cand_o, eq, nsel;
        DBuf<int> pid, pid_o, cptr, cnt, nptr;
        DBuf<uint8_t> drop;
        DBuf<SelState> sel;
        DBuf<unsigned long long> nge;
        DBuf<int> di, nidx;            // kept across calls: no allocation per step
        DBuf<float> dw, dm, nw, nimp;
    } topk;
    DBuf<int> imp_len, imp_boff;       // import_csr scratch, kept across rebuilds
    DBuf<int64_t> imp_rb, imp_rn;
    DBuf<uint8_t> idx_spare, val_spare;  // the arrays the last rebuild replaced
    DBuf<int> csr_p, csr_i;               // staging of host CSR arguments
    DBuf<float> csr_v;
    // optional CUDA-event timing of the main forward / backward kernels
    bool timing = false;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    bool ev_fwd = false, ev_bwd = false;

    LayerView view() const {
        LayerView v;
        v.n_in = rows; v.n_out = cols; v.rank = rank;
        v.bs = bs.p; v.be = be.p; v.es = es.p; v.ee = ee.p;
        v.idx = idx.p; v.val = val.p;
        v.vs = vs.p; v.os = os.p; v.vsi = vsi.p; v.osi = osi.p; v.vsm = vsm.p;
        v.vstep = vstep.p; v.ostep = ostep.p; v.is = is.p; v.ois = ois.p;
        v.rowptr = rowptr.p; v.abs_cols = abs_cols.p; v.colptr = colptr.p; v.crow = crow.p; v.cvpos = cvpos.p;
        v.b4_nt = b4_ntiles > 0 ? b4_nt.p : nullptr;
        v.true_units = scale_policy == SILI_SCALE_POLICY_RESYNC;
        return v;
    }
    B4View b4view() const {
        B4View v;
        v.BR = b4_BR; v.BC = b4_BC;
        v.es = b4_es.p; v.nt = b4_nt.p; v.bc = b4_bc.p; v.tile = b4_tile.p; v.sparse = b4_sparse.p;
        v.alloc = b4_alloc.p; v.counters = b4_cnt.p; v.switch_point = b4_switch;
        v.cptr = b4_cptr.p; v.ctile = b4_ctile.p; v.cbr = b4_cbr.p;
        return v;
    }
};
using SynState = sili_layer::SynStateT;
using TopkState = sili_layer::TopkStateT;

namespace {

int use(sili_layer* h) {
    if (!h) return fail(SILI_EINVAL, "null layer handle");
    CK(cudaSetDevice(h->dev));
    return SILI_OK;
}

cudaStream_t pick(sili_layer* h, void* stream) { return stream ? (cudaStream_t)stream : h->stream; }

// ── cub helpers ─────────────────────────────────────────────────────────────
int scan_excl_int(sili_layer* h, const int* in, int* out, int64_t n, cudaStream_t s) {
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, in, out, (int)n, s);
    RC(h->cub_tmp.reserve((int64_t)bytes + 1));
    CK(cub::DeviceScan::ExclusiveSum(h->cub_tmp.p, bytes, in, out, (int)n, s));
    return SILI_OK;
}
int scan_incl_int(sili_layer* h, const int* in, int* out, int64_t n, cudaStream_t s) {
    size_t bytes = 0;
    cub::DeviceScan::InclusiveSum(nullptr, bytes, in, out, (int)n, s);
    RC(h->cub_tmp.reserve((int64_t)bytes + 1));
    CK(cub::DeviceScan::InclusiveSum(h->cub_tmp.p, bytes, in, out, (int)n, s));
    return SILI_OK;
}

// copy helpers: host or device source/destination
int to_dev(const void* src, void* dst, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return SILI_OK;
    CK(cudaMemcpyAsync(dst, src, bytes, is_device_ptr(src) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    return SILI_OK;
}
int from_dev(const void* src, void* dst, size_t bytes, cudaStream_t s) {
    if (bytes == 0 || !dst) return SILI_OK;
    CK(cudaMemcpyAsync(dst, src, bytes, is_device_ptr(dst) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s));
    return SILI_OK;
}

// Device view of an input array: the array itself when it is device memory,
// else a copy in the given staging buffer.
int stage_in(sili_layer* h, const float* src, size_t n, DBuf<float>& stage, const float** out, cudaStream_t s) {
    if (is_device_ptr(src)) { *out = src; return SILI_OK; }
    RC(stage.reserve((int64_t)n + 1));
    CK(cudaMemcpyAsync(stage.p, src, n * 4, cudaMemcpyHostToDevice, s));
    *out = stage.p;
    return SILI_OK;
}
// Device views of a CSR argument (row pointers, indices, values): the arrays
// themselves when they are device memory, else copies in the layer's staging
// buffers (kept across calls).
int stage_csr(sili_layer* h, const int* ptrs, const int* idx, const float* vals, int rows, int nnz, const int** dp,
              const int** di, const float** dv, cudaStream_t s) {
    if (is_device_ptr(ptrs)) { *dp = ptrs; }
    else { RC(h->csr_p.reserve(rows + 1)); RC(to_dev(ptrs, h->csr_p.p, (size_t)(rows + 1) * 4, s)); *dp = h->csr_p.p; }
    if (nnz == 0 || is_device_ptr(idx)) { *di = idx; }
    else { RC(h->csr_i.reserve(nnz + 1)); RC(to_dev(idx, h->csr_i.p, (size_t)nnz * 4, s)); *di = h->csr_i.p; }
    if (nnz == 0 || is_device_ptr(vals)) { *dv = vals; }
    else { RC(h->csr_v.reserve(nnz + 1)); RC(to_dev(vals, h->csr_v.p, (size_t)nnz * 4, s)); *dv = h->csr_v.p; }
    return SILI_OK;
}
// dst = transpose of the row-major [rows, cols] array src (host or device).
int stage_transposed(sili_layer* h, const float* src, int64_t rows, int64_t cols, DBuf<float>& dst, cudaStream_t s) {
    const float* d = nullptr;
    RC(stage_in(h, src, (size_t)(rows * cols), h->x_stage, &d, s));
    // [cols, rows] plus one zero row (row `cols`), which the forward kernels'
    // CSC padding entries point at
    RC(dst.reserve(rows * cols + rows + 1));
    if (rows == 1) {   // a single sample: one launch
        launch_copy_pad(d, dst.p, cols, s);
        return SILI_OK;
    }
    launch_transpose(d, dst.p, rows, cols, s);
    CK(cudaMemsetAsync(dst.p + rows * cols, 0, (size_t)rows * sizeof(float), s));
    return SILI_OK;
}
UpdateParams update_params(sili_layer* h, float lr, unsigned flags, float beta2, float eps) {
    UpdateParams P;
    P.lr = lr; P.beta2 = beta2; P.eps = eps;
    P.lr_per_row_nnz = (flags & SILI_LR_PER_ROW_NNZ) != 0;
    P.damp = (flags & SILI_DAMP_BY_IMPORTANCE) != 0;
    P.stochastic = false;
    P.os_trainable = false;
    P.call_key = host_mix64(h->seed ^ (h->call * 0x9E3779B97F4A7C15ULL));
    P.pow_tab = h->pow_tab.p; P.pow_n = h->pow_n;
    P.colg = h->colg.p; P.colc = h->colc.p;
    P.stats = h->d_st.p; P.stat_max = h->d_stmax.p;
    P.scale_noop = h->scale_policy == SILI_SCALE_POLICY_NONE;
    P.resync = h->scale_policy == SILI_SCALE_POLICY_RESYNC;
    return P;
}

// Validates a row-major CSR argument: ptrs[0] == 0, non-decreasing,
// ptrs[rows] == nnz and (for host arrays) every index in [0, cols).
int check_csr(const int* ptrs, const int* idx, int rows, int nnz, int64_t cols, const char* what) {
    std::vector<int> hp((size_t)rows + 1);
    if (is_device_ptr(ptrs)) CK(cudaMemcpy(hp.data(), ptrs, hp.size() * 4, cudaMemcpyDeviceToHost));
    else std::memcpy(hp.data(), ptrs, hp.size() * 4);
    if (hp[0] != 0 || hp[rows] != nnz) return fail(SILI_EINVAL, std::string(what) + ": ptrs[0] must be 0 and ptrs[batch] == nnz");
    for (int b = 0; b < rows; ++b)
        if (hp[b + 1] < hp[b]) return fail(SILI_EINVAL, std::string(what) + ": ptrs must be non-decreasing");
    if (idx && !is_device_ptr(idx))
        for (int j = 0; j < nnz; ++j)
            if (idx[j] < 0 || idx[j] >= cols) return fail(SILI_EINVAL, std::string(what) + ": index out of range");
    return SILI_OK;
}

// ── derived index: flat decode + CSC shadow ─────────────────────────────────
// Rebuild scratch kept between rebuilds up to this size (smaller layers
// rebuild often -- synaptogenesis steps -- and should not allocate each time).
constexpr int64_t kRebuildKeepBytes = (int64_t)256 << 20;

int ensure_aux(sili_layer* h, cudaStream_t s) {
    if (!h->aux_dirty) return SILI_OK;
    const int64_t R = h->rows, C = h->cols, nnz = h->total_nnz;
    RC(h->rowptr.reserve(R + 1));
    RC(h->colptr.reserve(C + 1));
    RC(h->colcount.reserve(C + 1));
    const int64_t nz = std::max<int64_t>(nnz, 1);
    const int64_t nzp = nz + 7 * C + 8;   // padded CSC bound
    RC(h->abs_cols.reserve(nz)); RC(h->frow.reserve(nz)); RC(h->fvpos.reserve(nz));
    RC(h->crow.reserve(nzp)); RC(h->cvpos.reserve(nzp)); RC(h->colptr_x.reserve(C + 1)); RC(h->padcnt.reserve(C + 1));
    RC(h->fcpos.reserve(nz));
    RC(h->sort_k.reserve(nz)); RC(h->sort_ko.reserve(nz)); RC(h->sort_v.reserve(nz)); RC(h->sort_vo.reserve(nz));
    CK(cudaMemsetAsync(h->rowptr.p, 0, sizeof(int), s));
    launch_row_nnz(h->es.p, h->ee.p, R, h->rowptr.p + 1, s);
    if (R > 0) RC(scan_incl_int(h, h->rowptr.p + 1, h->rowptr.p + 1, R, s));
    CK(cudaMemsetAsync(h->colcount.p, 0, (size_t)(C + 1) * sizeof(int), s));
    LayerView v = h->view();
    launch_decode_rows(v, h->abs_cols.p, h->frow.p, h->fvpos.p, h->colcount.p, s);
    if (nnz > 0) {
        CK(cudaMemcpyAsync(h->sort_k.p, h->abs_cols.p, (size_t)nnz * sizeof(int), cudaMemcpyDeviceToDevice, s));
        launch_iota(h->sort_v.p, nnz, s);
        int bits = 1;
        while ((int64_t(1) << bits) < C) ++bits;
        size_t bytes = 0;
        cub::DeviceRadixSort::SortPairs(nullptr, bytes, h->sort_k.p, h->sort_ko.p, h->sort_v.p, h->sort_vo.p,
                                        (int)nnz, 0, bits, s);
        RC(h->cub_tmp.reserve((int64_t)bytes + 1));
        CK(cub::DeviceRadixSort::SortPairs(h->cub_tmp.p, bytes, h->sort_k.p, h->sort_ko.p, h->sort_v.p,
                                           h->sort_vo.p, (int)nnz, 0, bits, s));
    }
    // exact column offsets, then the padded ones the forward kernels use
    RC(scan_excl_int(h, h->colcount.p, h->colptr_x.p, C + 1, s));
    launch_pad_counts(h->colcount.p, C + 1, h->padcnt.p, s);
    RC(scan_excl_int(h, h->padcnt.p, h->colptr.p, C + 1, s));
    if (nnz > 0)
        launch_gather_csc(h->sort_vo.p, h->sort_ko.p, h->frow.p, h->fvpos.p, h->colptr_x.p, h->colptr.p, nnz,
                          h->crow.p, h->cvpos.p, h->fcpos.p, s);
    launch_pad_csc(h->colcount.p, h->colptr.p, C, (int)R, h->crow.p, h->cvpos.p, s);
    CK(cudaGetLastError());
    // the rebuild's own arrays (24 bytes per synapse: the row and value
    // position of every synapse, the sort's keys and values, plus the sort's
    // temporary storage) are not read again until the next rebuild: a large
    // layer gives them back, keeping only abs_cols, crow, cvpos, fcpos and
    // cpack (20 bytes per synapse)
    if ((int64_t)nz * 24 > kRebuildKeepBytes) {
        h->frow.release(); h->fvpos.release();
        h->sort_k.release(); h->sort_ko.release(); h->sort_v.release(); h->sort_vo.release();
        h->cub_tmp.release();   // the sort's temporary storage (about 8 bytes per synapse)
    }
    {   // rows with no synapse take the dead-row bootstrap (linear_disldo.hpp:1985-2042)
        std::vector<int> rp((size_t)R + 1);
        CK(cudaMemcpyAsync(rp.data(), h->rowptr.p, (size_t)(R + 1) * 4, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        h->has_dead_rows = false;
        for (int64_t r = 0; r < R; ++r) if (rp[r + 1] == rp[r]) { h->has_dead_rows = true; break; }
    }
    h->aux_dirty = false;
    h->pack_valid = false;
    return SILI_OK;
}

// The dense / sparse-formula forward over xT: the row-tiled kernel (x staged
// in shared memory, packed column index rebuilt here when the weight codes
// changed) where its shape rules allow, else the per-synapse gather kernels.
int forward_columns(sili_layer* h, const float* xT, int batch, float* y, bool sparse, cudaStream_t s) {
    LayerView v = h->view();
    if (h->total_nnz > 0) {
        // the packed column index: rebuilt here after a change of the weight
        // codes that did not keep it current (the dense update keeps it)
        const int64_t bound = std::max<int64_t>(h->total_nnz, 1) + 7 * h->cols + 8;   // padded CSC bound
        if (!h->pack_valid) {
            RC(h->cpack.reserve(bound));
            launch_pack_csc(v, bound, h->cpack.p, s);
            h->pack_valid = true;
        }
        v.cpack = h->cpack.p;
        v.colptr_x = h->colptr_x.p;
        if (forward_rows_applies(v, batch) && launch_forward_rows(v, xT, batch, y, sparse, s)) return SILI_OK;
    }
    launch_forward(v, xT, batch, y, sparse, s);
    return SILI_OK;
}

// ── layout helpers on the host (O(rows) metadata) ───────────────────────────
struct HostLayout {
    std::vector<int64_t> bs, be, es, ee;
};
int get_layout(sili_layer* h, HostLayout& L) {
    const int64_t R = h->rows;
    L.bs.resize(R + 1); L.be.resize(R + 1); L.es.resize(R + 1); L.ee.resize(R + 1);
    CK(cudaMemcpyAsync(L.bs.data(), h->bs.p, (R + 1) * 8, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(L.es.data(), h->es.p, (R + 1) * 8, cudaMemcpyDeviceToHost, h->stream));
    if (R > 0) {
        CK(cudaMemcpyAsync(L.be.data(), h->be.p, R * 8, cudaMemcpyDeviceToHost, h->stream));
        CK(cudaMemcpyAsync(L.ee.data(), h->ee.p, R * 8, cudaMemcpyDeviceToHost, h->stream));
    }
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}
int put_layout(sili_layer* h, const HostLayout& L) {
    const int64_t R = h->rows;
    RC(h->bs.reserve(R + 1)); RC(h->be.reserve(R + 1)); RC(h->es.reserve(R + 1)); RC(h->ee.reserve(R + 1));
    CK(cudaMemcpyAsync(h->bs.p, L.bs.data(), (R + 1) * 8, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->es.p, L.es.data(), (R + 1) * 8, cudaMemcpyHostToDevice, h->stream));
    if (R > 0) {
        CK(cudaMemcpyAsync(h->be.p, L.be.data(), R * 8, cudaMemcpyHostToDevice, h->stream));
        CK(cudaMemcpyAsync(h->ee.p, L.ee.data(), R * 8, cudaMemcpyHostToDevice, h->stream));
    }
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

// Moves every row to the offsets in N (allocations may change), copying the
// live bytes/values; new buffers are zero-filled.
int relayout(sili_layer* h, const HostLayout& N, int64_t new_idx_n, int64_t new_val_n, bool recode) {
    cudaStream_t s = h->stream;
    DBuf<int64_t> nbs, nes;
    RC(nbs.reserve(h->rows + 1));
    RC(nes.reserve(h->rows + 1));
    CK(cudaMemcpyAsync(nbs.p, N.bs.data(), (h->rows + 1) * 8, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(nes.p, N.es.data(), (h->rows + 1) * 8, cudaMemcpyHostToDevice, s));
    DBuf<uint8_t> nidx, nval;
    RC(nidx.reserve(new_idx_n + 64));
    RC(nval.reserve(new_val_n + 64));
    CK(cudaMemsetAsync(nidx.p, 0, (size_t)nidx.cap, s));
    CK(cudaMemsetAsync(nval.p, 0, (size_t)nval.cap, s));
    launch_copy_rows(h->view(), nbs.p, nes.p, nidx.p, nval.p, recode, s);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    h->idx.swap(nidx);
    h->val.swap(nval);
    h->idx_n = new_idx_n;
    h->val_n = new_val_n;
    RC(put_layout(h, N));
    h->aux_dirty = true;
    return SILI_OK;
}

// ── scale bookkeeping ───────────────────────────────────────────────────────
int alloc_scales(sili_layer* h) {
    cudaStream_t s = h->stream;
    const int64_t R = h->rows, C = h->cols, k = h->rank;
    RC(h->vs.reserve(R * k + 1)); RC(h->vsi.reserve(R * k + 1)); RC(h->vsm.reserve(R * k + 1));
    RC(h->vstep.reserve(R * k + 1));
    RC(h->os.reserve(C * k + 1)); RC(h->osi.reserve(C * k + 1)); RC(h->ostep.reserve(C * k + 1));
    RC(h->colg.reserve(C * k + 1)); RC(h->colc.reserve(C * k + 1));
    return SILI_OK;
}

// Rebuild a rank-strided vector for a new rank from its logical prefix.
int relayout_scale(sili_layer* h, DBuf<float>& v, int64_t n_entities, int old_rank, int new_rank,
                   int64_t logical_n, bool scale_default) {
    std::vector<float> old((size_t)(n_entities * old_rank));
    if (!old.empty())
        CK(cudaMemcpy(old.data(), v.p, old.size() * sizeof(float), cudaMemcpyDeviceToHost));
    std::vector<float> nv((size_t)(n_entities * new_rank));
    for (size_t i = 0; i < nv.size(); ++i) {
        if ((int64_t)i < logical_n && i < old.size()) nv[i] = old[i];
        else nv[i] = scale_default ? ((i % new_rank) == 0 ? 1.0f : 0.0f) : 0.0f;
    }
    DBuf<float> q;
    RC(q.reserve((int64_t)nv.size() + 1));
    if (!nv.empty()) CK(cudaMemcpy(q.p, nv.data(), nv.size() * sizeof(float), cudaMemcpyHostToDevice));
    v.swap(q);
    return SILI_OK;
}
int relayout_steps(sili_layer* h, DBuf<uint32_t>& v, int64_t n_entities, int old_rank, int new_rank) {
    std::vector<uint32_t> old((size_t)(n_entities * old_rank));
    if (!old.empty()) CK(cudaMemcpy(old.data(), v.p, old.size() * 4, cudaMemcpyDeviceToHost));
    std::vector<uint32_t> nv((size_t)(n_entities * new_rank), 0u);
    for (size_t i = 0; i < nv.size() && i < old.size(); ++i) nv[i] = old[i];
    DBuf<uint32_t> q;
    RC(q.reserve((int64_t)nv.size() + 1));
    if (!nv.empty()) CK(cudaMemcpy(q.p, nv.data(), nv.size() * 4, cudaMemcpyHostToDevice));
    v.swap(q);
    return SILI_OK;
}

// Grows the logical size of value_scale / output_scale to n, filling new
// entries with `fill` (std::vector::resize semantics of the reference).
// fills on the stream of the call that grows the vector (its kernels read it next)
void grow_logical(sili_layer* h, DBuf<float>& v, int64_t& n_logical, int64_t n, float fill, cudaStream_t s = nullptr) {
    if (n <= n_logical) return;
    launch_fill_f32(v.p + n_logical, n - n_logical, fill, s ? s : h->stream);
    n_logical = n;
}

// Bias-correction table: pow_tab[s] = powf(beta2, s) evaluated by the host
// libm, exactly the reference's std::pow(beta2, (float)step)
// (delta_csr_types.hpp:457, linear_disldo.hpp:1941, sisldo_ops.hpp:793).
int ensure_pow_table(sili_layer* h, float beta2, uint32_t need) {
    const bool same = (beta2 == h->pow_beta2) || (std::isnan(beta2) && std::isnan(h->pow_beta2));
    if (same && (int64_t)need < h->pow_n) return SILI_OK;
    int n = 1;
    if (beta2 > 0.0f && beta2 < 1.0f) {
        // entries until powf(beta2, s) <= 2^-26, after which 1 - p == 1 in fp32
        while (n < (1 << 22) && std::pow(beta2, (float)n) > 1.4901161e-08f) ++n;
        n += 1;
    } else {
        n = 1 << 16;
    }
    n = std::max<int>(n, (int)need + 1);
    std::vector<float> t((size_t)n);
    for (int i = 0; i < n; ++i) t[i] = std::pow(beta2, (float)i);
    RC(h->pow_tab.reserve(n));
    CK(cudaMemcpy(h->pow_tab.p, t.data(), (size_t)n * sizeof(float), cudaMemcpyHostToDevice));
    h->pow_beta2 = beta2;
    h->pow_n = n;
    return SILI_OK;
}

int flush_stats(sili_layer* h) {
    if (!h->st_pending) return SILI_OK;
    double d[2];
    float m;
    CK(cudaMemcpy(d, h->d_st.p, 2 * sizeof(double), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(&m, h->d_stmax.p, sizeof(float), cudaMemcpyDeviceToHost));
    h->st[2] += d[0];
    h->st[3] += d[1];
    h->st_imax = std::max(h->st_imax * h->max_abs_decay, m);
    CK(cudaMemset(h->d_st.p, 0, 2 * sizeof(double)));
    CK(cudaMemset(h->d_stmax.p, 0, sizeof(float)));
    h->st_pending = false;
    return SILI_OK;
}

int recompute_stats(sili_layer* h) {
    RC(flush_stats(h));
    DBuf<double> sums;
    DBuf<float> mx;
    RC(sums.reserve(4));
    RC(mx.reserve(2));
    CK(cudaMemsetAsync(sums.p, 0, 4 * sizeof(double), h->stream));
    CK(cudaMemsetAsync(mx.p, 0, 2 * sizeof(float), h->stream));
    launch_stats(h->view(), sums.p, mx.p, h->stream);
    double d[4];
    float m[2];
    CK(cudaMemcpyAsync(d, sums.p, sizeof d, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(m, mx.p, sizeof m, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    h->st[0] = d[0]; h->st[1] = d[1]; h->st[2] = d[2]; h->st[3] = d[3];
    h->st_vmax = m[0]; h->st_imax = m[1];
    return SILI_OK;
}

// delta_csr_from_absolute on device (delta_csr_memory.hpp:16-93): per-synapse
// ULEB128 lengths and a scan give each row's byte count; the host lays out the
// per-row headroom (0.2 * bytes + 5 bytes, max(1, 0.2 * n + 1) elements) and a
// kernel writes every delta and FP4 byte in place.
int import_csr(sili_layer* h, const int* d_ptrs, const int* d_idx, const float* d_vals, int nnz,
               const float* d_imps = nullptr) {
    cudaStream_t s = h->stream;
    const int R = (int)h->rows;
    DBuf<int>& len = h->imp_len;
    DBuf<int>& boff = h->imp_boff;
    RC(len.reserve(nnz + 1));
    RC(boff.reserve(nnz + 1));
    CK(cudaMemsetAsync(len.p, 0, (size_t)(nnz + 1) * sizeof(int), s));
    launch_import_lengths(d_ptrs, d_idx, R, len.p, s);
    RC(scan_excl_int(h, len.p, boff.p, nnz + 1, s));
    DBuf<int64_t>& rb = h->imp_rb;
    DBuf<int64_t>& rn = h->imp_rn;
    RC(rb.reserve(R + 1));
    RC(rn.reserve(R + 1));
    launch_import_rows(d_ptrs, boff.p, R, rb.p, rn.p, s);
    std::vector<int64_t> hrb(R + 1), hrn(R + 1);
    if (R > 0) {
        CK(cudaMemcpyAsync(hrb.data(), rb.p, (size_t)R * 8, cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(hrn.data(), rn.p, (size_t)R * 8, cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    HostLayout N;
    N.bs.assign(R + 1, 0); N.be.assign(R + 1, 0); N.es.assign(R + 1, 0); N.ee.assign(R + 1, 0);
    for (int r = 0; r < R; ++r) {
        const int64_t nb = hrb[r], n = hrn[r];
        N.be[r] = N.bs[r] + nb;
        N.bs[r + 1] = N.be[r] + (int64_t)((float)nb * 0.2f) + 5;
        N.ee[r] = N.es[r] + n;
        N.es[r + 1] = N.ee[r] + std::max<int64_t>(1, (int64_t)((float)n * 0.2f) + 1);
    }
    RC(put_layout(h, N));
    const int64_t ib = N.bs[R], vb = N.es[R];
    // the previous rebuild's arrays are the spares: a rebuild of the same
    // size (a synaptogenesis step) allocates and frees nothing
    DBuf<uint8_t>& nidx = h->idx_spare;
    DBuf<uint8_t>& nval = h->val_spare;
    RC(nidx.reserve(ib + 64));
    RC(nval.reserve(vb + 64));
    CK(cudaMemsetAsync(nidx.p, 0, (size_t)(ib + 64), s));
    CK(cudaMemsetAsync(nval.p, 0, (size_t)(vb + 64), s));
    launch_import_write(d_ptrs, d_idx, d_vals, d_imps, boff.p, R, h->bs.p, h->es.p, nidx.p, nval.p, s);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    h->idx.swap(nidx);
    h->val.swap(nval);
    h->idx_n = ib;
    h->val_n = vb;
    h->total_nnz = nnz;
    h->aux_dirty = true;
    // a large layer gives back the import's scratch (8 bytes per synapse)
    // and the arrays it replaced (the constructor's budget, or the last
    // layout): the next rebuild allocates them again
    if ((int64_t)nnz * 8 > kRebuildKeepBytes) {
        h->imp_len.release(); h->imp_boff.release();
        h->idx_spare.release(); h->val_spare.release();
    }
    return SILI_OK;
}

// ── block4 store management ─────────────────────────────────────────────────
// Block4Store::init (block4.hpp:1103-1117): empty, every allocation zero.
// Each block-row gets `cap` tile slots of device capacity.
int b4_init(sili_layer* h, int64_t cap, cudaStream_t s) {
    h->b4_BR = (h->rows + 3) / 4;
    h->b4_BC = (h->cols + 3) / 4;
    const int64_t BR = h->b4_BR, total = std::max<int64_t>(BR * cap, 1);
    RC(h->b4_es.reserve(BR + 1)); RC(h->b4_nt.reserve(BR + 1)); RC(h->b4_alloc.reserve(3 * BR + 1));
    RC(h->b4_used.reserve(3 * BR + 1)); RC(h->b4_cnt.reserve(3));
    RC(h->b4_bc.reserve(total)); RC(h->b4_tile.reserve(total)); RC(h->b4_sparse.reserve(total));
    std::vector<int64_t> es((size_t)BR + 1);
    for (int64_t br = 0; br <= BR; ++br) es[(size_t)br] = br * cap;
    CK(cudaMemcpyAsync(h->b4_es.p, es.data(), es.size() * 8, cudaMemcpyHostToDevice, s));
    CK(cudaMemsetAsync(h->b4_nt.p, 0, (size_t)(BR + 1) * 4, s));
    CK(cudaMemsetAsync(h->b4_alloc.p, 0, (size_t)(3 * BR + 1) * 8, s));
    CK(cudaMemsetAsync(h->b4_cnt.p, 0, 3 * sizeof(unsigned long long), s));
    CK(cudaStreamSynchronize(s));
    h->b4_ntiles = 0;
    h->b4_dirty = true;
    h->b4_pmap_dirty = h->b4_pmapT_dirty = true;
    return SILI_OK;
}

// per block-row [3*BR]: tile bytes used, index bytes used, live slots
int b4_row_stats(sili_layer* h, std::vector<int64_t>& out, cudaStream_t s) {
    const int64_t BR = h->b4_BR;
    out.assign((size_t)(3 * BR), 0);
    if (BR == 0) return SILI_OK;
    launch_b4_row_used(h->b4view(), h->b4_used.p, s);
    CK(cudaMemcpyAsync(out.data(), h->b4_used.p, (size_t)(3 * BR) * 8, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}
int b4_get_allocs(sili_layer* h, std::vector<int64_t>& a, cudaStream_t s) {
    a.assign((size_t)(3 * h->b4_BR), 0);
    if (h->b4_BR == 0) return SILI_OK;
    CK(cudaMemcpyAsync(a.data(), h->b4_alloc.p, a.size() * 8, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}
int b4_put_allocs(sili_layer* h, const std::vector<int64_t>& a, cudaStream_t s) {
    if (h->b4_BR == 0) return SILI_OK;
    CK(cudaMemcpyAsync(h->b4_alloc.p, a.data(), a.size() * 8, cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// Tile column index for the forward: every live tile keyed by its
// block-column, stably sorted, so each block-column lists its tiles in
// ascending block-row.
int ensure_b4_index(sili_layer* h, cudaStream_t s) {
    if (!h->b4_dirty || h->b4_ntiles == 0) return SILI_OK;
    const int64_t BR = h->b4_BR, BC = h->b4_BC, n = h->b4_ntiles;
    RC(h->b4_off.reserve(BR + 1));
    RC(h->b4_keys.reserve(n)); RC(h->b4_keys_o.reserve(n)); RC(h->b4_perm.reserve(n)); RC(h->b4_perm_o.reserve(n));
    RC(h->b4_slots.reserve(n)); RC(h->b4_brs.reserve(n));
    RC(h->b4_cptr.reserve(BC + 1)); RC(h->b4_ctile.reserve(n)); RC(h->b4_cbr.reserve(n));
    RC(scan_excl_int(h, h->b4_nt.p, h->b4_off.p, BR, s));
    launch_b4_list(h->b4view(), h->b4_off.p, h->b4_keys.p, h->b4_slots.p, h->b4_brs.p, s);
    launch_iota(h->b4_perm.p, n, s);
    int bits = 1;
    while ((int64_t(1) << bits) < BC) ++bits;
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, h->b4_keys.p, h->b4_keys_o.p, h->b4_perm.p, h->b4_perm_o.p,
                                    (int)n, 0, bits, s);
    RC(h->cub_tmp.reserve((int64_t)bytes + 1));
    CK(cub::DeviceRadixSort::SortPairs(h->cub_tmp.p, bytes, h->b4_keys.p, h->b4_keys_o.p, h->b4_perm.p,
                                       h->b4_perm_o.p, (int)n, 0, bits, s));
    launch_b4_index(h->b4_keys_o.p, h->b4_perm_o.p, (int)n, BC, h->b4_slots.p, h->b4_brs.p, h->b4_cptr.p,
                    h->b4_ctile.p, h->b4_cbr.p, s);
    CK(cudaGetLastError());
    h->b4_dirty = false;
    return SILI_OK;
}

int make_layer(int n_in, int n_out, int max_weights, int device, int stochastic, sili_layer** out) {
    if (n_in < 0 || n_out < 0 || max_weights < 0) return fail(SILI_EINVAL, "negative layer size");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(SILI_ECUDA, "sili_b200: no CUDA device available (this library has no CPU path)");
    }
    if (device < 0 || device >= ndev) return fail(SILI_EINVAL, "device index out of range");
    CK(cudaSetDevice(device));
    sili_layer* h = new sili_layer();
    h->dev = device;
    h->rows = n_in;
    h->cols = n_out;
    h->stochastic = stochastic != 0;
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete h;
        return fail(SILI_ECUDA, "cudaStreamCreate failed");
    }
    int rc = SILI_OK;
    auto chk = [&](int r) { if (!rc) rc = r; };
    chk(alloc_scales(h));
    chk(h->is.reserve(n_in + 1)); chk(h->ois.reserve(n_out + 1));
    chk(h->in_acc.reserve(n_in + 1)); chk(h->grad_acc.reserve(n_out + 1)); chk(h->out_degree.reserve(n_out + 1));
    chk(h->d_st.reserve(2)); chk(h->d_stmax.reserve(1)); chk(h->d_dyflag.reserve(1)); chk(h->tc_err.reserve(1));
    if (rc) { delete h; return rc; }
    cudaStream_t s = h->stream;
    launch_fill_scale_default(h->vs.p, 0, (int64_t)n_in, 1, s);
    launch_fill_scale_default(h->os.p, 0, (int64_t)n_out, 1, s);
    cudaMemsetAsync(h->vsi.p, 0, (size_t)h->vsi.cap * 4, s);
    cudaMemsetAsync(h->vsm.p, 0, (size_t)h->vsm.cap * 4, s);
    cudaMemsetAsync(h->osi.p, 0, (size_t)h->osi.cap * 4, s);
    cudaMemsetAsync(h->vstep.p, 0, (size_t)h->vstep.cap * 4, s);
    cudaMemsetAsync(h->ostep.p, 0, (size_t)h->ostep.cap * 4, s);
    launch_fill_f32(h->is.p, n_in, 1.0f, s);
    launch_fill_f32(h->ois.p, n_out, 1.0f, s);
    cudaMemsetAsync(h->in_acc.p, 0, (size_t)(n_in + 1) * 4, s);
    cudaMemsetAsync(h->grad_acc.p, 0, (size_t)(n_out + 1) * 4, s);
    cudaMemsetAsync(h->out_degree.p, 0, (size_t)(n_out + 1) * 4, s);
    cudaMemsetAsync(h->d_st.p, 0, 2 * sizeof(double), s);
    cudaMemsetAsync(h->d_stmax.p, 0, sizeof(float), s);
    cudaMemsetAsync(h->d_dyflag.p, 0, sizeof(unsigned long long), s);
    cudaMemsetAsync(h->tc_err.p, 0, sizeof(unsigned int), s);
    // empty delta-CSR with per-row headroom (cpu_backend.cpp:380-389)
    h->idx_budget = (int64_t)max_weights * 8 + 4096;
    h->val_budget = (int64_t)max_weights + 64;
    std::vector<int> zp((size_t)n_in + 1, 0);
    DBuf<int> dp;
    rc = dp.reserve(n_in + 1);
    if (!rc && cudaMemcpy(dp.p, zp.data(), zp.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = SILI_ECUDA;
    if (!rc) rc = import_csr(h, dp.p, dp.p, nullptr, 0);
    if (rc) { cudaStreamDestroy(h->stream); delete h; return rc; }
    h->max_idx_bytes = h->idx_budget;
    h->max_val_bytes = h->val_budget;
    // block4 store with the constructor's limits (cpu_backend.cpp:390-393)
    rc = b4_init(h, 0, s);
    if (rc) { cudaStreamDestroy(h->stream); delete h; return rc; }
    h->b4_max_idx = (int64_t)max_weights * 8 + 4096;
    h->b4_max_tile = std::max<int64_t>(4, (int64_t)max_weights / 16) * 16;
    *out = h;
    return SILI_OK;
}

}  // namespace

// Host copy of the live block4 tiles, in block-row / stored order.
struct HostTiles {
    std::vector<int> br, bc;
    std::vector<uint8_t> slots, sparse;   // 16 per tile, 1 per tile
};
int b4_download(sili_layer* h, HostTiles& T, cudaStream_t s) {
    const int64_t BR = h->b4_BR;
    std::vector<int64_t> es((size_t)BR + 1);
    std::vector<int> nt((size_t)BR + 1);
    if (BR > 0) {
        CK(cudaMemcpyAsync(es.data(), h->b4_es.p, es.size() * 8, cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)BR * 4, cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    const int64_t cap = BR > 0 ? es[(size_t)BR] : 0;
    std::vector<int> bc((size_t)std::max<int64_t>(cap, 1));
    std::vector<uint4> tl((size_t)std::max<int64_t>(cap, 1));
    std::vector<uint8_t> sp((size_t)std::max<int64_t>(cap, 1));
    if (cap > 0) {
        CK(cudaMemcpyAsync(bc.data(), h->b4_bc.p, (size_t)cap * 4, cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(tl.data(), h->b4_tile.p, (size_t)cap * 16, cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(sp.data(), h->b4_sparse.p, (size_t)cap, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
    }
    T = HostTiles();
    for (int64_t br = 0; br < BR; ++br)
        for (int e = 0; e < nt[(size_t)br]; ++e) {
            const int64_t ti = es[(size_t)br] + e;
            T.br.push_back((int)br);
            T.bc.push_back(bc[(size_t)ti]);
            const uint8_t* b = reinterpret_cast<const uint8_t*>(&tl[(size_t)ti]);
            T.slots.insert(T.slots.end(), b, b + 16);
            T.sparse.push_back(sp[(size_t)ti]);
        }
    return SILI_OK;
}

int put_out(const void* host_src, void* dst, size_t bytes) {
    if (bytes == 0) return SILI_OK;
    if (is_device_ptr(dst)) CK(cudaMemcpy(dst, host_src, bytes, cudaMemcpyHostToDevice));
    else std::memcpy(dst, host_src, bytes);
    return SILI_OK;
}

// delta_csr_combined_to_absolute (delta_csr_memory.hpp:127-213): per row the
// scattered synapses then the row's live block4 slots, ordered by std::sort
// on the column with the reference's comparator (same algorithm here).
int export_combined(sili_layer* h, int* ptrs, int* idx, float* w, float* imp, cudaStream_t s) {
    const int64_t nnz = h->total_nnz, R = h->rows;
    DBuf<int> di;
    DBuf<float> dw, dm;
    RC(di.reserve(nnz + 1)); RC(dw.reserve(nnz + 1)); RC(dm.reserve(nnz + 1));
    launch_export(h->view(), di.p, dw.p, dm.p, s);
    CK(cudaGetLastError());
    std::vector<int> sp((size_t)R + 1), si((size_t)nnz + 1);
    std::vector<float> sw((size_t)nnz + 1), sm((size_t)nnz + 1);
    RC(from_dev(h->rowptr.p, sp.data(), (size_t)(R + 1) * 4, s));
    RC(from_dev(di.p, si.data(), (size_t)nnz * 4, s));
    RC(from_dev(dw.p, sw.data(), (size_t)nnz * 4, s));
    RC(from_dev(dm.p, sm.data(), (size_t)nnz * 4, s));
    CK(cudaStreamSynchronize(s));
    HostTiles T;
    RC(b4_download(h, T, s));
    std::vector<std::vector<size_t>> row_tiles((size_t)h->b4_BR);
    for (size_t t = 0; t < T.br.size(); ++t) row_tiles[(size_t)T.br[t]].push_back(t);
    struct Entry { int col; float w, imp; };
    std::vector<int> op((size_t)R + 1, 0), oi;
    std::vector<float> ow, om;
    std::vector<Entry> ent;
    for (int64_t r = 0; r < R; ++r) {
        ent.clear();
        for (int k = sp[(size_t)r]; k < sp[(size_t)r + 1]; ++k) ent.push_back({si[(size_t)k], sw[(size_t)k], sm[(size_t)k]});
        const int li = (int)(r % 4);
        for (size_t t : row_tiles[(size_t)(r / 4)])
            for (int lj = 0; lj < 4; ++lj) {
                const uint8_t byte = T.slots[t * 16 + (size_t)(lj * 4 + li)];
                const int64_t col = (int64_t)T.bc[t] * 4 + lj;
                if (byte == 0 || col >= h->cols) continue;
                ent.push_back({(int)col, fp4_decode_host(byte & 0xF), fp4_decode_host((uint8_t)(byte >> 4))});
            }
        std::sort(ent.begin(), ent.end(), [](const Entry& a, const Entry& b) { return a.col < b.col; });
        for (const Entry& e : ent) { oi.push_back(e.col); ow.push_back(e.w); om.push_back(e.imp); }
        op[(size_t)r + 1] = (int)oi.size();
    }
    RC(put_out(op.data(), ptrs, (size_t)(R + 1) * 4));
    RC(put_out(oi.data(), idx, oi.size() * 4));
    RC(put_out(ow.data(), w, ow.size() * 4));
    RC(put_out(om.data(), imp, om.size() * 4));
    return SILI_OK;
}

int64_t b4_live_total(sili_layer* h, cudaStream_t s) {
    std::vector<int64_t> st;
    if (b4_row_stats(h, st, s)) return -1;
    int64_t n = 0;
    for (int64_t br = 0; br < h->b4_BR; ++br) n += st[(size_t)(2 * h->b4_BR + br)];
    return n;
}

// ── synaptogenesis support ──────────────────────────────────────────────────
// Re-lay the block4 store out so block-row br has newcap[br] tile slots.
int b4_relayout(sili_layer* h, const std::vector<int64_t>& newcap, cudaStream_t s) {
    const int64_t BR = h->b4_BR;
    std::vector<int> nt((size_t)BR + 1);
    CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)BR * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    std::vector<int64_t> ne((size_t)BR + 1, 0);
    for (int64_t br = 0; br < BR; ++br) ne[(size_t)br + 1] = ne[(size_t)br] + std::max<int64_t>(newcap[(size_t)br], nt[(size_t)br]);
    const int64_t total = std::max<int64_t>(ne[(size_t)BR], 1);
    DBuf<int> nbc;
    DBuf<uint4> ntile;
    DBuf<uint8_t> nsp;
    DBuf<int64_t> nes;
    RC(nbc.reserve(total)); RC(ntile.reserve(total)); RC(nsp.reserve(total)); RC(nes.reserve(BR + 1));
    CK(cudaMemcpyAsync(nes.p, ne.data(), (size_t)(BR + 1) * 8, cudaMemcpyHostToDevice, s));
    launch_b4_move(BR, h->b4_es.p, nes.p, h->b4_nt.p, h->b4_bc.p, h->b4_tile.p, h->b4_sparse.p, nbc.p, ntile.p, nsp.p, s);
    CK(cudaMemcpyAsync(h->b4_es.p, nes.p, (size_t)(BR + 1) * 8, cudaMemcpyDeviceToDevice, s));
    CK(cudaStreamSynchronize(s));
    h->b4_bc.swap(nbc); h->b4_tile.swap(ntile); h->b4_sparse.swap(nsp);
    h->b4_dirty = true;
    h->b4_pmap_dirty = h->b4_pmapT_dirty = true;
    return SILI_OK;
}

// Probe-by-row index, scratch sizing and block4 capacity for a sweep of
// nrows rows.
int synap_prepare(sili_layer* h, int64_t nrows, cudaStream_t s) {
    SynState& Z = h->syn;
    const int64_t R = h->rows, C = h->cols, BR = h->b4_BR, np = h->n_probes;
    RC(Z.pr_ptr.reserve(R + 1));
    RC(Z.keys.reserve(np + 1)); RC(Z.keys_o.reserve(np + 1)); RC(Z.ids.reserve(np + 1)); RC(Z.ids_o.reserve(np + 1));
    if (np > 0) {
        CK(cudaMemcpyAsync(Z.keys.p, h->prow.p, (size_t)np * 4, cudaMemcpyDeviceToDevice, s));
        launch_iota(Z.ids.p, np, s);
        int bits = 1;
        while ((int64_t(1) << bits) <= R) ++bits;
        size_t bytes = 0;
        cub::DeviceRadixSort::SortPairs(nullptr, bytes, Z.keys.p, Z.keys_o.p, Z.ids.p, Z.ids_o.p, (int)np, 0, bits, s);
        RC(h->cub_tmp.reserve((int64_t)bytes + 1));
        CK(cub::DeviceRadixSort::SortPairs(h->cub_tmp.p, bytes, Z.keys.p, Z.keys_o.p, Z.ids.p, Z.ids_o.p, (int)np, 0,
                                           bits, s));
    }
    launch_lower_bound(Z.keys_o.p, (int)np, R, Z.pr_ptr.p, s);
    std::vector<int> pp((size_t)R + 1);
    CK(cudaMemcpyAsync(pp.data(), Z.pr_ptr.p, (size_t)(R + 1) * 4, cudaMemcpyDeviceToHost, s));
    HostLayout L;
    RC(get_layout(h, L));
    std::vector<int> nt((size_t)BR + 1, 0);
    std::vector<int64_t> es4((size_t)BR + 1, 0);
    if (BR > 0) {
        CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)BR * 4, cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(es4.data(), h->b4_es.p, (size_t)(BR + 1) * 8, cudaMemcpyDeviceToHost, s));
    }
    CK(cudaStreamSynchronize(s));
    // tile capacity: every add of a row may create one tile in its block-row
    const int64_t passes = (nrows + R - 1) / R;
    std::vector<int64_t> need((size_t)BR, 0);
    bool grow = false;
    int64_t maxp = 0, maxcap_tiles = 0, maxrow = 0;
    for (int64_t r = 0; r < R; ++r) {
        const int64_t pr = pp[(size_t)r + 1] - pp[(size_t)r];
        maxp = std::max(maxp, pr);
        need[(size_t)(r / 4)] += pr * passes;
        maxrow = std::max(maxrow, L.es[(size_t)r + 1] - L.es[(size_t)r]);
    }
    for (int64_t br = 0; br < BR; ++br) {
        need[(size_t)br] += nt[(size_t)br];
        if (need[(size_t)br] > es4[(size_t)br + 1] - es4[(size_t)br]) grow = true;
    }
    if (grow) {
        // a quarter more than this sweep can need, so that the tiles created
        // by the next sweeps' promotions rarely force another relayout
        for (int64_t br = 0; br < BR; ++br)
            need[(size_t)br] = std::max(need[(size_t)br] + std::max<int64_t>(8, need[(size_t)br] / 4),
                                        es4[(size_t)br + 1] - es4[(size_t)br]);
        RC(b4_relayout(h, need, s));
    }
    for (int64_t br = 0; br < BR; ++br)
        maxcap_tiles = std::max(maxcap_tiles, grow ? need[(size_t)br] : es4[(size_t)br + 1] - es4[(size_t)br]);
    Z.m = maxrow + 4 * maxcap_tiles + 16;
    Z.p = maxp + 1;
    Z.stride = synap_scratch_stride(Z.m, Z.p);
    const int64_t threads = std::max<int64_t>(BR, 1);
    RC(Z.scratch.reserve(Z.stride * threads + 16));
    RC(Z.od0.reserve(C + 1)); RC(Z.od_decs.reserve(C + 1)); RC(Z.did.reserve(nrows + 1)); RC(Z.res.reserve(8));
    return SILI_OK;
}

// Save (save=true) or restore the state a sweep changes.
int snapshot_state(sili_layer* h, bool save, cudaStream_t s) {
    SynState& Z = h->syn;
    const int64_t R = h->rows, C = h->cols, BR = h->b4_BR;
    int64_t cap4 = 0;
    if (BR > 0) {
        CK(cudaMemcpyAsync(&cap4, h->b4_es.p + BR, 8, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
    }
    struct Item { void* live; DBuf<uint8_t>* snap; size_t bytes; };
    Item items[] = {
        {h->idx.p, &Z.s_idx, (size_t)h->idx_n}, {h->val.p, &Z.s_val, (size_t)h->val_n},
        {h->be.p, &Z.s_be, (size_t)R * 8}, {h->ee.p, &Z.s_ee, (size_t)R * 8},
        {h->out_degree.p, &Z.s_od, (size_t)C * 4}, {h->b4_nt.p, &Z.s_nt, (size_t)BR * 4},
        {h->b4_bc.p, &Z.s_bc, (size_t)cap4 * 4}, {h->b4_tile.p, &Z.s_tile, (size_t)cap4 * 16},
        {h->b4_sparse.p, &Z.s_sp, (size_t)cap4}, {h->b4_alloc.p, &Z.s_alloc, (size_t)(3 * BR) * 8},
        {h->b4_cnt.p, &Z.s_cnt, 3 * sizeof(unsigned long long)},
    };
    for (Item& it : items) {
        if (it.bytes == 0) continue;
        if (save) {
            RC(it.snap->reserve((int64_t)it.bytes));
            CK(cudaMemcpyAsync(it.snap->p, it.live, it.bytes, cudaMemcpyDeviceToDevice, s));
        } else {
            CK(cudaMemcpyAsync(it.live, it.snap->p, it.bytes, cudaMemcpyDeviceToDevice, s));
        }
    }
    if (save && C > 0) CK(cudaMemcpyAsync(Z.od0.p, h->out_degree.p, (size_t)C * 4, cudaMemcpyDeviceToDevice, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int synap_reset_results(sili_layer* h, int64_t nrows, cudaStream_t s) {
    SynState& Z = h->syn;
    long long init[8] = {0, 0, 0, LLONG_MAX, 0, 0, 0, 0};
    CK(cudaMemcpyAsync(Z.res.p, init, sizeof(init), cudaMemcpyHostToDevice, s));
    CK(cudaMemsetAsync(Z.od_decs.p, 0, (size_t)(h->cols + 1) * 4, s));
    CK(cudaMemsetAsync(Z.did.p, 0, (size_t)nrows + 1, s));
    return SILI_OK;
}

SynView synap_view(sili_layer* h) {
    SynState& Z = h->syn;
    SynView V;
    V.n_in = h->rows; V.n_out = h->cols;
    V.bs = h->bs.p; V.be = h->be.p; V.es = h->es.p; V.ee = h->ee.p;
    V.idx = h->idx.p; V.val = h->val.p;
    V.out_degree = h->out_degree.p; V.od_decs = Z.od_decs.p;
    V.b4_es = h->b4_es.p; V.nt = h->b4_nt.p; V.b4_bc = h->b4_bc.p; V.b4_tile = h->b4_tile.p;
    V.b4_sparse = h->b4_sparse.p; V.alloc = h->b4_alloc.p; V.counters = h->b4_cnt.p; V.switch_point = h->b4_switch;
    V.max_idx = h->b4_max_idx; V.max_tile = h->b4_max_tile;
    std::vector<int64_t> a((size_t)(3 * h->b4_BR), 0);
    if (h->b4_BR > 0) {
        cudaMemcpy(a.data(), h->b4_alloc.p, a.size() * 8, cudaMemcpyDeviceToHost);
        for (int64_t br = 0; br < h->b4_BR; ++br) { V.tot_idx0 += a[(size_t)br]; V.tot_tile0 += a[(size_t)(h->b4_BR + br)]; }
    }
    long long* r = reinterpret_cast<long long*>(Z.res.p);
    V.grow = reinterpret_cast<unsigned long long*>(r);         // res[0..1]
    V.nnz_delta = reinterpret_cast<unsigned long long*>(r + 2);
    V.err_i = r + 3;
    V.err_code = reinterpret_cast<int*>(r + 4);
    V.flags = reinterpret_cast<int*>(r + 6);
    V.n_probes = h->n_probes; V.pcol = h->pcol.p; V.pval = h->pval.p;
    V.pr_ptr = Z.pr_ptr.p; V.pr_idx = Z.ids_o.p;
    V.did = Z.did.p;
    V.scratch = Z.scratch.p; V.scratch_stride = Z.stride; V.scratch_m = Z.m; V.scratch_p = Z.p;
    return V;
}

// ═══════════════════════════════════════════════════════════════════════════
// the error slot sili_last_error reads, for the library's other files
namespace sili {
int set_error(int code, const std::string& msg) { return fail(code, msg); }
}

extern "C" {

const char* sili_last_error(void) { return g_err.c_str(); }

int sili_kernel_launches(int64_t* count) {
    if (count) *count = (int64_t)launch_count();
    return SILI_OK;
}

int sili_layer_set_kernel_timing(sili_layer* h, int enable) {
    RC(use(h));
    if (enable && !h->ev[0])
        for (auto& e : h->ev) CK(cudaEventCreate(&e));
    h->timing = enable != 0;
    h->ev_fwd = h->ev_bwd = false;
    return SILI_OK;
}

int sili_layer_kernel_ms(sili_layer* h, float* fwd, float* bwd) {
    RC(use(h));
    if (fwd) *fwd = 0.f;
    if (bwd) *bwd = 0.f;
    if (h->ev_fwd && fwd) { CK(cudaEventSynchronize(h->ev[1])); CK(cudaEventElapsedTime(fwd, h->ev[0], h->ev[1])); }
    if (h->ev_bwd && bwd) { CK(cudaEventSynchronize(h->ev[3])); CK(cudaEventElapsedTime(bwd, h->ev[2], h->ev[3])); }
    return SILI_OK;
}

// Bytes of device memory a layer holds, by role (capacities, headroom and
// kept scratch included).
extern "C++" {
template <typename... Bufs>
static int64_t dbytes(const Bufs&... b) {
    return (int64_t(0) + ... + (b.cap * (int64_t)sizeof(*b.p)));
}
}
int sili_layer_device_bytes(sili_layer* h, int64_t* format, int64_t* index, int64_t* total) {
    RC(use(h));
    const int64_t fmt = dbytes(h->idx, h->val, h->bs, h->be, h->es, h->ee);
    const int64_t ix = dbytes(h->rowptr, h->abs_cols, h->frow, h->fvpos, h->colcount, h->colptr, h->crow, h->cvpos,
                              h->sort_k, h->sort_ko, h->sort_v, h->sort_vo, h->colptr_x, h->padcnt, h->fcpos,
                              h->cpack, h->cub_tmp);
    int64_t rest = dbytes(h->vs, h->os, h->vsi, h->osi, h->vsm, h->is, h->ois, h->vstep, h->ostep, h->def_cw,
                          h->def_ci, h->in_acc, h->grad_acc, h->out_degree, h->prow, h->pcol, h->pval, h->pb_keys,
                          h->pb_iota, h->pb_in, h->pb_out, h->pb_flags, h->pb_pos, h->pb_tr, h->pb_tc, h->pb_counts,
                          h->pb_tv, h->d_st, h->d_stmax, h->d_dyflag, h->xT, h->dyT, h->dxT, h->colg, h->colc,
                          h->ytmp, h->x_stage, h->dy_stage, h->dx_stage, h->xsT, h->fold_raw, h->shard_nnz, h->rpart,
                          h->presT, h->presX, h->dS, h->sgs, h->sgc, h->i_tmp0, h->i_tmp1, h->i_tmp2, h->f_tmp0,
                          h->pow_tab);
    rest += dbytes(h->b4_es, h->b4_alloc, h->b4_used, h->b4_nt, h->b4_bc, h->b4_tile, h->b4_sparse, h->b4_cnt,
                   h->b4_hs, h->b4_mr, h->b4_mc, h->b4_cptr, h->b4_ctile, h->b4_cbr, h->b4_keys, h->b4_keys_o,
                   h->b4_perm, h->b4_perm_o, h->b4_slots, h->b4_brs, h->b4_off, h->b4_xs, h->b4_part, h->tc_err,
                   h->b4_pmap, h->b4_pmapT);
    const auto& y = h->syn;
    rest += dbytes(y.pr_ptr, y.keys, y.keys_o, y.ids, y.ids_o, y.od0, y.od_decs, y.scratch, y.did, y.res, y.s_idx,
                   y.s_val, y.s_be, y.s_ee, y.s_od, y.s_nt, y.s_bc, y.s_tile, y.s_sp, y.s_alloc, y.s_cnt);
    const auto& t = h->topk;
    rest += dbytes(t.bits, t.keys, t.pk, t.pk_o, t.hist, t.cand, t.cand_o, t.eq, t.nsel, t.pid, t.pid_o, t.cptr,
                   t.cnt, t.nptr, t.drop, t.sel, t.nge, t.di, t.nidx, t.dw, t.dm, t.nw, t.nimp);
    rest += dbytes(h->imp_len, h->imp_boff, h->imp_rb, h->imp_rn, h->idx_spare, h->val_spare, h->csr_p, h->csr_i,
                   h->csr_v);
    if (format) *format = fmt;
    if (index) *index = ix;
    if (total) *total = fmt + ix + rest;
    return SILI_OK;
}

int sili_device_count(int* count) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); n = 0; }
    if (count) *count = n;
    return SILI_OK;
}

int sili_layer_create(int n_in, int n_out, int max_weights, int device, int stochastic, sili_layer** out) {
    if (!out) return fail(SILI_EINVAL, "null out pointer");
    return make_layer(n_in, n_out, max_weights, device, stochastic, out);
}

int sili_layer_destroy(sili_layer* h) {
    if (!h) return SILI_OK;
    cudaSetDevice(h->dev);
    cudaStreamSynchronize(h->stream);
    cudaStream_t s = h->stream;
    for (auto& e : h->ev) if (e) cudaEventDestroy(e);
    delete h;
    cudaStreamDestroy(s);
    return SILI_OK;
}

static int check_tc_err(sili_layer* h);

int sili_layer_sync(sili_layer* h) {
    RC(use(h));
    CK(cudaStreamSynchronize(h->stream));
    return check_tc_err(h);
}

int sili_layer_seed_rng(sili_layer* h, uint64_t seed) {
    RC(use(h));
    h->seed = seed;
    h->call = 0;
    return SILI_OK;
}

int sili_layer_load_weights(sili_layer* h, const int* ptrs, const int* idx, const float* vals, int nnz) {
    RC(use(h));
    if (nnz < 0 || !ptrs) return fail(SILI_EINVAL, "load_weights: bad arguments");
    const int R = (int)h->rows;
    cudaStream_t s = h->stream;
    std::vector<int> hp(R + 1);
    if (is_device_ptr(ptrs)) CK(cudaMemcpy(hp.data(), ptrs, (R + 1) * 4, cudaMemcpyDeviceToHost));
    else std::memcpy(hp.data(), ptrs, (R + 1) * 4);
    if (hp[0] != 0 || hp[R] != nnz) return fail(SILI_EINVAL, "load_weights: ptrs[0] must be 0 and ptrs[n_in] == nnz");
    for (int r = 0; r < R; ++r)
        if (hp[r + 1] < hp[r]) return fail(SILI_EINVAL, "load_weights: ptrs must be non-decreasing");
    DBuf<int> dp, di;
    DBuf<float> dv;
    RC(dp.reserve(R + 1)); RC(di.reserve(nnz + 1)); RC(dv.reserve(nnz + 1));
    CK(cudaMemcpyAsync(dp.p, hp.data(), (R + 1) * 4, cudaMemcpyHostToDevice, s));
    RC(to_dev(idx, di.p, (size_t)nnz * 4, s));
    RC(to_dev(vals, dv.p, (size_t)nnz * 4, s));
    // column range check on the host copy.  Columns need not ascend within a
    // row: like delta_csr_from_absolute (delta_csr_memory.hpp:16-93) a
    // descending step is stored as the wrapped 32-bit delta (a 5-byte
    // ULEB128) and decodes back to the same column, so such rows load,
    // forward and train in their given order as in the reference.
    std::vector<int> hi(nnz);
    if (nnz) CK(cudaMemcpyAsync(hi.data(), di.p, (size_t)nnz * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    for (int f = 0; f < nnz; ++f)
        if (hi[f] < 0 || hi[f] >= h->cols) return fail(SILI_EINVAL, "load_weights: column index out of range");
    RC(import_csr(h, dp.p, di.p, dv.p, nnz));
    h->idx_budget = std::max<int64_t>(h->idx_budget, (int64_t)nnz * 8 + 4096);
    h->val_budget = std::max<int64_t>(h->val_budget, (int64_t)nnz + 64);
    h->max_idx_bytes = h->idx_budget;
    h->max_val_bytes = h->val_budget;
    // out_degree rebuilt from the loaded indices (cpu_backend.cpp:899-900)
    std::vector<int> deg((size_t)h->cols, 0);
    for (int f = 0; f < nnz; ++f) deg[hi[f]]++;
    if (h->cols) CK(cudaMemcpy(h->out_degree.p, deg.data(), (size_t)h->cols * 4, cudaMemcpyHostToDevice));
    h->st_pending = false;
    CK(cudaMemset(h->d_st.p, 0, 2 * sizeof(double)));
    CK(cudaMemset(h->d_stmax.p, 0, sizeof(float)));
    return recompute_stats(h);
}

int sili_layer_set_value_bytes(sili_layer* h, const uint8_t* values, int64_t n) {
    RC(use(h));
    n = std::min<int64_t>(n, h->val_n);
    RC(to_dev(values, h->val.p, (size_t)n, h->stream));
    h->pack_valid = false;
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

// ── scales ──────────────────────────────────────────────────────────────────
int sili_layer_set_scale_rank(sili_layer* h, int rank) {
    RC(use(h));
    if (rank < 1) return fail(SILI_EINVAL, "scale_rank must be >= 1");
    if (rank > 4) return fail(SILI_EINVAL, "scale_rank exceeds SCALE_RANK_MAX (4)");
    if (rank == h->rank) return SILI_OK;
    if (h->scale_policy == SILI_SCALE_POLICY_RESYNC && rank != 1)
        return fail(SILI_EINVAL, "set_scale_rank: a Resync layer keeps scale rank 1 on this library");
    const int old = h->rank;
    CK(cudaStreamSynchronize(h->stream));
    RC(relayout_scale(h, h->vs, h->rows, old, rank, h->n_vs, true));
    RC(relayout_scale(h, h->os, h->cols, old, rank, h->n_os, true));
    RC(relayout_scale(h, h->vsi, h->rows, old, rank, h->rows * old, false));
    RC(relayout_scale(h, h->osi, h->cols, old, rank, h->cols * old, false));
    RC(relayout_scale(h, h->vsm, h->rows, old, rank, h->rows * old, false));
    RC(relayout_steps(h, h->vstep, h->rows, old, rank));
    RC(relayout_steps(h, h->ostep, h->cols, old, rank));
    h->rank = rank;
    RC(h->colg.reserve(h->cols * rank + 1));
    RC(h->colc.reserve(h->cols * rank + 1));
    return SILI_OK;
}

int sili_layer_get_scale_rank(sili_layer* h, int* rank) {
    RC(use(h));
    *rank = h->rank;
    return SILI_OK;
}

int sili_layer_set_scale(sili_layer* h, int kind, int index, int k, float v) {
    RC(use(h));
    CK(cudaStreamSynchronize(h->stream));
    switch (kind) {
    case SILI_SCALE_VALUE: {
        if (index < 0 || index >= h->rows || k < 0 || k >= h->rank) return fail(SILI_EINVAL, "value_scale index out of range");
        const int64_t i = (int64_t)index * h->rank + k;
        grow_logical(h, h->vs, h->n_vs, i + 1, 1.0f);
        CK(cudaMemcpyAsync(h->vs.p + i, &v, 4, cudaMemcpyHostToDevice, h->stream));
        break;
    }
    case SILI_SCALE_OUTPUT: {
        if (index < 0 || index >= h->cols || k < 0 || k >= h->rank) return fail(SILI_EINVAL, "output_scale index out of range");
        const int64_t i = (int64_t)index * h->rank + k;
        grow_logical(h, h->os, h->n_os, i + 1, 1.0f);
        CK(cudaMemcpyAsync(h->os.p + i, &v, 4, cudaMemcpyHostToDevice, h->stream));
        h->os_trainable = true;
        break;
    }
    case SILI_SCALE_IMPORTANCE:
        if (index < 0 || index >= h->rows) return fail(SILI_EINVAL, "importance_scale index out of range");
        CK(cudaMemcpyAsync(h->is.p + index, &v, 4, cudaMemcpyHostToDevice, h->stream));
        break;
    case SILI_SCALE_OUTPUT_IMPORTANCE:
        if (index < 0 || index >= h->cols) return fail(SILI_EINVAL, "output_importance_scale index out of range");
        CK(cudaMemcpyAsync(h->ois.p + index, &v, 4, cudaMemcpyHostToDevice, h->stream));
        break;
    default:
        return fail(SILI_EINVAL, "set_scale: unknown kind");
    }
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

static float* scale_ptr(sili_layer* h, int kind, int64_t* n_entities, int* stride);

int sili_layer_set_scales(sili_layer* h, int kind, const float* v, int n) {
    RC(use(h));
    if (n < 0 || (n > 0 && !v)) return fail(SILI_EINVAL, "set_scales: bad arguments");
    if (kind != SILI_SCALE_VALUE && kind != SILI_SCALE_OUTPUT && kind != SILI_SCALE_IMPORTANCE &&
        kind != SILI_SCALE_OUTPUT_IMPORTANCE)
        return fail(SILI_EINVAL, "set_scales: kind must be value, output, importance or output importance");
    int64_t ents;
    int stride;
    float* p = scale_ptr(h, kind, &ents, &stride);
    if (n > ents * stride) return fail(SILI_EINVAL, "set_scales: more entries than the vector holds");
    CK(cudaStreamSynchronize(h->stream));
    if (kind == SILI_SCALE_VALUE) grow_logical(h, h->vs, h->n_vs, n, 1.0f);
    if (kind == SILI_SCALE_OUTPUT) {
        grow_logical(h, h->os, h->n_os, n, 1.0f);
        if (n > 0) h->os_trainable = true;
    }
    if (n > 0) RC(to_dev(v, p, (size_t)n * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

static float* scale_ptr(sili_layer* h, int kind, int64_t* n_entities, int* stride) {
    *stride = h->rank;
    switch (kind) {
    case SILI_SCALE_VALUE: *n_entities = h->rows; return h->vs.p;
    case SILI_SCALE_OUTPUT: *n_entities = h->cols; return h->os.p;
    case SILI_SCALE_IMPORTANCE: *n_entities = h->rows; *stride = 1; return h->is.p;
    case SILI_SCALE_OUTPUT_IMPORTANCE: *n_entities = h->cols; *stride = 1; return h->ois.p;
    case SILI_SCALE_VALUE_IMPORTANCE: *n_entities = h->rows; return h->vsi.p;
    case SILI_SCALE_OUTPUT_SCALE_IMPORTANCE: *n_entities = h->cols; return h->osi.p;
    case SILI_SCALE_VALUE_MOMENTUM: *n_entities = h->rows; return h->vsm.p;
    default: return nullptr;
    }
}

int sili_layer_get_scale(sili_layer* h, int kind, int index, int k, float* v) {
    RC(use(h));
    int64_t n;
    int stride;
    float* p = scale_ptr(h, kind, &n, &stride);
    if (!p) return fail(SILI_EINVAL, "get_scale: unknown kind");
    if (index < 0 || index >= n || k < 0 || k >= stride) return fail(SILI_EINVAL, "get_scale: index out of range");
    CK(cudaStreamSynchronize(h->stream));
    CK(cudaMemcpy(v, p + (int64_t)index * stride + k, 4, cudaMemcpyDeviceToHost));
    return SILI_OK;
}

int sili_layer_get_scales(sili_layer* h, int kind, float* out, int n_req) {
    RC(use(h));
    int64_t n;
    int stride;
    float* p = scale_ptr(h, kind, &n, &stride);
    if (!p) return fail(SILI_EINVAL, "get_scales: unknown kind");
    const int64_t m = std::min<int64_t>(n_req, n * stride);
    CK(cudaStreamSynchronize(h->stream));
    RC(from_dev(p, out, (size_t)m * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

int sili_layer_get_steps(sili_layer* h, int which, uint32_t* out, int n_req) {
    RC(use(h));
    const int64_t n = (which == 0 ? h->rows : h->cols) * h->rank;
    const int64_t m = std::min<int64_t>(n_req, n);
    CK(cudaStreamSynchronize(h->stream));
    RC(from_dev(which == 0 ? h->vstep.p : h->ostep.p, out, (size_t)m * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

// rescale_value_row / rescale_importance_row (delta_csr_types.hpp:1389-1431)
int sili_layer_rescale_row(sili_layer* h, int kind, int row, float new_scale) {
    RC(use(h));
    if (kind != SILI_SCALE_VALUE && kind != SILI_SCALE_IMPORTANCE) return fail(SILI_EINVAL, "rescale_row: kind");
    float old;
    if (row < 0 || row >= h->rows) return SILI_OK;   // reference: `if (row >= L.rows) return;`
    RC(sili_layer_get_scale(h, kind, row, 0, &old));
    if (new_scale == old) return SILI_OK;
    launch_rescale_row(h->view(), row, old, new_scale, kind == SILI_SCALE_VALUE, h->stream);
    h->pack_valid = false;
    CK(cudaGetLastError());
    return sili_layer_set_scale(h, kind, row, 0, new_scale);
}

// ── compute ─────────────────────────────────────────────────────────────────
// A kernel's bounded device-side wait that gave up (the word the block4
// tensor-core forward / dx set), reported once as SILI_ETIMEOUT at the next
// synchronising call.
static int check_tc_err(sili_layer* h) {
    unsigned int e = 0;
    CK(cudaMemcpy(&e, h->tc_err.p, sizeof(e), cudaMemcpyDeviceToHost));
    if (e) {
        CK(cudaMemset(h->tc_err.p, 0, sizeof(e)));
        return fail(SILI_ETIMEOUT, "block4 tensor cores: a bounded device-side wait gave up");
    }
    return SILI_OK;
}

// The panel map costs n_in * n_out / 4 bytes; past this many entries (1 GiB)
// the tensor-core forward is not taken.
constexpr int64_t kB4PanelMapMax = (int64_t)1 << 28;

// The block4 part of forward_dense (dx = false) and of the lr = 0 backward's
// dx (dx = true): on the tensor cores when the layer asks for it and the
// shape allows (rank 1, batch >= 16), else the exact CUDA-core kernels.
static int b4_tc_or_exact(sili_layer* h, bool dx, const float* actT, int batch, float* out, cudaStream_t s) {
    const LayerView v = h->view();
    const B4View V = h->b4view();
    if (h->b4_tc && b4_tc_applies(v, V, batch) && b4_tc_pmap_elems(v, dx) <= kB4PanelMapMax) {
        DBuf<int>& map = dx ? h->b4_pmapT : h->b4_pmap;
        bool& dirty = dx ? h->b4_pmapT_dirty : h->b4_pmap_dirty;
        if (dirty) {
            RC(map.reserve(b4_tc_pmap_elems(v, dx) + 1));
            launch_b4_panel_map(v, V, dx, map.p, s);
            dirty = false;
        }
        int ks = 1;
        const int64_t nf = b4_tc_scratch_floats(v, batch, dx, &ks);
        RC(h->b4_part.reserve(nf + 1));
        RC(h->b4_xs.reserve(b4_tc_xsplit_elems(v, batch, dx) + 8));
        return dx ? launch_b4_dx_tc(v, V, actT, batch, out, h->b4_xs.p, h->b4_part.p, ks, map.p, h->tc_err.p, s)
                  : launch_b4_forward_tc(v, V, actT, batch, out, h->b4_xs.p, h->b4_part.p, ks, map.p, h->tc_err.p, s);
    }
    if (dx) launch_b4_dx(v, V, actT, batch, out, s);
    else launch_b4_forward(v, V, actT, batch, out, s);
    return SILI_OK;
}

static int b4_forward(sili_layer* h, const float* xT, int batch, float* y, cudaStream_t s) {
    return b4_tc_or_exact(h, false, xT, batch, y, s);
}

int sili_layer_set_scale_policy(sili_layer* h, int policy) {
    RC(use(h));
    if (policy != SILI_SCALE_POLICY_RMSPROP && policy != SILI_SCALE_POLICY_NONE && policy != SILI_SCALE_POLICY_RESYNC)
        return fail(SILI_EINVAL, "set_scale_policy: unknown policy");
    if (policy == SILI_SCALE_POLICY_RESYNC && h->rank != 1)
        return fail(SILI_EINVAL, "set_scale_policy: the Resync policy needs scale rank 1 on this library");
    h->scale_policy = policy;
    return SILI_OK;
}

int sili_layer_set_b4_tensor_cores(sili_layer* h, int enable) {
    RC(use(h));
    h->b4_tc = enable != 0;
    return SILI_OK;
}

int sili_layer_forward_dense(sili_layer* h, const float* x, int batch, float* y, void* stream) {
    RC(use(h));
    if (batch < 0 || !x || !y) return fail(SILI_EINVAL, "forward_dense: bad arguments");
    cudaStream_t s = pick(h, stream);
    const int64_t n_in = h->rows, n_out = h->cols;
    RC(ensure_aux(h, s));
    // the layer keeps x (as xT [n_in, batch]) for backward_dense, like _last_input
    RC(stage_transposed(h, x, batch, n_in, h->xT, s));
    h->last_batch = batch;
    const bool dev_out = is_device_ptr(y);
    float* yd = y;
    if (!dev_out) {
        RC(h->ytmp.reserve((int64_t)batch * n_out + 1));
        yd = h->ytmp.p;
    }
    if (h->timing) CK(cudaEventRecord(h->ev[0], s));
    RC(forward_columns(h, h->xT.p, batch, yd, false, s));
    if (h->b4_ntiles > 0) {
        RC(ensure_b4_index(h, s));
        RC(b4_forward(h, h->xT.p, batch, yd, s));
    }
    if (h->timing) { CK(cudaEventRecord(h->ev[1], s)); h->ev_fwd = true; }
    CK(cudaGetLastError());
    if (!dev_out) {
        CK(cudaMemcpyAsync(y, yd, (size_t)batch * n_out * 4, cudaMemcpyDeviceToHost, s));
    }
    if (!dev_out || !is_device_ptr(x)) {
        CK(cudaStreamSynchronize(s));
        RC(check_tc_err(h));
    }
    return SILI_OK;
}

// FoldedLayer.forward (sili/sparse_rnn.py:1096-1125) over its suffix layers:
// one transposed copy of x for all of them (every layer keeps it as its
// last input, as each layer's forward_dense would), then one launch of
// k_folded_cols where its shape rules hold, else each layer's forward into
// a raw buffer, the suffix sum and the fold sum.  The sums are the
// reference's: raw = 0 + raw_0 + raw_1 + ... (Python's sum), y[b, j] = raw
// folds added in ascending order (numpy's reduction over the fold axis).
int sili_folded_forward(sili_layer* const* layers, int n_layers, const float* x, int batch, int n_folds,
                        int64_t out_dim, int fold_sum, float* y, void* stream) {
    if (!layers || n_layers < 1 || batch < 0 || n_folds < 1 || out_dim < 1 || !x || !y)
        return fail(SILI_EINVAL, "folded_forward: bad arguments");
    sili_layer* h0 = layers[0];
    RC(use(h0));
    for (int k = 0; k < n_layers; ++k) {
        sili_layer* h = layers[k];
        if (!h) return fail(SILI_EINVAL, "folded_forward: null layer");
        if (h->dev != h0->dev || h->rows != h0->rows || h->cols != (int64_t)n_folds * out_dim)
            return fail(SILI_EINVAL, "folded_forward: every suffix layer must be n_in -> n_folds * out_dim on one device");
    }
    cudaStream_t s = pick(h0, stream);
    const int64_t n_in = h0->rows, n_cols = h0->cols;
    for (int k = 0; k < n_layers; ++k) RC(ensure_aux(layers[k], s));
    RC(stage_transposed(h0, x, batch, n_in, h0->xT, s));
    h0->last_batch = batch;
    for (int k = 1; k < n_layers; ++k) {
        sili_layer* h = layers[k];
        RC(h->xT.reserve((int64_t)batch * n_in + batch + 1));
        CK(cudaMemcpyAsync(h->xT.p, h0->xT.p, (size_t)(batch * n_in + batch) * 4, cudaMemcpyDeviceToDevice, s));
        h->last_batch = batch;
    }
    const int64_t y_count = (int64_t)batch * (fold_sum ? out_dim : n_cols);
    const bool dev_out = is_device_ptr(y);
    float* yd = y;
    if (!dev_out) {
        RC(h0->ytmp.reserve(y_count + 1));
        yd = h0->ytmp.p;
    }
    FoldedView F;
    F.ns = n_layers;
    F.n_in = (int)n_in;
    F.n_cols = n_cols;
    F.out_dim = out_dim;
    F.n_folds = n_folds;
    F.fold_sum = fold_sum != 0;
    // one suffix: the stacked layer's own forward and the fold sum in two
    // launches measured faster than the one-launch kernel on config 5's
    // shards at 1-8 ranks (the row-tiled forward keeps three 256-thread CTAs
    // per SM; the fold-grouped CTAs of k_folded_cols fewer); two to four
    // suffixes share one x staging in k_folded_cols
    bool fused = n_layers >= 2 && n_layers <= kFoldedMaxSuffixes && batch > 0;
    for (int k = 0; k < n_layers && fused; ++k) {
        sili_layer* h = layers[k];
        if (h->rank != 1 || h->b4_ntiles > 0 || h->total_nnz == 0) { fused = false; break; }
        const int64_t bound = std::max<int64_t>(h->total_nnz, 1) + 7 * h->cols + 8;
        if (!h->pack_valid) {
            RC(h->cpack.reserve(bound));
            launch_pack_csc(h->view(), bound, h->cpack.p, s);
            h->pack_valid = true;
        }
        F.colptr[k] = h->colptr.p; F.colptr_x[k] = h->colptr_x.p; F.cpack[k] = h->cpack.p;
        F.vs[k] = h->vs.p; F.os[k] = h->os.p;
    }
    if (h0->timing) CK(cudaEventRecord(h0->ev[0], s));
    if (!(fused && launch_folded_forward(F, h0->xT.p, batch, yd, s))) {
        // each layer's own forward into raw, then the sums
        const int64_t raw_count = (int64_t)batch * n_cols;
        DBuf<float>& raws = h0->fold_raw;   // kept across calls (no allocation per step)
        RC(raws.reserve(raw_count * n_layers + 1));
        std::vector<const float*> rp((size_t)n_layers);
        for (int k = 0; k < n_layers; ++k) {
            sili_layer* h = layers[k];
            float* rk = raws.p + raw_count * k;
            RC(forward_columns(h, h0->xT.p, batch, rk, false, s));
            if (h->b4_ntiles > 0) {
                RC(ensure_b4_index(h, s));
                launch_b4_forward(h->view(), h->b4view(), h0->xT.p, batch, rk, s);
            }
            rp[(size_t)k] = rk;
        }
        float* sum = fold_sum ? raws.p : yd;   // the suffix sum in place over raw_0 when folding after
        launch_suffix_sum(rp.data(), std::min(n_layers, kFoldedMaxSuffixes), raw_count, sum, s);
        for (int k0 = kFoldedMaxSuffixes; k0 < n_layers; k0 += kFoldedMaxSuffixes - 1) {
            std::vector<const float*> more = {sum};
            for (int k = k0; k < std::min(n_layers, k0 + kFoldedMaxSuffixes - 1); ++k) more.push_back(rp[(size_t)k]);
            launch_suffix_sum(more.data(), (int)more.size(), raw_count, sum, s);
        }
        if (fold_sum) launch_fold_sum(sum, batch, n_folds, out_dim, yd, s);
        CK(cudaGetLastError());
    }
    if (h0->timing) { CK(cudaEventRecord(h0->ev[1], s)); h0->ev_fwd = true; }
    CK(cudaGetLastError());
    if (!dev_out) CK(cudaMemcpyAsync(y, yd, (size_t)y_count * 4, cudaMemcpyDeviceToHost, s));
    if (!dev_out || !is_device_ptr(x)) CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// The block4 part of the fused update: tiles in parallel (passes over chunks
// of block-rows whose per-tile scratch stays within 4 GiB, then the eviction
// of every block-row) when every tile is full width, else one half-warp per
// block-row.
static int b4_update(sili_layer* h, const LayerView& v, int batch, const UpdateParams& P, cudaStream_t s) {
    const B4View V = h->b4view();
    if (!b4_update_split_applies(v)) {
        launch_b4_update(v, V, h->xT.p, h->dyT.p, batch, P, h->dxT.p, s);
        return SILI_OK;
    }
    if (P.os_trainable) RC(ensure_b4_index(h, s));   // the column sums walk it
    const int64_t BR = h->b4_BR;
    if (b4_update_rows_applies(v, batch) && !P.os_trainable) {
        // a warp per row: no per-tile scratch
        launch_b4_update_rows(v, V, h->xT.p, h->dyT.p, batch, P, h->dxT.p, 0, BR, 0, nullptr, s);
        launch_b4_evict_rows(v, V, s);
        return SILI_OK;
    }
    std::vector<int64_t> es((size_t)BR + 1);
    CK(cudaMemcpyAsync(es.data(), h->b4_es.p, (size_t)(BR + 1) * 8, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (b4_update_rows_applies(v, batch)) {
        // the output scale trains: per-slot column sums in parts of at most 4 GiB
        const int64_t per_tile = (int64_t)16 * h->rank * 2 * 4;
        const int64_t limit = std::max<int64_t>(1, ((int64_t)4 << 30) / per_tile);
        std::vector<std::pair<int64_t, int64_t>> parts;
        int64_t most = 1;
        for (int64_t br0 = 0; br0 < BR;) {
            int64_t br1 = br0 + 1;
            while (br1 < BR && es[br1 + 1] - es[br0] <= limit) ++br1;
            parts.emplace_back(br0, br1);
            most = std::max(most, es[br1] - es[br0]);
            br0 = br1;
        }
        RC(h->b4_mc.reserve(most * 16 * h->rank * 2 + 1));
        for (const auto& c : parts)
            launch_b4_update_rows(v, V, h->xT.p, h->dyT.p, batch, P, h->dxT.p, c.first, c.second, es[c.first],
                                  h->b4_mc.p, s);
        launch_b4_evict_rows(v, V, s);
        return SILI_OK;
    }
    const int64_t per_tile = (int64_t)4 * batch * 4 + (int64_t)4 * h->rank * 2 * 8 + (int64_t)16 * h->rank * 2 * 4;
    const int64_t limit = std::max<int64_t>(1, ((int64_t)4 << 30) / per_tile);   // 4 GiB
    std::vector<std::pair<int64_t, int64_t>> chunks;
    int64_t most = 1;
    for (int64_t br0 = 0; br0 < BR;) {
        int64_t br1 = br0 + 1;
        // (at most 65535 block-rows: the tile pass puts them on the grid's y axis)
        while (br1 < BR && br1 - br0 < 65535 && es[br1 + 1] - es[br0] <= limit) ++br1;
        chunks.emplace_back(br0, br1);
        most = std::max(most, es[br1] - es[br0]);
        br0 = br1;
    }
    RC(h->b4_hs.reserve(most * 4 * batch + 1));
    RC(h->b4_mr.reserve(most * 4 * h->rank * 2 + 1));
    if (P.os_trainable) RC(h->b4_mc.reserve(most * 16 * h->rank * 2 + 1));
    for (const auto& c : chunks)
        launch_b4_update_split(v, V, h->xT.p, h->dyT.p, batch, P, h->dxT.p, c.first, c.second, es[c.first],
                               h->b4_hs.p, h->b4_mr.p, h->b4_mc.p, s);
    launch_b4_evict_rows(v, V, s);
    return SILI_OK;
}

// part != nullptr: a column shard's backward (device array of
// sili_layer_row_part_len doubles, zeroed here; the row steps wait for
// sili_layer_apply_row_part)
static int backward_dense_impl(sili_layer* h, const float* x, const float* dy, int batch, float lr, unsigned flags,
                               float beta2, float eps, float* dx, cudaStream_t s, double* part) {
    const int64_t n_in = h->rows, n_out = h->cols;
    if (x) {
        RC(stage_transposed(h, x, batch, n_in, h->xT, s));
        h->last_batch = batch;
    } else if (h->last_batch != batch) {
        return fail(SILI_EINVAL, "backward_dense: dy batch differs from the last forward input");
    }
    RC(ensure_aux(h, s));
    const float* dyd = nullptr;
    RC(stage_in(h, dy, (size_t)batch * n_out, h->dy_stage, &dyd, s));
    RC(h->dyT.reserve((int64_t)batch * n_out + 1));
    // accumulators, linear_disldo.hpp:515-520 (the |dy| sums with dy's transpose)
    launch_accum_abs_t(h->xT.p, h->in_acc.p, batch, n_in, s);
    const unsigned long long dy_tag = (unsigned long long)h->call + 1;   // never 0, the flag's initial value
    launch_transpose_accum(dyd, h->dyT.p, batch, n_out, h->grad_acc.p, h->d_dyflag.p, dy_tag, s);
    const bool dev_out = is_device_ptr(dx);
    float* dxd = dx;
    if (!dev_out) {
        RC(h->dx_stage.reserve((int64_t)batch * n_in + 1));
        dxd = h->dx_stage.p;
    }
    LayerView v = h->view();
    if (lr == 0.0f) {
        if (h->timing) CK(cudaEventRecord(h->ev[2], s));
        launch_backward_dx(v, h->dyT.p, batch, dxd, s);
        if (h->b4_ntiles > 0) RC(b4_tc_or_exact(h, true, h->dyT.p, batch, dxd, s));
        if (h->timing) { CK(cudaEventRecord(h->ev[3], s)); h->ev_bwd = true; }
        h->call++;   // every backward call advances the stochastic-rounding counter
    } else {
        RC(h->dxT.reserve((int64_t)batch * n_in + 1));
        // pre-size the lazily sized scale vectors (linear_disldo.hpp:571-594)
        grow_logical(h, h->vs, h->n_vs, n_in * h->rank, 1.0f, s);
        grow_logical(h, h->os, h->n_os, n_out * h->rank, 1.0f, s);
        RC(ensure_pow_table(h, beta2, (uint32_t)(h->call + 2)));
        UpdateParams P = update_params(h, lr, flags, beta2, eps);
        P.stochastic = h->stochastic;
        P.os_trainable = h->os_trainable;
        P.dy_flag = h->d_dyflag.p;
        P.dy_tag = dy_tag;
        if (part) {
            if (P.resync) return fail(SILI_EINVAL, "backward_dense_shard: Resync layers are not column-sharded");
            P.row_nnz_g = h->shard_nnz.p;
            P.row_part = part;
        }
        if (P.resync) {
            if (batch > 128)
                return fail(SILI_EINVAL, "backward_dense: a Resync layer's update takes batches of at most 128 here");
            RC(h->def_cw.reserve(h->val_n + 1));
            RC(h->def_ci.reserve(h->val_n + 1));
            P.def_cw = h->def_cw.p;
            P.def_ci = h->def_ci.p;
        }
        h->call++;
        if (h->pack_valid) {
            // the update kernels rewrite the packed words of the codes they rewrite
            v.cpack_upd = h->cpack.p;
            v.fcpos = h->fcpos.p;
        }
        if (h->os_trainable) {
            CK(cudaMemsetAsync(h->colg.p, 0, (size_t)n_out * h->rank * 4, s));
            CK(cudaMemsetAsync(h->colc.p, 0, (size_t)n_out * h->rank * 4, s));
        }
        if (h->total_nnz > 0) {
            if (h->timing) CK(cudaEventRecord(h->ev[2], s));
            launch_backward_update(v, h->xT.p, h->dyT.p, batch, P, h->dxT.p, s);
            if (h->timing) { CK(cudaEventRecord(h->ev[3], s)); h->ev_bwd = true; }
            h->st_pending = true;
        } else {
            CK(cudaMemsetAsync(h->dxT.p, 0, (size_t)batch * n_in * 4, s));
        }
        // block4 part after the scattered one (linear_disldo.hpp:939-1951)
        if (h->b4_ntiles > 0) RC(b4_update(h, v, batch, P, s));
        if (part) {
            // rows with no synapse on any shard: this shard's columns' part of S
            if (h->shard_any_dead) launch_dead_S(v, dyd, batch, part + 2 * n_in * h->rank, s);
        } else if (h->has_dead_rows) {
            RC(h->dS.reserve((int64_t)batch * h->rank + 1));
            launch_dead_rows(v, h->xT.p, dyd, batch, h->dS.p, P, s);
        }
        if (h->os_trainable) launch_output_scale_update(v, h->out_degree.p, P, s);
        // the Resync classes store their codes only now, under the final scales
        if (P.resync && h->total_nnz > 0) launch_resync_store(v, P, s);
        launch_transpose(h->dxT.p, dxd, n_in, batch, s);
    }
    CK(cudaGetLastError());
    if (!dev_out) CK(cudaMemcpyAsync(dx, dxd, (size_t)batch * n_in * 4, cudaMemcpyDeviceToHost, s));
    if (!dev_out || !is_device_ptr(dy) || (x && !is_device_ptr(x))) {
        CK(cudaStreamSynchronize(s));
        RC(check_tc_err(h));
    }
    return SILI_OK;
}

int sili_layer_backward_dense(sili_layer* h, const float* x, const float* dy, int batch, float lr, unsigned flags,
                              float beta2, float eps, float* dx, void* stream) {
    RC(use(h));
    if (batch < 0 || !dy || !dx) return fail(SILI_EINVAL, "backward_dense: bad arguments");
    return backward_dense_impl(h, x, dy, batch, lr, flags, beta2, eps, dx, pick(h, stream), nullptr);
}

// ── column shards (a folded stack split by output column over ranks) ──────
// Each synapse update is local to its (row, column); lr / nnz_row, the row's
// value_scale step (sums over all its synapses, linear_disldo.hpp:901-925)
// and the dead-row bootstrap (S over all columns, :1985-2042) couple a row's
// columns.  A shard divides by the global counts, hands out its part of the
// row sums, and applies the row steps once the parts are summed.
int sili_layer_set_row_shard(sili_layer* h, const int* global_row_nnz, int64_t n, int64_t global_n_out) {
    RC(use(h));
    if (n == 0) { h->shard_on = false; return SILI_OK; }
    if (n != h->rows || !global_row_nnz || global_n_out <= 0)
        return fail(SILI_EINVAL, "set_row_shard: one global count per input row and a positive column count");
    if (h->b4_ntiles > 0) return fail(SILI_EINVAL, "set_row_shard: a layer with block4 tiles is not column-sharded");
    std::vector<int> g((size_t)n);
    if (is_device_ptr(global_row_nnz)) CK(cudaMemcpy(g.data(), global_row_nnz, (size_t)n * 4, cudaMemcpyDeviceToHost));
    else std::memcpy(g.data(), global_row_nnz, (size_t)n * 4);
    bool any_dead = false;
    for (int64_t r = 0; r < n; ++r) {
        if (g[r] < 0) return fail(SILI_EINVAL, "set_row_shard: negative synapse count");
        any_dead |= g[r] == 0;
    }
    RC(h->shard_nnz.reserve(n));
    CK(cudaMemcpy(h->shard_nnz.p, g.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
    h->shard_n_out = global_n_out;
    h->shard_any_dead = any_dead;
    h->shard_on = true;
    return SILI_OK;
}

int sili_layer_row_part_len(sili_layer* h, int batch, int64_t* n) {
    RC(use(h));
    if (!n || batch < 0) return fail(SILI_EINVAL, "row_part_len: bad arguments");
    *n = 2 * h->rows * h->rank + (int64_t)batch * h->rank;
    return SILI_OK;
}

int sili_layer_backward_dense_shard(sili_layer* h, const float* x, const float* dy, int batch, float lr,
                                    unsigned flags, float beta2, float eps, float* dx, double* part, void* stream) {
    RC(use(h));
    if (batch < 0 || !dy || !dx || !part) return fail(SILI_EINVAL, "backward_dense_shard: bad arguments");
    if (!h->shard_on) return fail(SILI_EINVAL, "backward_dense_shard: no row shard set (sili_layer_set_row_shard)");
    if (h->b4_ntiles > 0) return fail(SILI_EINVAL, "backward_dense_shard: a layer with block4 tiles is not column-sharded");
    cudaStream_t s = pick(h, stream);
    const int64_t len = 2 * h->rows * h->rank + (int64_t)batch * h->rank;
    double* pd = part;
    const bool dev_part = is_device_ptr(part);
    if (!dev_part) {
        RC(h->rpart.reserve(len + 1));
        pd = h->rpart.p;
    }
    CK(cudaMemsetAsync(pd, 0, (size_t)len * sizeof(double), s));
    RC(backward_dense_impl(h, x, dy, batch, lr, flags, beta2, eps, dx, s, pd));
    h->sh_lr = lr; h->sh_beta2 = beta2; h->sh_eps = eps; h->sh_flags = flags; h->sh_batch = batch;
    if (!dev_part) {
        CK(cudaMemcpyAsync(part, pd, (size_t)len * sizeof(double), cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
    }
    return SILI_OK;
}

int sili_layer_apply_row_part(sili_layer* h, const double* part, void* stream) {
    RC(use(h));
    if (!part) return fail(SILI_EINVAL, "apply_row_part: bad arguments");
    if (!h->shard_on || h->sh_batch < 0)
        return fail(SILI_EINVAL, "apply_row_part: no shard backward to complete (sili_layer_backward_dense_shard)");
    const int batch = h->sh_batch;
    h->sh_batch = -1;
    if (h->sh_lr == 0.0f) return SILI_OK;
    cudaStream_t s = pick(h, stream);
    const int64_t len = 2 * h->rows * h->rank + (int64_t)batch * h->rank;
    const double* pd = part;
    if (!is_device_ptr(part)) {
        RC(h->rpart.reserve(len + 1));
        CK(cudaMemcpyAsync(h->rpart.p, part, (size_t)len * sizeof(double), cudaMemcpyHostToDevice, s));
        pd = h->rpart.p;
    }
    UpdateParams P = update_params(h, h->sh_lr, h->sh_flags, h->sh_beta2, h->sh_eps);
    launch_apply_row_part(h->view(), h->shard_nnz.p, h->shard_n_out, pd, h->xT.p, batch, P, s);
    CK(cudaGetLastError());
    if (!is_device_ptr(part)) CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_layer_forward_sparse(sili_layer* h, const int* ptrs, const int* idx, const float* vals, int nnz, int batch,
                              float* y, void* stream) {
    RC(use(h));
    if (batch < 0 || !ptrs || !y || nnz < 0) return fail(SILI_EINVAL, "forward_sparse: bad arguments");
    cudaStream_t s = pick(h, stream);
    const int64_t n_in = h->rows, n_out = h->cols;
    RC(check_csr(ptrs, idx, batch, nnz, n_in, "forward_sparse"));
    RC(ensure_aux(h, s));
    const int* dp = nullptr;
    const int* di = nullptr;
    const float* dv = nullptr;
    RC(stage_csr(h, ptrs, idx, vals, batch, nnz, &dp, &di, &dv, s));
    // the densified input goes to its own buffer: forward_sparse leaves the
    // last forward_dense input (which backward_dense uses) alone, as the
    // reference's does (cpu_backend.cpp:571-585 never touches _last_input)
    RC(h->xsT.reserve((int64_t)batch * (n_in + 1) + 1));
    CK(cudaMemsetAsync(h->xsT.p, 0, (size_t)batch * (n_in + 1) * 4, s));   // + the zero row
    uint8_t* xpres = nullptr;
    if (h->b4_ntiles > 0) {
        RC(h->presX.reserve((int64_t)batch * n_in + 1));
        CK(cudaMemsetAsync(h->presX.p, 0, (size_t)batch * n_in, s));
        xpres = h->presX.p;
    }
    launch_csr_to_dense_t(dp, di, dv, batch, (int)n_in, h->xsT.p, xpres, s);
    h->sparse_batch = batch;
    const bool dev_out = is_device_ptr(y);
    float* yd = y;
    if (!dev_out) {
        RC(h->ytmp.reserve((int64_t)batch * n_out + 1));
        yd = h->ytmp.p;
    }
    if (h->total_nnz > 0) RC(forward_columns(h, h->xsT.p, batch, yd, true, s));
    else CK(cudaMemsetAsync(yd, 0, (size_t)batch * n_out * 4, s));
    if (h->b4_ntiles > 0) {
        RC(ensure_b4_index(h, s));
        launch_b4_forward_sparse(h->view(), h->b4view(), h->xsT.p, xpres, batch, yd, s);
    }
    CK(cudaGetLastError());
    if (!dev_out) CK(cudaMemcpyAsync(y, yd, (size_t)batch * n_out * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_layer_backward_sparse(sili_layer* h, const float* x, const int* dptrs, const int* didx, const float* dvals,
                               int dnnz, int batch, float lr, unsigned flags, float beta2, float eps, float* dx,
                               void* stream) {
    RC(use(h));
    if (batch < 0 || !x || !dptrs || !dx || dnnz < 0) return fail(SILI_EINVAL, "backward_sparse: bad arguments");
    cudaStream_t s = pick(h, stream);
    const int64_t n_in = h->rows, n_out = h->cols;
    RC(check_csr(dptrs, didx, batch, dnnz, n_out, "backward_sparse"));
    RC(ensure_aux(h, s));
    const float* dxin = nullptr;
    RC(stage_in(h, x, (size_t)batch * n_in, h->x_stage, &dxin, s));
    const int* dp = nullptr;
    const int* di = nullptr;
    const float* dv = nullptr;
    RC(stage_csr(h, dptrs, didx, dvals, batch, dnnz, &dp, &di, &dv, s));
    // accumulators, sisldo_ops.hpp:611-617 (the dy part below, from dyT)
    launch_accum_abs(dxin, h->in_acc.p, batch, n_in, s);
    // value_scale / value_scale_importance sized to n_in (sisldo_ops.hpp:622-625)
    grow_logical(h, h->vs, h->n_vs, n_in, 1.0f, s);
    RC(h->xT.reserve((int64_t)batch * n_in + 1));
    launch_transpose(dxin, h->xT.p, batch, n_in, s);
    RC(h->dyT.reserve((int64_t)batch * n_out + 1));
    RC(h->presT.reserve((int64_t)batch * n_out + 1));
    CK(cudaMemsetAsync(h->dyT.p, 0, (size_t)batch * n_out * 4, s));
    CK(cudaMemsetAsync(h->presT.p, 0, (size_t)batch * n_out, s));
    launch_csr_to_dense_t(dp, di, dv, batch, (int)n_out, h->dyT.p, h->presT.p, s);
    // neuron_grad_accum[c] += |v| over dy's entries in CSR order: per column
    // that is its samples in order, and an absent entry (0 in dyT) adds +0 to
    // a non-negative sum, so the per-column sum over dyT is the same sum
    launch_accum_abs_t(h->dyT.p, h->grad_acc.p, batch, n_out, s);
    RC(h->dxT.reserve((int64_t)batch * n_in + 1));
    RC(h->sgs.reserve(n_in + 1)); RC(h->sgc.reserve(n_in + 1));
    RC(ensure_pow_table(h, beta2, (uint32_t)(h->call + 2)));
    UpdateParams P = update_params(h, lr, flags, beta2, eps);
    h->call++;
    if (lr != 0.0f) h->pack_valid = false;
    LayerView v = h->view();
    if (h->total_nnz > 0) {
        launch_backward_sparse(v, h->xT.p, h->dyT.p, h->presT.p, batch, P, h->sgs.p, h->sgc.p, h->dxT.p, s);
        if (lr != 0.0f) {
            h->st_pending = true;
            launch_sparse_scale_update(v, h->sgs.p, h->sgc.p, P, s);
        }
    } else {
        CK(cudaMemsetAsync(h->dxT.p, 0, (size_t)batch * n_in * 4, s));
    }
    // block4 part after the scattered one (sisldo_ops.hpp:835-1104)
    if (h->b4_ntiles > 0) {
        launch_b4_backward_sparse(v, h->b4view(), h->xT.p, h->dyT.p, h->presT.p, batch, P, h->dxT.p, s);
        if (lr != 0.0f) h->st_pending = true;
    }
    const bool dev_out = is_device_ptr(dx);
    float* dxd = dx;
    DBuf<float> dxtmp;
    if (!dev_out) {
        RC(dxtmp.reserve((int64_t)batch * n_in + 1));
        dxd = dxtmp.p;
    }
    launch_transpose(h->dxT.p, dxd, n_in, batch, s);
    CK(cudaGetLastError());
    if (!dev_out) CK(cudaMemcpyAsync(dx, dxd, (size_t)batch * n_in * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// ── synaptogenesis: probes ──────────────────────────────────────────────────
// delta_csr_build_probes (delta_csr_memory.hpp:1308-1427).  Top-k by a stable
// descending radix sort (ties keep ascending index; the reference's
// partial_sort leaves tie order unspecified).
static int sorted_desc(sili_layer* h, const float* keys, int64_t n, DBuf<int>& out_idx) {
    cudaStream_t s = h->stream;
    DBuf<float>& ko = h->pb_keys;
    DBuf<int>& vin = h->pb_iota;
    RC(ko.reserve(n + 1)); RC(vin.reserve(n + 1)); RC(out_idx.reserve(n + 1));
    launch_iota(vin.p, n, s);
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairsDescending(nullptr, bytes, keys, ko.p, vin.p, out_idx.p, (int)n, 0, 32, s);
    RC(h->cub_tmp.reserve((int64_t)bytes + 1));
    CK(cub::DeviceRadixSort::SortPairsDescending(h->cub_tmp.p, bytes, keys, ko.p, vin.p, out_idx.p, (int)n, 0, 32, s));
    return SILI_OK;
}

int sili_layer_build_probes(sili_layer* h, int k, int per_row) {
    RC(use(h));
    if (k > 0 && (int64_t)k * std::min<int64_t>(k, h->rows) > (int64_t)1 << 30)
        return fail(SILI_EINVAL, "build_probes: k too large");
    cudaStream_t s = h->stream;
    const int64_t R = h->rows, C = h->cols;
    h->n_probes = 0;
    if (R == 0 || C == 0 || k <= 0) return SILI_OK;
    RC(ensure_aux(h, s));
    const int kin = (int)std::min<int64_t>(k, R);
    DBuf<int>& in_sorted = h->pb_in;
    DBuf<int>& out_sorted = h->pb_out;
    RC(sorted_desc(h, h->in_acc.p, R, in_sorted));
    RC(sorted_desc(h, h->grad_acc.p, C, out_sorted));
    LayerView v = h->view();
    if (!per_row) {
        const int kout = (int)std::min<int64_t>(k, C);
        const int64_t n = (int64_t)kin * kout;
        DBuf<int>& flags = h->pb_flags;
        DBuf<int>& pos = h->pb_pos;
        RC(flags.reserve(n + 1)); RC(pos.reserve(n + 1));
        CK(cudaMemsetAsync(flags.p, 0, (size_t)(n + 1) * 4, s));
        launch_probe_flags(v, in_sorted.p, kin, out_sorted.p, kout, flags.p, s);
        RC(scan_excl_int(h, flags.p, pos.p, n + 1, s));
        int total = 0;
        CK(cudaMemcpyAsync(&total, pos.p + n, 4, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        RC(h->prow.reserve(total + 1)); RC(h->pcol.reserve(total + 1)); RC(h->pval.reserve(total + 1));
        launch_probe_emit(in_sorted.p, kin, out_sorted.p, kout, flags.p, pos.p, h->in_acc.p, h->grad_acc.p,
                          h->prow.p, h->pcol.p, h->pval.p, s);
        h->n_probes = total;
    } else {
        const int64_t cap = (int64_t)kin * k;
        DBuf<int>& tr = h->pb_tr;
        DBuf<int>& tc = h->pb_tc;
        DBuf<int>& counts = h->pb_counts;
        DBuf<float>& tv = h->pb_tv;
        RC(tr.reserve(cap + 1)); RC(tc.reserve(cap + 1)); RC(tv.reserve(cap + 1)); RC(counts.reserve(kin + 1));
        launch_probe_per_row(v, in_sorted.p, kin, out_sorted.p, C, k, h->in_acc.p, h->grad_acc.p, tr.p, tc.p, tv.p,
                             counts.p, s);
        std::vector<int> hc(kin);
        CK(cudaMemcpyAsync(hc.data(), counts.p, (size_t)kin * 4, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        int64_t total = 0;
        for (int a = 0; a < kin; ++a) total += hc[a];
        RC(h->prow.reserve(total + 1)); RC(h->pcol.reserve(total + 1)); RC(h->pval.reserve(total + 1));
        int64_t o = 0;
        for (int a = 0; a < kin; ++a) {
            if (!hc[a]) continue;
            const size_t off = (size_t)a * k;
            CK(cudaMemcpyAsync(h->prow.p + o, tr.p + off, (size_t)hc[a] * 4, cudaMemcpyDeviceToDevice, s));
            CK(cudaMemcpyAsync(h->pcol.p + o, tc.p + off, (size_t)hc[a] * 4, cudaMemcpyDeviceToDevice, s));
            CK(cudaMemcpyAsync(h->pval.p + o, tv.p + off, (size_t)hc[a] * 4, cudaMemcpyDeviceToDevice, s));
            o += hc[a];
        }
        h->n_probes = total;
    }
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_layer_num_probes(sili_layer* h, int64_t* n) {
    RC(use(h));
    *n = h->n_probes;
    return SILI_OK;
}

int sili_layer_get_probes(sili_layer* h, int* rows, int* cols, float* scores) {
    RC(use(h));
    const size_t n = (size_t)h->n_probes;
    RC(from_dev(h->prow.p, rows, n * 4, h->stream));
    RC(from_dev(h->pcol.p, cols, n * 4, h->stream));
    RC(from_dev(h->pval.p, scores, n * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

int sili_layer_synap_rows(sili_layer* h, int row0, int nrows, float importance_cutoff, int max_row_weights,
                          int max_prune_per_step, float importance_eps, uint8_t* did) {
    RC(use(h));
    cudaStream_t s = h->stream;
    const int64_t R = h->rows, C = h->cols, BR = h->b4_BR;
    if (nrows <= 0 || R == 0) return SILI_OK;
    if (max_prune_per_step < 0) return fail(SILI_EINVAL, "synap_rows: max_prune_per_step < 0");
    RC(synap_prepare(h, nrows, s));
    SynState& Z = h->syn;
    // snapshot of everything a sweep may change
    RC(snapshot_state(h, true, s));
    SynView V = synap_view(h);
    SynParams P;
    P.row0 = row0; P.nrows = nrows; P.limit = nrows - 1;
    P.cutoff = importance_cutoff; P.eps = importance_eps; P.max_rw = max_row_weights; P.max_prune = max_prune_per_step;
    bool sequential = false;
    for (int attempt = 0; attempt < 4; ++attempt) {
        RC(synap_reset_results(h, nrows, s));
        launch_synap(V, P, sequential, s);
        CK(cudaGetLastError());
        launch_od_check(Z.od0.p, Z.od_decs.p, C, reinterpret_cast<int*>(Z.res.p + 6), s);
        long long res[8];
        CK(cudaMemcpyAsync(res, Z.res.p, sizeof(res), cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        const unsigned long long grow_i = (unsigned long long)res[0], grow_t = (unsigned long long)res[1];
        const long long err_i = res[3];
        const int err_code = (int)(res[4] & 0xFFFFFFFF), flags = (int)(res[6] & 0xFFFFFFFF);
        if (flags & 4) return fail(SILI_ECUDA, "synap_rows: block4 tile capacity reservation too small");
        const bool over_budget = V.tot_idx0 + (int64_t)grow_i > h->b4_max_idx || V.tot_tile0 + (int64_t)grow_t > h->b4_max_tile;
        if (!sequential && ((flags & 1) || over_budget)) {
            // order-dependent: re-run the whole sweep in order, in one thread
            RC(snapshot_state(h, false, s));
            sequential = true;
            continue;
        }
        if (!sequential && err_i != LLONG_MAX && P.limit != err_i) {
            // stop at the first failing row, as the reference does
            RC(snapshot_state(h, false, s));
            P.limit = err_i;
            continue;
        }
        h->total_nnz += (int64_t)res[2];
        h->aux_dirty = true;
        h->b4_dirty = true;
    h->b4_pmap_dirty = h->b4_pmapT_dirty = true;
        std::vector<int> nt((size_t)BR + 1, 0);
        if (BR > 0) CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)BR * 4, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        h->b4_ntiles = 0;
        for (int64_t br = 0; br < BR; ++br) h->b4_ntiles += nt[(size_t)br];
        if (did) RC(from_dev(Z.did.p, did, (size_t)nrows, s));
        CK(cudaStreamSynchronize(s));
        if (err_i != LLONG_MAX) {
            const int64_t r = ((int64_t)row0 + err_i) % R;
            if (err_code == SILI_ENOMEM)
                return fail(SILI_ENOMEM, "synap_row_step: block4 budget exceeded at row " + std::to_string(r));
            return fail(SILI_EHEADROOM, "delta_csr_synap_row_step: row " + std::to_string(r) +
                                            " ran out of blank space. Call equalizer_step() to redistribute space "
                                            "from adjacent rows before retrying, or reduce max_row_weights / raise "
                                            "importance_cutoff.");
        }
        return SILI_OK;
    }
    return fail(SILI_ECUDA, "synap_rows: no consistent result");
}

// ── headroom management ─────────────────────────────────────────────────────
// delta_csr_shift_row (delta_csr_memory.hpp:225-293) for one row: the tail of
// both buffers after the row moves by the allocation change (a memmove, as in
// the reference, so blank bytes keep their old contents).
static int shift_row(sili_layer* h, HostLayout& L, int64_t row, int64_t tb, int64_t te) {
    cudaStream_t s = h->stream;
    const int64_t R = h->rows;
    const int64_t cb = L.bs[row + 1] - L.bs[row];
    if (cb != tb && row + 1 < R) {
        const int64_t src = L.bs[row + 1], len = L.bs[R] - src, dst = L.bs[row] + tb;
        int64_t nt = h->idx_n;
        if (tb > cb) {
            nt = h->idx_n + (tb - cb);
            if (nt > h->max_idx_bytes) return fail(SILI_ENOMEM, "std::bad_alloc");
            RC(h->idx.grow(nt + 64, h->idx_n, s));
            CK(cudaMemsetAsync(h->idx.p + h->idx_n, 0, (size_t)(nt - h->idx_n), s));
        }
        if (len > 0) {
            DBuf<uint8_t> tmp;
            RC(tmp.reserve(len));
            CK(cudaMemcpyAsync(tmp.p, h->idx.p + src, (size_t)len, cudaMemcpyDeviceToDevice, s));
            CK(cudaMemcpyAsync(h->idx.p + dst, tmp.p, (size_t)len, cudaMemcpyDeviceToDevice, s));
            CK(cudaStreamSynchronize(s));
        }
        if (tb < cb) nt = h->idx_n - (cb - tb);
        h->idx_n = nt;
        const int64_t d = tb - cb;
        for (int64_t r = row + 1; r <= R; ++r) L.bs[r] += d;
        for (int64_t r = row + 1; r < R; ++r) L.be[r] += d;
    }
    const int64_t ce = L.es[row + 1] - L.es[row];
    if (ce != te && row + 1 < R) {
        const int64_t src = L.es[row + 1], len = L.es[R] - src, dst = L.es[row] + te;
        const int64_t cur = L.es[R];
        if (te > ce) {
            const int64_t nt = cur + (te - ce);
            if (nt > h->max_val_bytes) { RC(put_layout(h, L)); return fail(SILI_ENOMEM, "std::bad_alloc"); }
            RC(h->val.grow(nt + 64, h->val_n, s));
            CK(cudaMemsetAsync(h->val.p + h->val_n, 0, (size_t)(nt - h->val_n), s));
            h->val_n = nt;
        }
        if (len > 0) {
            DBuf<uint8_t> tmp;
            RC(tmp.reserve(len));
            CK(cudaMemcpyAsync(tmp.p, h->val.p + src, (size_t)len, cudaMemcpyDeviceToDevice, s));
            CK(cudaMemcpyAsync(h->val.p + dst, tmp.p, (size_t)len, cudaMemcpyDeviceToDevice, s));
            CK(cudaStreamSynchronize(s));
        }
        if (te < ce) h->val_n = cur - (ce - te);
        const int64_t d = te - ce;
        for (int64_t r = row + 1; r <= R; ++r) L.es[r] += d;
        for (int64_t r = row + 1; r < R; ++r) L.ee[r] += d;
    }
    return SILI_OK;
}

int sili_layer_equalize_row(sili_layer* h, int row_in) {
    RC(use(h));
    if (h->rows == 0) return SILI_OK;
    const int64_t R = h->rows, row = row_in % R;
    HostLayout L;
    RC(get_layout(h, L));
    const int64_t tb = (L.bs[R] + R - 1) / R, te = (L.es[R] + R - 1) / R;
    const int rc = shift_row(h, L, row, tb, te);
    RC(put_layout(h, L));
    h->aux_dirty = true;
    return rc;
}

// equalize_to_capacity (cpu_backend.cpp:684-729).  The reference shifts rows
// one by one; the final allocations are max(current, target) per row, so the
// arrays are rebuilt once.  A budget failure leaves the rows before the
// failing one grown, as the reference's sequence of shifts would.
int sili_layer_equalize_to_capacity(sili_layer* h, int target_elems, int target_bytes) {
    RC(use(h));
    const int64_t R = h->rows;
    const int64_t te = target_elems, tb = target_bytes > 0 ? target_bytes : te * 5 + 4;
    HostLayout L;
    RC(get_layout(h, L));
    HostLayout N = L;
    int64_t idx_total = h->idx_n, val_total = L.es[R];
    int status = SILI_OK;
    std::vector<int64_t> ab(R), ae(R);
    for (int64_t r = 0; r < R; ++r) { ab[r] = L.bs[r + 1] - L.bs[r]; ae[r] = L.es[r + 1] - L.es[r]; }
    for (int64_t r = 0; r + 1 < R; ++r) {
        const int64_t ub = std::max(ab[r], tb), ue = std::max(ae[r], te);
        if (ub == ab[r] && ue == ae[r]) continue;
        if (ub > ab[r]) {
            if (idx_total + (ub - ab[r]) > h->max_idx_bytes) { status = SILI_ENOMEM; break; }
            idx_total += ub - ab[r];
        }
        ab[r] = ub;
        if (ue > ae[r]) {
            if (val_total + (ue - ae[r]) > h->max_val_bytes) { status = SILI_ENOMEM; break; }
            val_total += ue - ae[r];
        }
        ae[r] = ue;
    }
    if (status == SILI_OK && R > 0) {
        const int64_t r = R - 1;
        const int64_t ub = std::max(ab[r], tb), ue = std::max(ae[r], te);
        if (ub > ab[r]) { idx_total += ub - ab[r]; ab[r] = ub; }
        if (ue > ae[r]) { val_total += ue - ae[r]; ae[r] = ue; }
    }
    for (int64_t r = 0; r < R; ++r) {
        N.bs[r + 1] = N.bs[r] + ab[r];
        N.be[r] = N.bs[r] + (L.be[r] - L.bs[r]);
        N.es[r + 1] = N.es[r] + ae[r];
        N.ee[r] = N.es[r] + (L.ee[r] - L.es[r]);
    }
    RC(relayout(h, N, N.bs[R], N.es[R], false));
    if (status) return fail(status, "std::bad_alloc");
    return SILI_OK;
}

// compact (sisldo_ops.hpp:44-96): rows packed back to back, zero headroom.
int sili_layer_compact(sili_layer* h) {
    RC(use(h));
    const int64_t R = h->rows;
    HostLayout L, N;
    RC(get_layout(h, L));
    N = L;
    N.bs[0] = N.es[0] = 0;
    for (int64_t r = 0; r < R; ++r) {
        N.be[r] = N.bs[r] + (L.be[r] - L.bs[r]);
        N.bs[r + 1] = N.be[r];
        N.ee[r] = N.es[r] + (L.ee[r] - L.es[r]);
        N.es[r + 1] = N.ee[r];
    }
    return relayout(h, N, N.bs[R], N.es[R], true);
}

// expand_headroom / expand_headroom_to (sisldo_ops.hpp:127-186): the
// delta_csr_from_absolute layout of the live content, after the same budget
// requests the reference makes against the layer's limits.
static int expand(sili_layer* h, int64_t budget, float bf) {
    const double f = 1.0 + (double)bf;
    const int64_t ibytes = (int64_t)((double)budget * f * 6.0 + 4096.0);
    const int64_t vbytes = (int64_t)((double)budget * f) + 64;
    if (vbytes > h->max_val_bytes || ibytes > h->max_idx_bytes) return fail(SILI_ENOMEM, "std::bad_alloc");
    const int64_t R = h->rows;
    HostLayout L, N;
    RC(get_layout(h, L));
    N = L;
    N.bs[0] = N.es[0] = 0;
    for (int64_t r = 0; r < R; ++r) {
        const int64_t nb = L.be[r] - L.bs[r], n = L.ee[r] - L.es[r];
        N.be[r] = N.bs[r] + nb;
        N.bs[r + 1] = N.be[r] + (int64_t)((float)nb * bf) + 5;
        N.ee[r] = N.es[r] + n;
        N.es[r + 1] = N.ee[r] + std::max<int64_t>(1, (int64_t)((float)n * bf) + 1);
    }
    RC(relayout(h, N, N.bs[R], N.es[R], true));
    h->max_idx_bytes = h->idx_budget;
    h->max_val_bytes = h->val_budget;
    return SILI_OK;
}
int sili_layer_expand_headroom(sili_layer* h, float bf) {
    RC(use(h));
    return expand(h, h->total_nnz, bf);
}
int sili_layer_expand_headroom_to(sili_layer* h, int min_nnz_per_row, float bf) {
    RC(use(h));
    return expand(h, std::max<int64_t>(h->total_nnz, h->rows * (int64_t)min_nnz_per_row), bf);
}

int sili_layer_zero_accum(sili_layer* h) {
    RC(use(h));
    CK(cudaMemsetAsync(h->in_acc.p, 0, (size_t)h->rows * 4, h->stream));
    CK(cudaMemsetAsync(h->grad_acc.p, 0, (size_t)h->cols * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

// Predicates for cub::DeviceSelect over flat (r, c) positions
struct KeyGreater {
    const uint32_t* keys; uint32_t t;
    __host__ __device__ bool operator()(const int64_t& i) const { return keys[i] > t; }
};
struct KeyEqual {
    const uint32_t* keys; uint32_t t;
    __host__ __device__ bool operator()(const int64_t& i) const { return keys[i] == t; }
};

int sili_layer_topk_dyx_step(sili_layer* h, const float* x, const float* dy, int batch, int64_t k, void* stream) {
    RC(use(h));
    if (batch <= 0 || !x || !dy || k < 0) return fail(SILI_EINVAL, "topk_dyx_step: bad arguments");
    if (h->b4_ntiles > 0) return fail(SILI_EINVAL, "topk_dyx_step: defined on the scattered store (layer has block4 tiles)");
    cudaStream_t s = pick(h, stream);
    const int64_t R = h->rows, C = h->cols, n = R * C, nnz = h->total_nnz;
    if (n >= ((int64_t)1 << 31)) return fail(SILI_EINVAL, "topk_dyx_step: n_in * n_out must be below 2^31");
    RC(ensure_aux(h, s));
    const int64_t total_ne = n - nnz;
    if (k > total_ne) k = total_ne;
    const int64_t nc = std::max<int64_t>(k, 0);
    const int64_t npr = std::min(nc, nnz), nn = nnz - npr + nc;
    if (nn + 64 > h->max_val_bytes || nn * 8 + 4096 > h->max_idx_bytes)
        return fail(SILI_ENOMEM, "topk_dyx_step: rebuild exceeds the layer's byte budget");
    TopkState& T = h->topk;
    const float* dx_ = nullptr;
    const float* ddy = nullptr;
    RC(stage_in(h, x, (size_t)batch * R, h->x_stage, &dx_, s));
    RC(stage_in(h, dy, (size_t)batch * C, h->dy_stage, &ddy, s));
    const int64_t words = (C + 31) / 32;
    RC(T.bits.reserve(R * words + 1)); RC(T.keys.reserve(n + 1));
    CK(cudaMemsetAsync(T.bits.p, 0, (size_t)(R * words + 1) * 4, s));
    LayerView v = h->view();
    launch_exist_bits(h->rowptr.p, h->abs_cols.p, R, words, T.bits.p, s);
    launch_dyx_scores(dx_, ddy, batch, R, C, T.bits.p, words, T.keys.p, s);
    // radix select of the k-th largest key on the device, 8 bits at a time
    // from the top; one read-back of its result
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->dev);
    RC(T.hist.reserve(256)); RC(T.sel.reserve(1)); RC(T.nge.reserve(1));
    SelState st{0u, 0u, 0, 0};
    if (nc > 0) {
        CK(cudaMemsetAsync(T.hist.p, 0, 256 * sizeof(unsigned int), s));
        launch_sel_init(T.sel.p, nc, s);
        for (int shift = 24; shift >= 0; shift -= 8) {
            launch_digit_hist(T.keys.p, n, shift, T.sel.p, T.hist.p, sms, s);
            launch_digit_pick(T.hist.p, shift, T.sel.p, s);
        }
        CK(cudaMemcpyAsync(&st, T.sel.p, sizeof st, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
    }
    const uint32_t thr = st.prefix;
    const int64_t need = st.need, eq_count = st.eq_count;
    // candidates: every key above the threshold, then the first `need` equal
    // keys in (r, c) order; merged into (r, c) order
    RC(T.cand.reserve(nc + 1)); RC(T.cand_o.reserve(nc + 1)); RC(T.nsel.reserve(2));
    if (nc > 0 && need == eq_count) {
        // every key equal to the threshold is taken: the candidates are the
        // keys >= thr, gathered in one pass and sorted into (r, c) order
        CK(cudaMemsetAsync(T.nge.p, 0, sizeof(unsigned long long), s));
        launch_select_ge(T.keys.p, n, T.sel.p, T.cand.p, T.nge.p, nc, sms, s);
        size_t b3 = 0;
        cub::DeviceRadixSort::SortKeys(nullptr, b3, T.cand.p, T.cand_o.p, (int)nc, 0, 64, s);
        RC(h->cub_tmp.reserve((int64_t)b3 + 1));
        CK(cub::DeviceRadixSort::SortKeys(h->cub_tmp.p, b3, T.cand.p, T.cand_o.p, (int)nc, 0, 64, s));
    } else if (nc > 0) {
        int64_t n_gt = 0;
        cub::CountingInputIterator<int64_t> it(0);
        RC(T.eq.reserve(eq_count + 1));
        size_t b1 = 0, b2 = 0;
        cub::DeviceSelect::If(nullptr, b1, it, T.cand.p, T.nsel.p, (int)n, KeyGreater{T.keys.p, thr}, s);
        cub::DeviceSelect::If(nullptr, b2, it, T.eq.p, T.nsel.p + 1, (int)n, KeyEqual{T.keys.p, thr}, s);
        RC(h->cub_tmp.reserve((int64_t)std::max(b1, b2) + 1));
        b1 = std::max(b1, b2);
        CK(cub::DeviceSelect::If(h->cub_tmp.p, b1, it, T.cand.p, T.nsel.p, (int)n, KeyGreater{T.keys.p, thr}, s));
        int64_t sel[2] = {0, 0};
        CK(cudaMemcpyAsync(sel, T.nsel.p, 8, cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        n_gt = sel[0];
        b2 = b1;
        CK(cub::DeviceSelect::If(h->cub_tmp.p, b2, it, T.eq.p, T.nsel.p + 1, (int)n, KeyEqual{T.keys.p, thr}, s));
        if (n_gt + need != nc) return fail(SILI_ECUDA, "topk_dyx_step: selection count mismatch");
        CK(cudaMemcpyAsync(T.cand.p + n_gt, T.eq.p, (size_t)need * 8, cudaMemcpyDeviceToDevice, s));
        size_t b3 = 0;
        cub::DeviceRadixSort::SortKeys(nullptr, b3, T.cand.p, T.cand_o.p, (int)nc, 0, 64, s);
        RC(h->cub_tmp.reserve((int64_t)b3 + 1));
        CK(cub::DeviceRadixSort::SortKeys(h->cub_tmp.p, b3, T.cand.p, T.cand_o.p, (int)nc, 0, 64, s));
    }
    // prune: the npr existing synapses of smallest |w * S|, ties in (r, c) order
    DBuf<int>& di = T.di;
    DBuf<float>& dw = T.dw;
    DBuf<float>& dm = T.dm;
    RC(di.reserve(nnz + 1)); RC(dw.reserve(nnz + 1)); RC(dm.reserve(nnz + 1));
    launch_export(v, di.p, dw.p, dm.p, s);
    RC(T.pk.reserve(nnz + 1)); RC(T.pk_o.reserve(nnz + 1)); RC(T.pid.reserve(nnz + 1)); RC(T.pid_o.reserve(nnz + 1));
    RC(T.drop.reserve(nnz + 1));
    CK(cudaMemsetAsync(T.drop.p, 0, (size_t)nnz + 1, s));
    if (npr > 0) {
        launch_prune_keys(v, dw.p, T.pk.p, T.pid.p, s);
        size_t b4 = 0;
        cub::DeviceRadixSort::SortPairs(nullptr, b4, T.pk.p, T.pk_o.p, T.pid.p, T.pid_o.p, (int)nnz, 0, 32, s);
        RC(h->cub_tmp.reserve((int64_t)b4 + 1));
        CK(cub::DeviceRadixSort::SortPairs(h->cub_tmp.p, b4, T.pk.p, T.pk_o.p, T.pid.p, T.pid_o.p, (int)nnz, 0, 32, s));
        launch_mark_drop(T.pid_o.p, (int)npr, h->abs_cols.p, T.drop.p, h->out_degree.p, s);
    }
    // merge rows, rebuild with delta_csr_from_absolute's headroom
    RC(T.cptr.reserve(R + 1)); RC(T.cnt.reserve(R + 1)); RC(T.nptr.reserve(R + 1));
    launch_cand_rowptr(T.cand_o.p, (int)nc, C, R, T.cptr.p, s);
    CK(cudaMemsetAsync(T.cnt.p, 0, (size_t)(R + 1) * 4, s));
    launch_topk_merge(v, dw.p, dm.p, T.drop.p, T.cand_o.p, T.keys.p, T.cptr.p, 0, T.cnt.p, nullptr, nullptr, nullptr,
                      nullptr, h->out_degree.p, s);
    RC(scan_excl_int(h, T.cnt.p, T.nptr.p, R + 1, s));
    DBuf<int>& nidx = T.nidx;
    DBuf<float>& nw = T.nw;
    DBuf<float>& nimp = T.nimp;
    RC(nidx.reserve(nn + 1)); RC(nw.reserve(nn + 1)); RC(nimp.reserve(nn + 1));
    launch_topk_merge(v, dw.p, dm.p, T.drop.p, T.cand_o.p, T.keys.p, T.cptr.p, 1, T.cnt.p, T.nptr.p, nidx.p, nw.p,
                      nimp.p, h->out_degree.p, s);
    CK(cudaGetLastError());
    // the rebuild runs on the layer's own stream: its inputs, written above on
    // the caller's stream, must be complete first
    CK(cudaStreamSynchronize(s));
    RC(import_csr(h, T.nptr.p, nidx.p, nw.p, (int)nn, nimp.p));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// ── export ──────────────────────────────────────────────────────────────────
int sili_layer_sizes(sili_layer* h, int64_t* sizes) {
    RC(use(h));
    sizes[0] = h->rows; sizes[1] = h->cols; sizes[2] = h->total_nnz;
    sizes[3] = h->idx_n; sizes[4] = h->val_n; sizes[5] = h->b4_ntiles;
    return SILI_OK;
}

int sili_layer_export(sili_layer* h, int* ptrs, int* idx, float* w, float* imp) {
    RC(use(h));
    cudaStream_t s = h->stream;
    RC(ensure_aux(h, s));
    if (h->b4_ntiles > 0) return export_combined(h, ptrs, idx, w, imp, s);
    const int64_t nnz = h->total_nnz;
    DBuf<int> di;
    DBuf<float> dw, dm;
    RC(di.reserve(nnz + 1)); RC(dw.reserve(nnz + 1)); RC(dm.reserve(nnz + 1));
    launch_export(h->view(), di.p, dw.p, dm.p, s);
    CK(cudaGetLastError());
    RC(from_dev(h->rowptr.p, ptrs, (size_t)(h->rows + 1) * 4, s));
    RC(from_dev(di.p, idx, (size_t)nnz * 4, s));
    RC(from_dev(dw.p, w, (size_t)nnz * 4, s));
    RC(from_dev(dm.p, imp, (size_t)nnz * 4, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_layer_raw(sili_layer* h, int64_t* bs, int64_t* be, int64_t* es, int64_t* ee, uint8_t* indices,
                   uint8_t* values) {
    RC(use(h));
    cudaStream_t s = h->stream;
    const size_t R = (size_t)h->rows;
    RC(from_dev(h->bs.p, bs, (R + 1) * 8, s));
    RC(from_dev(h->be.p, be, R * 8, s));
    RC(from_dev(h->es.p, es, (R + 1) * 8, s));
    RC(from_dev(h->ee.p, ee, R * 8, s));
    RC(from_dev(h->idx.p, indices, (size_t)h->idx_n, s));
    RC(from_dev(h->val.p, values, (size_t)h->val_n, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// ── checkpoint: the whole training state as one flat image ─────────────────
// The reference's state dict (sili/sparse_rnn.py:817-851) carries weights and
// the per-row scales only; importance cannot be restored there.  The image
// holds everything a training run reads: the delta-CSR layout with its
// headroom (value positions key the stochastic rounding draws), the value
// bytes (weight and importance codes), every scale / optimiser vector and
// step counter, the accumulators, out_degree, the running statistics and the
// RNG seed and call counter.  A layer loaded from it continues bit for bit.
// Layout: CkptHead, then each section in ckpt_sections() order at a 16-byte
// aligned offset.  Block4 tiles are not part of it.
struct CkptHead {
    uint64_t magic;
    uint32_t version, rank;
    int64_t rows, cols;
    uint64_t seed, call;
    int64_t idx_n, val_n, total_nnz, max_idx_bytes, max_val_bytes, idx_budget, val_budget, n_vs, n_os;
    double st[4];
    float st_vmax, st_imax, max_abs_decay;
    int32_t os_trainable, stochastic, reserved;
};
constexpr uint64_t kCkptMagic = 0x3130434B42494C53ULL;   // "SLIBKC01"
constexpr uint32_t kCkptVersion = 1;
static size_t ckpt_align(size_t n) { return (n + 15) & ~(size_t)15; }

struct CkptSec { void* dev; size_t bytes; };
static std::vector<CkptSec> ckpt_sections(sili_layer* h) {
    const size_t R = (size_t)h->rows, C = (size_t)h->cols, k = (size_t)h->rank;
    return {{h->bs.p, (R + 1) * 8}, {h->be.p, R * 8}, {h->es.p, (R + 1) * 8}, {h->ee.p, R * 8},
            {h->idx.p, (size_t)h->idx_n}, {h->val.p, (size_t)h->val_n},
            {h->vs.p, R * k * 4}, {h->os.p, C * k * 4}, {h->vsi.p, R * k * 4}, {h->osi.p, C * k * 4},
            {h->vsm.p, R * k * 4}, {h->is.p, R * 4}, {h->ois.p, C * 4},
            {h->vstep.p, R * k * 4}, {h->ostep.p, C * k * 4},
            {h->in_acc.p, R * 4}, {h->grad_acc.p, C * 4}, {h->out_degree.p, C * 4}};
}
static int64_t ckpt_bytes(sili_layer* h) {
    size_t n = ckpt_align(sizeof(CkptHead));
    for (const auto& sec : ckpt_sections(h)) n += ckpt_align(sec.bytes);
    return (int64_t)n;
}

int sili_layer_state_size(sili_layer* h, int64_t* bytes) {
    RC(use(h));
    if (!bytes) return fail(SILI_EINVAL, "state_size: bad arguments");
    *bytes = ckpt_bytes(h);
    return SILI_OK;
}

int sili_layer_save_state(sili_layer* h, void* buf, int64_t bytes, void* stream) {
    RC(use(h));
    if (!buf) return fail(SILI_EINVAL, "save_state: bad arguments");
    if (h->b4_ntiles > 0) return fail(SILI_EINVAL, "save_state: block4 tiles are not part of the checkpoint image");
    if (bytes < ckpt_bytes(h)) return fail(SILI_EINVAL, "save_state: buffer smaller than sili_layer_state_size");
    cudaStream_t s = pick(h, stream);
    CK(cudaStreamSynchronize(s));
    CK(cudaStreamSynchronize(h->stream));
    RC(flush_stats(h));
    CkptHead hd{};
    hd.magic = kCkptMagic; hd.version = kCkptVersion; hd.rank = (uint32_t)h->rank;
    hd.rows = h->rows; hd.cols = h->cols; hd.seed = h->seed; hd.call = h->call;
    hd.idx_n = h->idx_n; hd.val_n = h->val_n; hd.total_nnz = h->total_nnz;
    hd.max_idx_bytes = h->max_idx_bytes; hd.max_val_bytes = h->max_val_bytes;
    hd.idx_budget = h->idx_budget; hd.val_budget = h->val_budget; hd.n_vs = h->n_vs; hd.n_os = h->n_os;
    for (int i = 0; i < 4; ++i) hd.st[i] = h->st[i];
    hd.st_vmax = h->st_vmax; hd.st_imax = h->st_imax; hd.max_abs_decay = h->max_abs_decay;
    hd.os_trainable = h->os_trainable ? 1 : 0; hd.stochastic = h->stochastic ? 1 : 0;
    uint8_t* out = (uint8_t*)buf;
    // the alignment gaps between sections are zero, so equal states give equal images
    const int64_t total = ckpt_bytes(h);
    if (is_device_ptr(buf)) CK(cudaMemsetAsync(out, 0, (size_t)total, s));
    else std::memset(out, 0, (size_t)total);
    CK(cudaMemcpyAsync(out, &hd, sizeof hd, cudaMemcpyDefault, s));
    size_t off = ckpt_align(sizeof hd);
    for (const auto& sec : ckpt_sections(h)) {
        if (sec.bytes) CK(cudaMemcpyAsync(out + off, sec.dev, sec.bytes, cudaMemcpyDefault, s));
        off += ckpt_align(sec.bytes);
    }
    CK(cudaStreamSynchronize(s));   // hd lives on this frame
    return SILI_OK;
}

int sili_layer_load_state(sili_layer* h, const void* buf, int64_t bytes, void* stream) {
    RC(use(h));
    if (!buf || bytes < (int64_t)sizeof(CkptHead)) return fail(SILI_EINVAL, "load_state: bad arguments");
    if (h->b4_ntiles > 0) return fail(SILI_EINVAL, "load_state: the layer holds block4 tiles");
    cudaStream_t s = pick(h, stream);
    CK(cudaStreamSynchronize(s));
    CK(cudaStreamSynchronize(h->stream));
    CkptHead hd;
    CK(cudaMemcpy(&hd, buf, sizeof hd, cudaMemcpyDefault));
    if (hd.magic != kCkptMagic || hd.version != kCkptVersion)
        return fail(SILI_EINVAL, "load_state: not a checkpoint image of this library version");
    if (hd.rows != h->rows || hd.cols != h->cols)
        return fail(SILI_EINVAL, "load_state: image of a " + std::to_string(hd.rows) + "x" + std::to_string(hd.cols) +
                                     " layer, this layer is " + std::to_string(h->rows) + "x" + std::to_string(h->cols));
    if (hd.rank < 1 || hd.rank > 4 || hd.idx_n < 0 || hd.val_n < 0 || hd.total_nnz < 0)
        return fail(SILI_EINVAL, "load_state: corrupt header");
    RC(sili_layer_set_scale_rank(h, (int)hd.rank));
    const int64_t R = h->rows;
    RC(h->bs.reserve(R + 1)); RC(h->be.reserve(R + 1)); RC(h->es.reserve(R + 1)); RC(h->ee.reserve(R + 1));
    RC(h->idx.reserve(hd.idx_n + 64));
    RC(h->val.reserve(hd.val_n + 64));
    h->idx_n = hd.idx_n; h->val_n = hd.val_n;
    if (bytes < ckpt_bytes(h)) return fail(SILI_EINVAL, "load_state: image shorter than its header says");
    CK(cudaMemsetAsync(h->idx.p + hd.idx_n, 0, 64, s));
    CK(cudaMemsetAsync(h->val.p + hd.val_n, 0, 64, s));
    const uint8_t* in = (const uint8_t*)buf;
    size_t off = ckpt_align(sizeof hd);
    for (const auto& sec : ckpt_sections(h)) {
        if (sec.bytes) CK(cudaMemcpyAsync(sec.dev, in + off, sec.bytes, cudaMemcpyDefault, s));
        off += ckpt_align(sec.bytes);
    }
    CK(cudaStreamSynchronize(s));
    h->seed = hd.seed; h->call = hd.call; h->total_nnz = hd.total_nnz;
    h->max_idx_bytes = hd.max_idx_bytes; h->max_val_bytes = hd.max_val_bytes;
    h->idx_budget = hd.idx_budget; h->val_budget = hd.val_budget; h->n_vs = hd.n_vs; h->n_os = hd.n_os;
    for (int i = 0; i < 4; ++i) h->st[i] = hd.st[i];
    h->st_vmax = hd.st_vmax; h->st_imax = hd.st_imax; h->max_abs_decay = hd.max_abs_decay;
    h->os_trainable = hd.os_trainable != 0;
    h->st_pending = false;
    CK(cudaMemset(h->d_st.p, 0, 2 * sizeof(double)));
    CK(cudaMemset(h->d_stmax.p, 0, sizeof(float)));
    h->aux_dirty = true;      // column index and dead-row set follow the new layout
    h->pack_valid = false;
    h->last_batch = 0;        // the image carries no forward input
    return SILI_OK;
}

int sili_layer_accums(sili_layer* h, float* a, float* g) {
    RC(use(h));
    RC(from_dev(h->in_acc.p, a, (size_t)h->rows * 4, h->stream));
    RC(from_dev(h->grad_acc.p, g, (size_t)h->cols * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

int sili_layer_set_accums(sili_layer* h, const float* a, const float* g) {
    RC(use(h));
    if (a) RC(to_dev(a, h->in_acc.p, (size_t)h->rows * 4, h->stream));
    if (g) RC(to_dev(g, h->grad_acc.p, (size_t)h->cols * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

int sili_layer_out_degree(sili_layer* h, int* out) {
    RC(use(h));
    RC(from_dev(h->out_degree.p, out, (size_t)h->cols * 4, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    return SILI_OK;
}

int sili_layer_stats(sili_layer* h, double* stats) {
    RC(use(h));
    CK(cudaStreamSynchronize(h->stream));
    RC(flush_stats(h));
    stats[0] = h->st[0]; stats[1] = h->st[1]; stats[2] = h->st_vmax;
    stats[3] = h->st[2]; stats[4] = h->st[3]; stats[5] = h->st_imax;
    return SILI_OK;
}

int sili_layer_recompute_stats(sili_layer* h) {
    RC(use(h));
    return recompute_stats(h);
}

int sili_layer_last_sparse_input(sili_layer* h, float* out, int* batch, int* cols) {
    RC(use(h));
    if (batch) *batch = h->sparse_batch;
    if (cols) *cols = (int)h->rows;
    if (out && h->sparse_batch > 0) {
        DBuf<float> t;
        RC(t.reserve((int64_t)h->sparse_batch * h->rows + 1));
        launch_transpose(h->xsT.p, t.p, h->rows, h->sparse_batch, h->stream);
        RC(from_dev(t.p, out, (size_t)h->sparse_batch * h->rows * 4, h->stream));
        CK(cudaStreamSynchronize(h->stream));
    }
    return SILI_OK;
}

int sili_layer_last_input(sili_layer* h, float* out, int* batch, int* cols) {
    RC(use(h));
    if (batch) *batch = h->last_batch;
    if (cols) *cols = (int)h->rows;
    if (out && h->last_batch > 0) {
        DBuf<float> t;
        RC(t.reserve((int64_t)h->last_batch * h->rows + 1));
        launch_transpose(h->xT.p, t.p, h->rows, h->last_batch, h->stream);
        RC(from_dev(t.p, out, (size_t)h->last_batch * h->rows * 4, h->stream));
        CK(cudaStreamSynchronize(h->stream));
    }
    return SILI_OK;
}

// ── module functions ────────────────────────────────────────────────────────
int sili_fp4_quantize(const float* vals, uint8_t* codes, int64_t n, void* stream) {
    if (n < 0) return fail(SILI_EINVAL, "negative size");
    if (n == 0) return SILI_OK;
    cudaStream_t s = (cudaStream_t)stream;
    float* dv = nullptr;
    uint8_t* dc = nullptr;
    CK(cudaMallocAsync((void**)&dv, (size_t)n * 4, s));
    CK(cudaMallocAsync((void**)&dc, (size_t)n, s));
    RC(to_dev(vals, dv, (size_t)n * 4, s));
    launch_fp4_quantize(dv, dc, n, s);
    RC(from_dev(dc, codes, (size_t)n, s));
    cudaFreeAsync(dv, s);
    cudaFreeAsync(dc, s);
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_dense_to_csr(const float* x, int rows, int cols, float thr, int* ptrs, int* idx, float* vals,
                      int64_t* nnz_out, void* stream) {
    if (rows < 0 || cols < 0) return fail(SILI_EINVAL, "negative size");
    cudaStream_t s = (cudaStream_t)stream;
    const size_t n = (size_t)rows * cols;
    float* dx = nullptr;
    int *dcount = nullptr, *dptrs = nullptr;
    CK(cudaMallocAsync((void**)&dx, n * 4 + 4, s));
    CK(cudaMallocAsync((void**)&dcount, (size_t)(rows + 1) * 4, s));
    CK(cudaMallocAsync((void**)&dptrs, (size_t)(rows + 1) * 4, s));
    RC(to_dev(x, dx, n * 4, s));
    CK(cudaMemsetAsync(dcount, 0, (size_t)(rows + 1) * 4, s));
    launch_dense_to_csr_count(dx, rows, cols, thr, dcount, s);
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, dcount, dptrs, rows + 1, s);
    void* tmp = nullptr;
    CK(cudaMallocAsync(&tmp, bytes + 1, s));
    CK(cub::DeviceScan::ExclusiveSum(tmp, bytes, dcount, dptrs, rows + 1, s));
    int total = 0;
    CK(cudaMemcpyAsync(&total, dptrs + rows, 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (nnz_out) *nnz_out = total;
    RC(from_dev(dptrs, ptrs, (size_t)(rows + 1) * 4, s));
    if (idx && vals) {
        int* di = nullptr;
        float* dv = nullptr;
        CK(cudaMallocAsync((void**)&di, (size_t)total * 4 + 4, s));
        CK(cudaMallocAsync((void**)&dv, (size_t)total * 4 + 4, s));
        launch_dense_to_csr_fill(dx, rows, cols, thr, dptrs, di, dv, s);
        RC(from_dev(di, idx, (size_t)total * 4, s));
        RC(from_dev(dv, vals, (size_t)total * 4, s));
        cudaFreeAsync(di, s);
        cudaFreeAsync(dv, s);
    }
    cudaFreeAsync(tmp, s);
    cudaFreeAsync(dx, s);
    cudaFreeAsync(dcount, s);
    cudaFreeAsync(dptrs, s);
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// dense_to_top_k_csr: stable descending radix sort of |v| (ties -> lower flat
// index), first k, re-sorted by flat index, emitted as row-major CSR.
int sili_dense_to_top_k_csr(const float* x, int rows, int cols, int64_t k, int* ptrs, int* idx, float* vals,
                            void* stream) {
    if (rows < 0 || cols < 0 || k < 0) return fail(SILI_EINVAL, "negative size");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t n = (int64_t)rows * cols;
    if (k > n) k = n;
    float* dx = nullptr;
    uint32_t *keys = nullptr, *keys_o = nullptr;
    int *ids = nullptr, *ids_o = nullptr, *fl = nullptr, *fl_o = nullptr, *rc = nullptr, *dptrs = nullptr;
    int* di = nullptr;
    float* dv = nullptr;
    const size_t nn = (size_t)n + 1;
    CK(cudaMallocAsync((void**)&dx, nn * 4, s));
    CK(cudaMallocAsync((void**)&keys, nn * 4, s));
    CK(cudaMallocAsync((void**)&keys_o, nn * 4, s));
    CK(cudaMallocAsync((void**)&ids, nn * 4, s));
    CK(cudaMallocAsync((void**)&ids_o, nn * 4, s));
    CK(cudaMallocAsync((void**)&fl, (size_t)k * 4 + 4, s));
    CK(cudaMallocAsync((void**)&fl_o, (size_t)k * 4 + 4, s));
    CK(cudaMallocAsync((void**)&rc, (size_t)(rows + 1) * 4, s));
    CK(cudaMallocAsync((void**)&dptrs, (size_t)(rows + 1) * 4, s));
    CK(cudaMallocAsync((void**)&di, (size_t)k * 4 + 4, s));
    CK(cudaMallocAsync((void**)&dv, (size_t)k * 4 + 4, s));
    RC(to_dev(x, dx, (size_t)n * 4, s));
    launch_abs_keys(dx, n, keys, ids, s);
    size_t b1 = 0, b2 = 0, b3 = 0;
    cub::DeviceRadixSort::SortPairsDescending(nullptr, b1, keys, keys_o, ids, ids_o, (int)n, 0, 32, s);
    cub::DeviceRadixSort::SortKeys(nullptr, b2, fl, fl_o, (int)k, 0, 32, s);
    cub::DeviceScan::ExclusiveSum(nullptr, b3, rc, dptrs, rows + 1, s);
    const size_t bytes = std::max(b1, std::max(b2, b3)) + 1;
    void* tmp = nullptr;
    CK(cudaMallocAsync(&tmp, bytes, s));
    size_t bb = bytes;
    CK(cub::DeviceRadixSort::SortPairsDescending(tmp, bb, keys, keys_o, ids, ids_o, (int)n, 0, 32, s));
    CK(cudaMemcpyAsync(fl, ids_o, (size_t)k * 4, cudaMemcpyDeviceToDevice, s));
    bb = bytes;
    CK(cub::DeviceRadixSort::SortKeys(tmp, bb, fl, fl_o, (int)k, 0, 32, s));
    CK(cudaMemsetAsync(rc, 0, (size_t)(rows + 1) * 4, s));
    launch_topk_emit(dx, fl_o, k, cols, rc, di, dv, s);
    bb = bytes;
    CK(cub::DeviceScan::ExclusiveSum(tmp, bb, rc, dptrs, rows + 1, s));
    RC(from_dev(dptrs, ptrs, (size_t)(rows + 1) * 4, s));
    RC(from_dev(di, idx, (size_t)k * 4, s));
    RC(from_dev(dv, vals, (size_t)k * 4, s));
    CK(cudaStreamSynchronize(s));
    for (void* p : {(void*)dx, (void*)keys, (void*)keys_o, (void*)ids, (void*)ids_o, (void*)fl, (void*)fl_o,
                    (void*)rc, (void*)dptrs, (void*)di, (void*)dv, tmp})
        cudaFreeAsync(p, s);
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

// ── block4 ──────────────────────────────────────────────────────────────────
int sili_layer_export_nnz(sili_layer* h, int64_t* n) {
    RC(use(h));
    int64_t live = 0;
    if (h->b4_ntiles > 0) {
        live = b4_live_total(h, h->stream);
        if (live < 0) return SILI_ECUDA;
    }
    *n = h->total_nnz + live;
    return SILI_OK;
}

int sili_layer_load_dense_codes(sili_layer* h, const uint8_t* wc, const uint8_t* ic) {
    RC(use(h));
    if (!wc || !ic) return fail(SILI_EINVAL, "load_dense_codes: null codes");
    cudaStream_t s = h->stream;
    const int64_t n = h->rows * h->cols;
    DBuf<uint8_t> dw, di;
    const uint8_t* pw = wc;
    const uint8_t* pi = ic;
    if (!is_device_ptr(wc)) { RC(dw.reserve(n + 1)); RC(to_dev(wc, dw.p, (size_t)n, s)); pw = dw.p; }
    if (!is_device_ptr(ic)) { RC(di.reserve(n + 1)); RC(to_dev(ic, di.p, (size_t)n, s)); pi = di.p; }
    const int64_t BC = (h->cols + 3) / 4;
    RC(b4_init(h, BC, s));
    const int64_t BR = h->b4_BR;
    std::vector<int> nt((size_t)BR + 1, (int)BC);
    if (BR > 0) CK(cudaMemcpyAsync(h->b4_nt.p, nt.data(), (size_t)BR * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemsetAsync(h->b4_used.p, 0, (size_t)(3 * BR + 1) * 8, s));
    launch_b4_load_dense(pw, pi, h->rows, h->cols, h->b4view(), h->b4_used.p, s);
    CK(cudaGetLastError());
    std::vector<int64_t> used((size_t)BR + 1, 0);
    if (BR > 0) CK(cudaMemcpyAsync(used.data(), h->b4_used.p, (size_t)BR * 8, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    // limits block4_load_dense sets (delta_csr_memory.hpp:857-899)
    const int64_t dense = BR * BC * 16;
    h->b4_max_idx = BR * BC * 16;
    h->b4_max_tile = (int64_t)((double)dense * (1.0 + (double)0.2f)) + BR * 16;
    // Each tile insertion finds the row full (block4_row_insert_tile) and
    // grows it by block4_ensure_row_headroom (+5 index bytes, +1 tile byte,
    // +1 slot); the commit then grows the tile bytes to exactly the packed
    // length.  So: index alloc 5*BC, slots BC, tile bytes = used, and
    // block4_expand_headroom(0.2, 16) adds the slack.
    std::vector<int64_t> a((size_t)(3 * BR), 0);
    int64_t total = 0;
    for (int64_t br = 0; br < BR; ++br) {
        const int64_t u = used[(size_t)br];
        a[(size_t)br] = 5 * BC;
        a[(size_t)(BR + br)] = u + (int64_t)((float)u * 0.2f) + 16;
        a[(size_t)(2 * BR + br)] = BC;
        total += a[(size_t)(BR + br)];
    }
    if (total > h->b4_max_tile) return fail(SILI_ENOMEM, "load_dense_codes: block4 tile budget exceeded");
    RC(b4_put_allocs(h, a, s));
    h->b4_ntiles = BR * BC;
    h->b4_dirty = true;
    h->b4_pmap_dirty = h->b4_pmapT_dirty = true;
    // out_degree[c] = n_in for every column (cpu_backend.cpp:916-920)
    std::vector<int> od((size_t)h->cols + 1, (int)h->rows);
    if (h->cols > 0) CK(cudaMemcpyAsync(h->out_degree.p, od.data(), (size_t)h->cols * 4, cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
    return SILI_OK;
}

int sili_layer_b4_expand_headroom(sili_layer* h, float blank_fraction, int64_t min_slack) {
    RC(use(h));
    cudaStream_t s = h->stream;
    const int64_t BR = h->b4_BR;
    if (BR == 0) return SILI_OK;
    std::vector<int64_t> st, a;
    RC(b4_row_stats(h, st, s));
    RC(b4_get_allocs(h, a, s));
    int64_t total = 0;
    for (int64_t br = 0; br < BR; ++br) {
        const int64_t rb = st[(size_t)br];
        a[(size_t)(BR + br)] = rb + (int64_t)((float)rb * blank_fraction) + min_slack;
        total += a[(size_t)(BR + br)];
    }
    if (total > h->b4_max_tile) return fail(SILI_ENOMEM, "expand_block4_headroom: block4 tile budget exceeded");
    return b4_put_allocs(h, a, s);
}

int sili_layer_b4_equalize_row(sili_layer* h, int64_t row) {
    RC(use(h));
    cudaStream_t s = h->stream;
    const int64_t R = h->b4_BR;
    if (R == 0) return SILI_OK;
    row %= R;
    std::vector<int64_t> st, a;
    RC(b4_row_stats(h, st, s));
    RC(b4_get_allocs(h, a, s));
    std::vector<int> nt((size_t)R);
    CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)R * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    int64_t si = 0, stt = 0, se = 0;
    for (int64_t br = 0; br < R; ++br) { si += a[(size_t)br]; stt += a[(size_t)(R + br)]; se += a[(size_t)(2 * R + br)]; }
    // Block4Store::equalize_step (block4.hpp:1208-1221) -> block4_row_shift (:497-609)
    int64_t ti = (si + R - 1) / R, tt = (stt + R - 1) / R, te = (se + R - 1) / R;
    ti = std::max(ti, st[(size_t)(R + row)]);
    tt = std::max(tt, st[(size_t)row]);
    te = std::max(te, (int64_t)nt[(size_t)row]);
    if (row + 1 >= R) return SILI_OK;
    int64_t& ai = a[(size_t)row];
    if (ai != ti) {
        if (ti > ai && si + (ti - ai) > h->b4_max_idx) return fail(SILI_ENOMEM, "equalizer_step: block4 index budget exceeded");
        ai = ti;
    }
    int64_t& at = a[(size_t)(R + row)];
    if (at != tt) {
        if (tt > at && stt + (tt - at) > h->b4_max_tile) {
            RC(b4_put_allocs(h, a, s));
            return fail(SILI_ENOMEM, "equalizer_step: block4 tile budget exceeded");
        }
        at = tt;
    }
    a[(size_t)(2 * R + row)] = te;
    return b4_put_allocs(h, a, s);
}

int sili_layer_b4_set_switch_point(sili_layer* h, uint32_t v) {
    RC(use(h));
    h->b4_switch = v;
    return SILI_OK;
}

int sili_layer_b4_view(sili_layer* h, int64_t* v) {
    RC(use(h));
    cudaStream_t s = h->stream;
    std::vector<int64_t> st, a;
    RC(b4_row_stats(h, st, s));
    RC(b4_get_allocs(h, a, s));
    unsigned long long c[3] = {0, 0, 0};
    CK(cudaMemcpyAsync(c, h->b4_cnt.p, sizeof(c), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    const int64_t R = h->b4_BR;
    int64_t live = 0, used = 0, alloc = 0;
    for (int64_t br = 0; br < R; ++br) { used += st[(size_t)br]; live += st[(size_t)(2 * R + br)]; alloc += a[(size_t)(R + br)]; }
    v[0] = h->b4_ntiles; v[1] = live; v[2] = h->b4_switch; v[3] = (int64_t)c[0];
    v[4] = (int64_t)c[1]; v[5] = (int64_t)c[2]; v[6] = used; v[7] = alloc;
    return SILI_OK;
}

int sili_layer_b4_export(sili_layer* h, int* br, int* bc, uint8_t* slots, uint8_t* sparse) {
    RC(use(h));
    HostTiles T;
    RC(b4_download(h, T, h->stream));
    RC(put_out(T.br.data(), br, T.br.size() * 4));
    RC(put_out(T.bc.data(), bc, T.bc.size() * 4));
    RC(put_out(T.slots.data(), slots, T.slots.size()));
    if (sparse) RC(put_out(T.sparse.data(), sparse, T.sparse.size()));
    return SILI_OK;
}

int sili_layer_b4_rows(sili_layer* h, int64_t* out) {
    RC(use(h));
    cudaStream_t s = h->stream;
    const int64_t R = h->b4_BR;
    std::vector<int64_t> st, a;
    RC(b4_row_stats(h, st, s));
    RC(b4_get_allocs(h, a, s));
    std::vector<int> nt((size_t)R + 1);
    if (R > 0) CK(cudaMemcpyAsync(nt.data(), h->b4_nt.p, (size_t)R * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    for (int64_t br = 0; br < R; ++br) {
        out[6 * br + 0] = a[(size_t)br];
        out[6 * br + 1] = st[(size_t)(R + br)];
        out[6 * br + 2] = a[(size_t)(R + br)];
        out[6 * br + 3] = st[(size_t)br];
        out[6 * br + 4] = a[(size_t)(2 * R + br)];
        out[6 * br + 5] = nt[(size_t)br];
    }
    return SILI_OK;
}

// ── folded stacks ───────────────────────────────────────────────────────────
int sili_fold_sum(const float* raw, int batch, int n_folds, int64_t out_dim, float* y, void* stream) {
    if (batch < 0 || n_folds < 0 || out_dim < 0 || !raw || !y) return fail(SILI_EINVAL, "fold_sum: bad arguments");
    if (!is_device_ptr(raw) || !is_device_ptr(y)) return fail(SILI_EINVAL, "fold_sum: device pointers expected");
    launch_fold_sum(raw, batch, n_folds, out_dim, y, (cudaStream_t)stream);
    CK(cudaGetLastError());
    return SILI_OK;
}
int sili_fold_broadcast(const float* dy, int batch, int64_t out_dim, int64_t j0, int64_t width, int n_folds,
                        float* raw, void* stream) {
    if (batch < 0 || n_folds < 0 || out_dim < 0 || j0 < 0 || width < 0 || j0 + width > out_dim || !dy || !raw)
        return fail(SILI_EINVAL, "fold_broadcast: bad arguments");
    if (!is_device_ptr(dy) || !is_device_ptr(raw)) return fail(SILI_EINVAL, "fold_broadcast: device pointers expected");
    launch_fold_broadcast(dy, batch, out_dim, j0, width, n_folds, raw, (cudaStream_t)stream);
    CK(cudaGetLastError());
    return SILI_OK;
}

}  // extern "C"

// ── forward_dense with no allocation ────────────────────────────────────────
// Some callers cannot call cudaMalloc: a host framework that has already
// reserved the device's memory for its own caching allocator (a cudaMalloc
// from inside it fails or steals from its pool), or a loop that must not
// stall, since cudaMalloc may synchronise the whole device and so wait on
// every other stream.  sili_layer_forward_dense_static serves them: the only
// scratch the forward needs, the transposed input xT [n_in, batch], lives in
// the file-scope array below instead of a per-layer buffer, and x / y must
// already be device memory, so nothing is staged.
//
// The array is one per device and shared by every layer on it: two calls
// whose executions overlap on one device (different streams, or different
// host threads without ordering) race on it and give wrong results.  Calls
// must be ordered, e.g. issued on one stream.
//
// Nothing in the scratch has to start at zero: the transpose writes every
// element xT[0, n_in * batch) and a memset the zero row after it before the
// gather kernel reads any of it.
namespace {
constexpr int64_t kStaticFwdScratch = SILI_STATIC_FWD_MAX_ELEMS;  // floats, 4 MiB
constexpr int kStaticMaxDevices = 64;
static __device__ __align__(256) float g_fwd_xT_scratch[kStaticFwdScratch];
std::mutex g_static_mu;
float* g_static_xT[kStaticMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once
// per device (the first call on a device does this lookup; make that first
// call before any work that must not see a runtime call other than launches).
int static_fwd_scratch(int dev, float** out) {
    if (dev < 0 || dev >= kStaticMaxDevices) return fail(SILI_EINVAL, "forward_dense_static: device id out of range");
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_xT[dev]) {
        float* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_fwd_xT_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(SILI_ECUDA, std::string("forward_dense_static: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_static_xT[dev] = ptr;
    }
    *out = g_static_xT[dev];
    return SILI_OK;
}
}  // namespace

extern "C" int sili_layer_forward_dense_static(sili_layer* h, const float* x, int batch, float* y, void* stream) {
    RC(use(h));
    if (batch < 0 || !x || !y) return fail(SILI_EINVAL, "forward_dense_static: bad arguments");
    const int64_t n_in = h->rows;
    if ((int64_t)batch * (n_in + 1) > kStaticFwdScratch)
        return fail(SILI_EINVAL, "forward_dense_static: batch * (n_inputs + 1) = " +
                                     std::to_string((int64_t)batch * (n_in + 1)) + " exceeds the static scratch of " +
                                     std::to_string(kStaticFwdScratch) + " floats");
    if (!is_device_ptr(x) || !is_device_ptr(y))
        return fail(SILI_EINVAL, "forward_dense_static: x and y must be device pointers");
    if (h->aux_dirty)
        return fail(SILI_EINVAL, "forward_dense_static: the column index is stale (load_weights or a structural "
                                 "change since the last forward_dense); call forward_dense once to rebuild it");
    // block4 tiles add their part through the tile column index, which only
    // forward_dense (re)builds: a stale one would need an allocation
    if (h->b4_ntiles > 0 && h->b4_dirty)
        return fail(SILI_EINVAL, "forward_dense_static: the block4 tile index is stale (tiles changed since the "
                                 "last forward_dense); call forward_dense once to rebuild it");
    float* xT = nullptr;
    RC(static_fwd_scratch(h->dev, &xT));
    cudaStream_t s = pick(h, stream);
    launch_transpose(x, xT, batch, n_in, s);
    CK(cudaMemsetAsync(xT + (int64_t)batch * n_in, 0, (size_t)batch * sizeof(float), s));   // zero row
    launch_forward(h->view(), xT, batch, y, false, s);
    if (h->b4_ntiles > 0) launch_b4_forward(h->view(), h->b4view(), xT, batch, y, s);
    CK(cudaGetLastError());
    return SILI_OK;
}
