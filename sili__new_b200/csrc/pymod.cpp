// sili__new_b200._cuda: the drop-in counterpart of the reference's pybind11
// module sili._cpu (sili/cpu_backend.cpp:1425-3246) for the FP4 delta-CSR
// sparse layer.  Same class names, method names, argument names and defaults;
// every call goes through the C ABI of libsili_b200 (include/sili_b200.h),
// whose compute runs on the GPU.  Host numpy arrays are copied in and fresh
// numpy arrays are returned, as the reference does (cpu_backend.cpp:487-491).
// The *_ptr methods take device pointers (e.g. torch CUDA tensors'
// data_ptr()) and enqueue work on a CUDA stream without copies.
#include <pybind11/numpy.h>
#include <pybind11/stl.h>
#include <pybind11/pybind11.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/sili_b200.h"

namespace py = pybind11;

namespace {

void check(int rc) {
    if (rc == SILI_OK) return;
    const std::string msg = sili_last_error();
    if (rc == SILI_EINVAL) throw py::value_error(msg);
    if (rc == SILI_ENOMEM) {
        PyErr_SetString(PyExc_MemoryError, msg.c_str());
        throw py::error_already_set();
    }
    throw std::runtime_error(msg);
}

using farr = py::array_t<float, py::array::c_style | py::array::forcecast>;
using iarr = py::array_t<int, py::array::c_style | py::array::forcecast>;
using u8arr = py::array_t<uint8_t, py::array::c_style | py::array::forcecast>;
using darr = py::array_t<double, py::array::c_style | py::array::forcecast>;

std::mutex g_live_mu;
std::set<sili_layer*> g_live;
uint64_t g_seed = 0x5EEDu;
bool g_seeded = false;

class Layer;

// Block4View (cpu_backend.cpp:51-98): live counters of the layer's block4 store.
struct Block4View {
    sili_layer* h = nullptr;
    std::vector<int64_t> v() const {
        std::vector<int64_t> out(8, 0);
        check(sili_layer_b4_view(h, out.data()));
        return out;
    }
    std::size_t tiles() const { return (std::size_t)v()[0]; }
    std::size_t synapses() const { return (std::size_t)v()[1]; }
    uint32_t get_switch_point() const { return (uint32_t)v()[2]; }
    void set_switch_point(uint32_t x) { check(sili_layer_b4_set_switch_point(h, x)); }
    uint64_t dropped_growth_events() const { return (uint64_t)v()[3]; }
    uint64_t row_merge_overflow_events() const { return (uint64_t)v()[4]; }
    uint64_t row_merge_overflow_bytes_dropped() const { return (uint64_t)v()[5]; }
    std::size_t used_bytes() const { return (std::size_t)v()[6]; }
    std::size_t alloc_bytes() const { return (std::size_t)v()[7]; }
};

class Layer {
public:
    sili_layer* h = nullptr;
    int n_in, n_out, cpus;
    int synap_row = 0, eq_row = 0, b4_eq_row = 0;

    Layer(int n_inputs, int n_outputs, int max_weights, int num_cpus, bool stochastic, int device)
        : n_in(n_inputs), n_out(n_outputs), cpus(num_cpus) {
        check(sili_layer_create(n_inputs, n_outputs, max_weights, device, stochastic ? 1 : 0, &h));
        std::lock_guard<std::mutex> g(g_live_mu);
        g_live.insert(h);
        if (g_seeded) sili_layer_seed_rng(h, g_seed);
    }
    ~Layer() {
        {
            std::lock_guard<std::mutex> g(g_live_mu);
            g_live.erase(h);
        }
        sili_layer_destroy(h);
    }

    int get_scale_rank() const {
        int r;
        check(sili_layer_get_scale_rank(h, &r));
        return r;
    }
    void set_scale_rank(int r) { check(sili_layer_set_scale_rank(h, r)); }

    py::array_t<float> forward_dense(farr x) {
        auto b = x.request();
        const int batch = b.ndim == 2 ? (int)b.shape[0] : 1;
        const int cols = b.ndim == 2 ? (int)b.shape[1] : (int)b.shape[0];
        if (cols != n_in) throw py::value_error("forward_dense: x has " + std::to_string(cols) + " features, layer has " + std::to_string(n_in));
        py::array_t<float> y({(py::ssize_t)batch, (py::ssize_t)n_out});
        check(sili_layer_forward_dense(h, (const float*)b.ptr, batch, y.mutable_data(), nullptr));
        return y;
    }

    py::array_t<float> backward_dense(farr dy, float lr, bool lr_per_row_nnz, bool damp, float beta2, float eps) {
        auto b = dy.request();
        int batch = 0, cols = 0;
        check(sili_layer_last_input(h, nullptr, &batch, &cols));
        if (batch == 0) throw std::runtime_error("backward_dense: no forward_dense input to differentiate");
        if ((int64_t)b.size != (int64_t)batch * n_out) throw py::value_error("backward_dense: dy shape does not match the last forward");
        warn_lr(lr);
        py::array_t<float> dx({(py::ssize_t)batch, (py::ssize_t)n_in});
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_dense(h, nullptr, (const float*)b.ptr, batch, lr, flags, beta2, eps,
                                        dx.mutable_data(), nullptr));
        return dx;
    }

    // checkpoint image (sili_layer_save_state / sili_layer_load_state)
    int64_t state_size() {
        int64_t n = 0;
        check(sili_layer_state_size(h, &n));
        return n;
    }
    py::array_t<uint8_t> save_state() {
        const int64_t n = state_size();
        py::array_t<uint8_t> out((py::ssize_t)n);
        check(sili_layer_save_state(h, out.mutable_data(), n, nullptr));
        return out;
    }
    void load_state(u8arr image) { check(sili_layer_load_state(h, image.data(), (int64_t)image.size(), nullptr)); }
    void save_state_ptr(uintptr_t buf, int64_t bytes, uintptr_t stream) {
        check(sili_layer_save_state(h, (void*)buf, bytes, (void*)stream));
    }
    void load_state_ptr(uintptr_t buf, int64_t bytes, uintptr_t stream) {
        check(sili_layer_load_state(h, (const void*)buf, bytes, (void*)stream));
    }

    // column shards (sili_layer_set_row_shard): host-array variants
    void set_row_shard(iarr global_row_nnz, int64_t global_n_out) {
        check(sili_layer_set_row_shard(h, global_row_nnz.data(), (int64_t)global_row_nnz.size(), global_n_out));
    }
    int64_t row_part_len(int batch) {
        int64_t n = 0;
        check(sili_layer_row_part_len(h, batch, &n));
        return n;
    }
    py::tuple backward_dense_shard(farr dy, float lr, bool lr_per_row_nnz, bool damp, float beta2, float eps) {
        auto b = dy.request();
        int batch = 0, cols = 0;
        check(sili_layer_last_input(h, nullptr, &batch, &cols));
        if (batch == 0) throw std::runtime_error("backward_dense_shard: no forward_dense input to differentiate");
        if ((int64_t)b.size != (int64_t)batch * n_out) throw py::value_error("backward_dense_shard: dy shape does not match the last forward");
        warn_lr(lr);
        py::array_t<float> dx({(py::ssize_t)batch, (py::ssize_t)n_in});
        py::array_t<double> part((py::ssize_t)row_part_len(batch));
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_dense_shard(h, nullptr, (const float*)b.ptr, batch, lr, flags, beta2, eps,
                                              dx.mutable_data(), part.mutable_data(), nullptr));
        return py::make_tuple(dx, part);
    }
    void apply_row_part(darr part) { check(sili_layer_apply_row_part(h, part.data(), nullptr)); }
    void backward_dense_shard_ptr(uintptr_t dy, int batch, float lr, bool lr_per_row_nnz, bool damp, float beta2,
                                  float eps, uintptr_t dx, uintptr_t part, uintptr_t stream) {
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_dense_shard(h, nullptr, (const float*)dy, batch, lr, flags, beta2, eps, (float*)dx,
                                              (double*)part, (void*)stream));
    }
    void apply_row_part_ptr(uintptr_t part, uintptr_t stream) {
        check(sili_layer_apply_row_part(h, (const double*)part, (void*)stream));
    }

    // cpu_backend.cpp:28-41: one-time warning above the validated lr range.
    static void warn_lr(float lr) {
        static bool warned = false;
        if (!warned && lr > 0.2f) {
            warned = true;
            std::fprintf(stderr,
                "sili: WARNING -- backward() called with learning_rate=%.4f, above the ~0.2 ceiling the "
                "bounded RMSprop synapse policy's max_abs_delta=2.0 was validated for.\n", lr);
        }
    }

    py::array_t<float> forward_sparse(iarr ptrs, iarr idx, farr vals, int batch) {
        auto pi = idx.request();
        if ((int)ptrs.size() < batch + 1) throw py::value_error("forward_sparse: ptrs shorter than batch+1");
        py::array_t<float> y({(py::ssize_t)batch, (py::ssize_t)n_out});
        check(sili_layer_forward_sparse(h, ptrs.data(), idx.data(), vals.data(), (int)pi.size, batch,
                                        y.mutable_data(), nullptr));
        return y;
    }

    py::array_t<float> backward_sparse(py::object xo, iarr dptrs, iarr didx, farr dvals, int batch, float lr,
                                       bool lr_per_row_nnz, bool damp, float beta2, float eps) {
        farr x;
        if (xo.is_none()) {
            // the reference's SISLDOLayer passes last_input, which its module
            // leaves unset after forward_sparse: the dense form of the last
            // forward_sparse input is what that caller means
            int sb = 0, sc = 0;
            check(sili_layer_last_sparse_input(h, nullptr, &sb, &sc));
            if (sb != batch) throw py::value_error("backward_sparse: x is None and the last forward_sparse batch differs");
            x = farr({(py::ssize_t)sb, (py::ssize_t)sc});
            check(sili_layer_last_sparse_input(h, x.mutable_data(), &sb, &sc));
        } else {
            x = xo.cast<farr>();
        }
        if ((int64_t)x.size() != (int64_t)batch * n_in) throw py::value_error("backward_sparse: x must be [batch, n_inputs]");
        py::array_t<float> dx({(py::ssize_t)batch, (py::ssize_t)n_in});
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_sparse(h, x.data(), dptrs.data(), didx.data(), dvals.data(), (int)didx.size(), batch,
                                         lr, flags, beta2, eps, dx.mutable_data(), nullptr));
        return dx;
    }

    // device-pointer entry points (no copies, stream-ordered)
    void forward_dense_ptr(uintptr_t x, int batch, uintptr_t y, uintptr_t stream) {
        check(sili_layer_forward_dense(h, (const float*)x, batch, (float*)y, (void*)stream));
    }
    void backward_dense_ptr(uintptr_t dy, int batch, float lr, bool lr_per_row_nnz, bool damp, float beta2, float eps,
                            uintptr_t dx, uintptr_t stream, uintptr_t x) {
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_dense(h, (const float*)x, (const float*)dy, batch, lr, flags, beta2, eps, (float*)dx,
                                        (void*)stream));
    }
    // device-resident variants of forward_sparse / backward_sparse (pointers
    // to CUDA memory, e.g. torch tensors' data_ptr(); no copies)
    void forward_sparse_ptr(uintptr_t ptrs, uintptr_t idx, uintptr_t vals, int nnz, int batch, uintptr_t y,
                            uintptr_t stream) {
        check(sili_layer_forward_sparse(h, (const int*)ptrs, (const int*)idx, (const float*)vals, nnz, batch,
                                        (float*)y, (void*)stream));
    }
    void backward_sparse_ptr(uintptr_t x, uintptr_t dptrs, uintptr_t didx, uintptr_t dvals, int dnnz, int batch,
                             float lr, bool lr_per_row_nnz, bool damp, float beta2, float eps, uintptr_t dx,
                             uintptr_t stream) {
        unsigned flags = (lr_per_row_nnz ? SILI_LR_PER_ROW_NNZ : 0u) | (damp ? SILI_DAMP_BY_IMPORTANCE : 0u);
        check(sili_layer_backward_sparse(h, (const float*)x, (const int*)dptrs, (const int*)didx, (const float*)dvals,
                                         dnnz, batch, lr, flags, beta2, eps, (float*)dx, (void*)stream));
    }
    void sync() { check(sili_layer_sync(h)); }
    void set_kernel_timing(bool on) { check(sili_layer_set_kernel_timing(h, on ? 1 : 0)); }
    py::tuple kernel_ms() {
        float f = 0.f, b = 0.f;
        check(sili_layer_kernel_ms(h, &f, &b));
        return py::make_tuple(f, b);
    }
    py::dict device_bytes() {
        int64_t fmt = 0, ix = 0, tot = 0;
        check(sili_layer_device_bytes(h, &fmt, &ix, &tot));
        py::dict d;
        d["format"] = fmt;
        d["index"] = ix;
        d["total"] = tot;
        return d;
    }

    void build_probes(int k, bool per_row) { check(sili_layer_build_probes(h, k, per_row ? 1 : 0)); }
    py::tuple probes() {
        int64_t n;
        check(sili_layer_num_probes(h, &n));
        py::array_t<int> r((py::ssize_t)n), c((py::ssize_t)n);
        py::array_t<float> v((py::ssize_t)n);
        if (n) check(sili_layer_get_probes(h, r.mutable_data(), c.mutable_data(), v.mutable_data()));
        return py::make_tuple(r, c, v);
    }
    bool synap_row_step(int row, float cutoff, int max_rw, int max_prune, float eps) {
        uint8_t did = 0;
        check(sili_layer_synap_rows(h, row, 1, cutoff, max_rw, max_prune, eps, &did));
        return did != 0;
    }
    // The top-k growth rule (benchmark configuration 3): exact top-k of |dy^T x| over non-existing
    // synapses, prune as many smallest |w*S|, rebuild (host or device arrays)
    void topk_dyx_step(farr x, farr dy, int64_t k) {
        if (x.ndim() != 2 || dy.ndim() != 2 || x.shape(0) != dy.shape(0) || x.shape(1) != n_in || dy.shape(1) != n_out)
            throw py::value_error("topk_dyx_step: x [B, n_inputs] and dy [B, n_outputs] expected");
        check(sili_layer_topk_dyx_step(h, x.data(), dy.data(), (int)x.shape(0), k, nullptr));
    }
    void topk_dyx_step_ptr(uintptr_t x, uintptr_t dy, int batch, int64_t k, uintptr_t stream) {
        check(sili_layer_topk_dyx_step(h, (const float*)x, (const float*)dy, batch, k, (void*)stream));
    }
    // nrows consecutive synap_row_step calls from row0 (wrapping) in one
    // device sweep; returns each step's result
    py::array_t<uint8_t> synap_rows(int row0, int nrows, float cutoff, int max_rw, int max_prune, float eps) {
        py::array_t<uint8_t> did((py::ssize_t)std::max(nrows, 0));
        check(sili_layer_synap_rows(h, row0, nrows, cutoff, max_rw, max_prune, eps, did.mutable_data()));
        return did;
    }
    bool synap_step(float cutoff, int max_rw, int max_prune, float eps) {
        const int row = synap_row;
        synap_row = n_in > 0 ? (synap_row + 1) % n_in : 0;
        return synap_row_step(row, cutoff, max_rw, max_prune, eps);
    }
    // equalizer_step, cpu_backend.cpp:631-641: scattered rows, then block4 rows,
    // each with its own cursor (advanced only when its step succeeds)
    void equalizer_step() {
        check(sili_layer_equalize_row(h, eq_row));
        eq_row = n_in > 0 ? (eq_row + 1) % n_in : 0;
        const int br = (n_in + 3) / 4;
        check(sili_layer_b4_equalize_row(h, b4_eq_row));
        b4_eq_row = br > 0 ? (b4_eq_row + 1) % br : 0;
    }
    void load_dense_codes(py::array_t<uint8_t, py::array::c_style | py::array::forcecast> w,
                          py::array_t<uint8_t, py::array::c_style | py::array::forcecast> imp) {
        if ((int64_t)w.size() != (int64_t)n_in * n_out || (int64_t)imp.size() != (int64_t)n_in * n_out)
            throw py::value_error("load_dense_codes: codes must be [n_inputs, n_outputs]");
        check(sili_layer_load_dense_codes(h, w.data(), imp.data()));
    }
    void expand_block4_headroom(float bf) { check(sili_layer_b4_expand_headroom(h, bf, 16)); }
    void compact_block4() { check(sili_layer_b4_expand_headroom(h, 0.0f, 0)); }
    py::tuple b4_tiles() {
        int64_t sz[6];
        check(sili_layer_sizes(h, sz));
        const py::ssize_t n = (py::ssize_t)sz[5];
        py::array_t<int> br(n), bc(n);
        py::array_t<uint8_t> sl({n, (py::ssize_t)16}), sp(n);
        check(sili_layer_b4_export(h, br.mutable_data(), bc.mutable_data(), sl.mutable_data(), sp.mutable_data()));
        return py::make_tuple(br, bc, sl, sp);
    }
    py::array_t<int64_t> b4_rows() {
        const py::ssize_t R = (n_in + 3) / 4;
        py::array_t<int64_t> out({R, (py::ssize_t)6});
        check(sili_layer_b4_rows(h, out.mutable_data()));
        return out;
    }
    py::array_t<int64_t> b4_view() {
        py::array_t<int64_t> out((py::ssize_t)8);
        check(sili_layer_b4_view(h, out.mutable_data()));
        return out;
    }
    int64_t combined_nnz() const {
        int64_t n = 0;
        check(sili_layer_export_nnz(h, &n));
        return n;
    }
    void equalize_to_capacity(int te, int tb) { check(sili_layer_equalize_to_capacity(h, te, tb)); }
    void compact() { check(sili_layer_compact(h)); }
    void expand_headroom(float bf) { check(sili_layer_expand_headroom(h, bf)); }
    void expand_headroom_to(int m, float bf) { check(sili_layer_expand_headroom_to(h, m, bf)); }

    float gs(int kind, int i, int k) const {
        float v;
        check(sili_layer_get_scale(h, kind, i, k, &v));
        return v;
    }
    void ss(int kind, int i, int k, float v) { check(sili_layer_set_scale(h, kind, i, k, v)); }
    // get_scale, delta_csr_types.hpp:1235-1240
    float get_scale(int row, int col) const {
        float s = 0.0f;
        const int rank = get_scale_rank();
        for (int k = 0; k < rank; ++k) s = std::fma(gs(SILI_SCALE_VALUE, row, k), gs(SILI_SCALE_OUTPUT, col, k), s);
        return s;
    }
    void rescale_importance(float v) { for (int r = 0; r < n_in; ++r) check(sili_layer_rescale_row(h, SILI_SCALE_IMPORTANCE, r, v)); }
    void rescale_value(float v) { for (int r = 0; r < n_in; ++r) check(sili_layer_rescale_row(h, SILI_SCALE_VALUE, r, v)); }

    std::vector<double> stats() const {
        std::vector<double> s(6);
        check(sili_layer_stats(h, s.data()));
        return s;
    }
    int64_t scattered_nnz() const {
        int64_t s[6];
        check(sili_layer_sizes(h, s));
        return s[2];
    }
    // Hoyer's measure from running stats (delta_csr_types.hpp:1371-1378)
    float hoyer(double l1, double l2_sq) const {
        const int64_t n = scattered_nnz();
        if (n <= 1) return 0.0f;
        const double l2 = std::sqrt(l2_sq);
        if (l2 <= 0.0) return 1.0f;
        const double sn = std::sqrt((double)n);
        return (float)((sn - l1 / l2) / (sn - 1.0));
    }

    py::tuple export_csr() {
        const py::ssize_t n = (py::ssize_t)combined_nnz();
        py::array_t<int> p((py::ssize_t)n_in + 1), i(n);
        py::array_t<float> w(n), m(n);
        check(sili_layer_export(h, p.mutable_data(), i.mutable_data(), w.mutable_data(), m.mutable_data()));
        return py::make_tuple(p, i, w, m);
    }
    py::tuple accums() {
        py::array_t<float> a((py::ssize_t)n_in), g((py::ssize_t)n_out);
        check(sili_layer_accums(h, a.mutable_data(), g.mutable_data()));
        return py::make_tuple(a, g);
    }
    void set_accums(farr a, farr g) { check(sili_layer_set_accums(h, a.data(), g.data())); }
    py::dict raw_state() {
        int64_t s[6];
        check(sili_layer_sizes(h, s));
        py::array_t<int64_t> bs((py::ssize_t)n_in + 1), be((py::ssize_t)n_in), es((py::ssize_t)n_in + 1), ee((py::ssize_t)n_in);
        py::array_t<uint8_t> ib((py::ssize_t)s[3]), vb((py::ssize_t)s[4]);
        check(sili_layer_raw(h, bs.mutable_data(), be.mutable_data(), es.mutable_data(), ee.mutable_data(),
                             ib.mutable_data(), vb.mutable_data()));
        py::dict d;
        d["rows"] = n_in; d["cols"] = n_out; d["nnz"] = s[2];
        d["byte_start"] = bs; d["byte_end"] = be; d["elem_start"] = es; d["elem_end"] = ee;
        d["indices_buf"] = ib; d["values"] = vb; d["tiles"] = s[5];
        return d;
    }
    py::array_t<float> scales(int kind) {
        const int rank = get_scale_rank();
        const int64_t n = (kind == SILI_SCALE_VALUE || kind == SILI_SCALE_VALUE_IMPORTANCE || kind == SILI_SCALE_VALUE_MOMENTUM)
                              ? (int64_t)n_in * rank
                              : (kind == SILI_SCALE_IMPORTANCE ? n_in : (kind == SILI_SCALE_OUTPUT_IMPORTANCE ? n_out : (int64_t)n_out * rank));
        py::array_t<float> out((py::ssize_t)n);
        check(sili_layer_get_scales(h, kind, out.mutable_data(), (int)n));
        return out;
    }
    py::array_t<uint32_t> steps(int which) {
        const int64_t n = (int64_t)(which == 0 ? n_in : n_out) * get_scale_rank();
        py::array_t<uint32_t> out((py::ssize_t)n);
        check(sili_layer_get_steps(h, which, out.mutable_data(), (int)n));
        return out;
    }
    void set_value_bytes(u8arr b) { check(sili_layer_set_value_bytes(h, b.data(), (int64_t)b.size())); }
    py::object last_input() {
        int batch = 0, cols = 0;
        check(sili_layer_last_input(h, nullptr, &batch, &cols));
        if (batch == 0) return py::none();
        py::array_t<float> x({(py::ssize_t)batch, (py::ssize_t)cols});
        check(sili_layer_last_input(h, x.mutable_data(), &batch, &cols));
        return x;
    }
};

// STOCH: stochastic rounding (SparseLinearLayer) or nearest (…Deterministic);
// POLICY: the scale policy (SILI_SCALE_POLICY_*, …NoScale…)
template <bool STOCH, int POLICY = SILI_SCALE_POLICY_RMSPROP>
struct LayerT : Layer {
    LayerT(int a, int b, int c, int d, int dev) : Layer(a, b, c, d, STOCH, dev) {
        if (POLICY != SILI_SCALE_POLICY_RMSPROP) check(sili_layer_set_scale_policy(h, POLICY));
    }
};

template <typename T>
void bind_layer(py::module_& m, const char* name) {
    py::class_<T>(m, name)
        .def(py::init<int, int, int, int, int>(), py::arg("n_inputs"), py::arg("n_outputs"), py::arg("max_weights"),
             py::arg("num_cpus") = 4, py::arg("device") = 0)
        .def("get_scale_rank", &T::get_scale_rank)
        .def("set_scale_rank", &T::set_scale_rank, py::arg("rank"))
        .def("forward_dense", &T::forward_dense, py::arg("x"))
        .def("backward_dense", &T::backward_dense, py::arg("dy"), py::arg("learning_rate"),
             py::arg("lr_per_row_nnz") = false, py::arg("damp_by_importance") = true, py::arg("beta2") = 0.999f,
             py::arg("eps") = 1e-8f)
        .def("forward_sparse", &T::forward_sparse, py::arg("ptrs"), py::arg("indices"), py::arg("values"), py::arg("batch"))
        .def("forward_sparse_ptr", &T::forward_sparse_ptr, py::arg("ptrs"), py::arg("indices"), py::arg("values"),
             py::arg("nnz"), py::arg("batch"), py::arg("y"), py::arg("stream") = 0)
        .def("backward_sparse_ptr", &T::backward_sparse_ptr, py::arg("x"), py::arg("dy_ptrs"), py::arg("dy_indices"),
             py::arg("dy_values"), py::arg("dnnz"), py::arg("batch"), py::arg("learning_rate") = 0.01f,
             py::arg("lr_per_row_nnz") = false, py::arg("damp_by_importance") = true, py::arg("beta2") = 0.999f,
             py::arg("eps") = 1e-8f, py::arg("dx") = 0, py::arg("stream") = 0)
        .def("backward_sparse", &T::backward_sparse, py::arg("x"), py::arg("dy_ptrs"), py::arg("dy_indices"),
             py::arg("dy_values"), py::arg("batch"), py::arg("learning_rate") = 0.01f, py::arg("lr_per_row_nnz") = false,
             py::arg("damp_by_importance") = true, py::arg("beta2") = 0.999f, py::arg("eps") = 1e-8f)
        .def("forward_dense_ptr", &T::forward_dense_ptr, py::arg("x_ptr"), py::arg("batch"), py::arg("y_ptr"),
             py::arg("stream") = 0)
        .def("backward_dense_ptr", &T::backward_dense_ptr, py::arg("dy_ptr"), py::arg("batch"), py::arg("learning_rate"),
             py::arg("lr_per_row_nnz") = false, py::arg("damp_by_importance") = true, py::arg("beta2") = 0.999f,
             py::arg("eps") = 1e-8f, py::arg("dx_ptr") = 0, py::arg("stream") = 0, py::arg("x_ptr") = 0)
        .def("state_size", &T::state_size)
        .def("save_state", &T::save_state)
        .def("load_state", &T::load_state, py::arg("image"))
        .def("save_state_ptr", &T::save_state_ptr, py::arg("buf"), py::arg("bytes"), py::arg("stream") = 0)
        .def("load_state_ptr", &T::load_state_ptr, py::arg("buf"), py::arg("bytes"), py::arg("stream") = 0)
        .def("set_row_shard", &T::set_row_shard, py::arg("global_row_nnz"), py::arg("global_n_outputs"))
        .def("row_part_len", &T::row_part_len, py::arg("batch"))
        .def("backward_dense_shard", &T::backward_dense_shard, py::arg("dy"), py::arg("learning_rate"),
             py::arg("lr_per_row_nnz") = false, py::arg("damp_by_importance") = true, py::arg("beta2") = 0.999f,
             py::arg("eps") = 1e-8f)
        .def("apply_row_part", &T::apply_row_part, py::arg("part"))
        .def("backward_dense_shard_ptr", &T::backward_dense_shard_ptr, py::arg("dy_ptr"), py::arg("batch"),
             py::arg("learning_rate"), py::arg("lr_per_row_nnz") = false, py::arg("damp_by_importance") = true,
             py::arg("beta2") = 0.999f, py::arg("eps") = 1e-8f, py::arg("dx_ptr") = 0, py::arg("part_ptr") = 0,
             py::arg("stream") = 0)
        .def("apply_row_part_ptr", &T::apply_row_part_ptr, py::arg("part_ptr"), py::arg("stream") = 0)
        .def("sync", &T::sync)
        .def("set_kernel_timing", &T::set_kernel_timing, py::arg("enable"))
        .def("kernel_ms", &T::kernel_ms)
        .def("device_bytes", &T::device_bytes)
        .def("build_probes", &T::build_probes, py::arg("k"), py::arg("per_row") = false)
        .def("probes", &T::probes)
        .def("synap_row_step", &T::synap_row_step, py::arg("current_row"), py::arg("importance_cutoff"),
             py::arg("max_row_weights"), py::arg("max_prune_per_step") = 8, py::arg("importance_eps") = 1e-3f)
        .def("topk_dyx_step", &T::topk_dyx_step, py::arg("x"), py::arg("dy"), py::arg("k"))
        .def("topk_dyx_step_ptr", &T::topk_dyx_step_ptr, py::arg("x"), py::arg("dy"), py::arg("batch"), py::arg("k"),
             py::arg("stream") = 0)
        .def("synap_rows", &T::synap_rows, py::arg("row0"), py::arg("nrows"), py::arg("importance_cutoff"),
             py::arg("max_row_weights"), py::arg("max_prune_per_step") = 8, py::arg("importance_eps") = 1e-3f)
        .def("synap_step", &T::synap_step, py::arg("importance_cutoff"), py::arg("max_row_weights"),
             py::arg("max_prune_per_step") = 8, py::arg("importance_eps") = 1e-3f)
        .def("equalizer_step", &T::equalizer_step)
        .def("equalize_to_capacity", &T::equalize_to_capacity, py::arg("target_elems_per_row"),
             py::arg("target_bytes_per_row") = 0)
        .def("compact", &T::compact)
        .def("expand_headroom", &T::expand_headroom, py::arg("blank_fraction") = 0.2f)
        .def("expand_headroom_to", &T::expand_headroom_to, py::arg("min_nnz_per_row"), py::arg("blank_fraction") = 0.2f)
        .def("get_importance_scale", [](T& s, int r) { return s.gs(SILI_SCALE_IMPORTANCE, r, 0); }, py::arg("row"))
        .def("get_value_scale", [](T& s, int r) { return s.gs(SILI_SCALE_VALUE, r, 0); }, py::arg("row"))
        .def("get_value_scale_k", [](T& s, int r, int k) { return s.gs(SILI_SCALE_VALUE, r, k); }, py::arg("row"), py::arg("k"))
        .def("get_output_scale_k", [](T& s, int c, int k) { return s.gs(SILI_SCALE_OUTPUT, c, k); }, py::arg("col"), py::arg("k"))
        .def("set_value_scale_raw_k", [](T& s, int r, int k, float v) { s.ss(SILI_SCALE_VALUE, r, k, v); },
             py::arg("row"), py::arg("k"), py::arg("v"))
        .def("set_output_scale_raw_k", [](T& s, int c, int k, float v) { s.ss(SILI_SCALE_OUTPUT, c, k, v); },
             py::arg("col"), py::arg("k"), py::arg("v"))
        .def("get_scale", &T::get_scale, py::arg("row"), py::arg("col"))
        .def("set_value_scale_raw", [](T& s, int r, float v) { s.ss(SILI_SCALE_VALUE, r, 0, v); }, py::arg("row"), py::arg("scale"))
        .def("set_block4_tensor_cores", [](T& s, bool enable) {
            check(sili_layer_set_b4_tensor_cores(s.h, enable ? 1 : 0));
        }, py::arg("enable"))
        .def("set_scales", [](T& s, int kind, farr v) {
            check(sili_layer_set_scales(s.h, kind, v.data(), (int)v.size()));
        }, py::arg("kind"), py::arg("values"))
        .def("set_scales_ptr", [](T& s, int kind, uintptr_t v, int n) {
            check(sili_layer_set_scales(s.h, kind, (const float*)v, n));
        }, py::arg("kind"), py::arg("values_ptr"), py::arg("n"))
        .def("set_importance_scale_raw", [](T& s, int r, float v) { s.ss(SILI_SCALE_IMPORTANCE, r, 0, v); },
             py::arg("row"), py::arg("scale"))
        .def("get_output_scale", [](T& s, int c) { return s.gs(SILI_SCALE_OUTPUT, c, 0); }, py::arg("col"))
        .def("set_output_scale_raw", [](T& s, int c, float v) { s.ss(SILI_SCALE_OUTPUT, c, 0, v); }, py::arg("col"), py::arg("scale"))
        .def("get_value_scale_importance", [](T& s, int r) { return s.gs(SILI_SCALE_VALUE_IMPORTANCE, r, 0); }, py::arg("row"))
        .def("get_output_scale_importance", [](T& s, int c) { return s.gs(SILI_SCALE_OUTPUT_SCALE_IMPORTANCE, c, 0); }, py::arg("col"))
        .def("get_output_importance_scale", [](T& s, int c) { return s.gs(SILI_SCALE_OUTPUT_IMPORTANCE, c, 0); }, py::arg("col"))
        .def("set_output_importance_scale_raw", [](T& s, int c, float v) { s.ss(SILI_SCALE_OUTPUT_IMPORTANCE, c, 0, v); },
             py::arg("col"), py::arg("scale"))
        .def("rescale_importance_row", [](T& s, int r, float v) { check(sili_layer_rescale_row(s.h, SILI_SCALE_IMPORTANCE, r, v)); },
             py::arg("row"), py::arg("new_scale"))
        .def("rescale_value_row", [](T& s, int r, float v) { check(sili_layer_rescale_row(s.h, SILI_SCALE_VALUE, r, v)); },
             py::arg("row"), py::arg("new_scale"))
        .def("rescale_importance", &T::rescale_importance, py::arg("new_scale"))
        .def("rescale_value", &T::rescale_value, py::arg("new_scale"))
        .def_property_readonly("value_l1", [](T& s) { return (float)s.stats()[0]; })
        .def_property_readonly("value_l2_sq", [](T& s) { return (float)s.stats()[1]; })
        .def_property_readonly("value_max_abs", [](T& s) { return (float)s.stats()[2]; })
        .def_property_readonly("importance_l1", [](T& s) { return (float)s.stats()[3]; })
        .def_property_readonly("importance_l2_sq", [](T& s) { return (float)s.stats()[4]; })
        .def_property_readonly("importance_max_abs", [](T& s) { return (float)s.stats()[5]; })
        .def("hoyer_value", [](T& s) { auto st = s.stats(); return s.hoyer(st[0], st[1]); })
        .def("hoyer_importance", [](T& s) { auto st = s.stats(); return s.hoyer(st[3], st[4]); })
        .def("recompute_stats", [](T& s) { check(sili_layer_recompute_stats(s.h)); })
        .def("zero_accum", [](T& s) { check(sili_layer_zero_accum(s.h)); })
        .def_property_readonly("neuron_input_accum", [](T& s) { py::tuple t = s.accums(); return py::object(t[0]); })
        .def_property_readonly("neuron_grad_accum", [](T& s) { py::tuple t = s.accums(); return py::object(t[1]); })
        .def("accums", &T::accums)
        .def("set_accums", &T::set_accums, py::arg("input_accum"), py::arg("grad_accum"))
        // (the element is taken as an owning object while the tuple is alive:
        // an accessor returned past the tuple's lifetime would dangle)
        .def_property_readonly("weights_vals", [](T& s) { py::tuple t = s.export_csr(); return py::object(t[2]); })
        .def_property_readonly("importance", [](T& s) { py::tuple t = s.export_csr(); return py::object(t[3]); })
        .def_property_readonly("indices", [](T& s) { py::tuple t = s.export_csr(); return py::object(t[1]); })
        .def_property_readonly("ptrs", [](T& s) { py::tuple t = s.export_csr(); return py::object(t[0]); })
        .def("export", &T::export_csr)
        .def("raw_state", &T::raw_state)
        .def("scales", &T::scales, py::arg("kind"))
        .def("steps", &T::steps, py::arg("which"))
        .def("set_value_bytes", &T::set_value_bytes, py::arg("values"))
        .def("load_weights", [](T& s, iarr p, iarr i, farr w) {
            if ((int)p.size() != s.n_in + 1) throw py::value_error("load_weights: ptrs must have n_inputs+1 entries");
            check(sili_layer_load_weights(s.h, p.data(), i.data(), w.data(), (int)i.size()));
        }, py::arg("ptrs"), py::arg("indices"), py::arg("weights"))
        .def("load_weights_ptr", [](T& s, uintptr_t p, uintptr_t i, uintptr_t w, int nnz) {
            check(sili_layer_load_weights(s.h, (const int*)p, (const int*)i, (const float*)w, nnz));
        }, py::arg("ptrs"), py::arg("indices"), py::arg("weights"), py::arg("nnz"))
        .def_property_readonly("out_degree", [](T& s) {
            py::array_t<int> o((py::ssize_t)s.n_out);
            check(sili_layer_out_degree(s.h, o.mutable_data()));
            return o;
        })
        .def_property_readonly("num_cpus", [](T& s) { return s.cpus; })
        .def_property_readonly("n_inputs", [](T& s) { return s.n_in; })
        .def_property_readonly("n_outputs", [](T& s) { return s.n_out; })
        .def_property_readonly("nnz", [](T& s) { return (int)s.combined_nnz(); })
        .def_property_readonly("block4", py::cpp_function([](T& s) { Block4View v; v.h = s.h; return v; },
                                                          py::keep_alive<0, 1>()))
        .def("load_dense_codes", &T::load_dense_codes, py::arg("weight_codes"), py::arg("importance_codes"))
        .def("expand_block4_headroom", &T::expand_block4_headroom, py::arg("blank_fraction") = 0.2f)
        .def("compact_block4", &T::compact_block4)
        .def("b4_tiles", &T::b4_tiles)
        .def("b4_rows", &T::b4_rows)
        .def("b4_view", &T::b4_view)
        .def("set_switch_point", [](T& s, uint32_t v) { check(sili_layer_b4_set_switch_point(s.h, v)); })
        .def_property_readonly("last_input", &T::last_input);
}

}  // namespace

PYBIND11_MODULE(_cuda, m) {
    m.doc() = "B200 (sm_100a) FP4 delta-CSR sparse layer: drop-in for sili._cpu's SparseLinearLayer";
    py::class_<Block4View>(m, "Block4View")
        .def_property_readonly("tiles", &Block4View::tiles)
        .def_property_readonly("synapses", &Block4View::synapses)
        .def_property("switch_point", &Block4View::get_switch_point, &Block4View::set_switch_point)
        .def_property_readonly("dropped_growth_events", &Block4View::dropped_growth_events)
        .def_property_readonly("row_merge_overflow_events", &Block4View::row_merge_overflow_events)
        .def_property_readonly("row_merge_overflow_bytes_dropped", &Block4View::row_merge_overflow_bytes_dropped)
        .def_property_readonly("used_bytes", &Block4View::used_bytes)
        .def_property_readonly("alloc_bytes", &Block4View::alloc_bytes);
    bind_layer<LayerT<true>>(m, "SparseLinearLayer");
    bind_layer<LayerT<false>>(m, "SparseLinearLayerDeterministic");
    bind_layer<LayerT<true, SILI_SCALE_POLICY_NONE>>(m, "SparseLinearLayerNoScale");
    bind_layer<LayerT<false, SILI_SCALE_POLICY_NONE>>(m, "SparseLinearLayerNoScaleDeterministic");
    bind_layer<LayerT<true, SILI_SCALE_POLICY_RESYNC>>(m, "SparseLinearLayerResync");
    bind_layer<LayerT<false, SILI_SCALE_POLICY_RESYNC>>(m, "SparseLinearLayerResyncDeterministic");
    m.attr("SCALE_VALUE") = SILI_SCALE_VALUE;
    m.attr("SCALE_OUTPUT") = SILI_SCALE_OUTPUT;
    m.attr("SCALE_IMPORTANCE") = SILI_SCALE_IMPORTANCE;
    m.attr("SCALE_OUTPUT_IMPORTANCE") = SILI_SCALE_OUTPUT_IMPORTANCE;
    m.attr("SCALE_VALUE_IMPORTANCE") = SILI_SCALE_VALUE_IMPORTANCE;
    m.attr("SCALE_OUTPUT_SCALE_IMPORTANCE") = SILI_SCALE_OUTPUT_SCALE_IMPORTANCE;
    m.attr("SCALE_VALUE_MOMENTUM") = SILI_SCALE_VALUE_MOMENTUM;

    m.def("device_count", []() { int n = 0; sili_device_count(&n); return n; });
    m.def("fold_sum_ptr", [](uintptr_t raw, int batch, int n_folds, int64_t out_dim, uintptr_t y, uintptr_t stream) {
        check(sili_fold_sum((const float*)raw, batch, n_folds, out_dim, (float*)y, (void*)stream));
    }, py::arg("raw"), py::arg("batch"), py::arg("n_folds"), py::arg("out_dim"), py::arg("y"), py::arg("stream") = 0);
    m.def("fold_broadcast_ptr", [](uintptr_t dy, int batch, int64_t out_dim, int64_t j0, int64_t width, int n_folds,
                                   uintptr_t raw, uintptr_t stream) {
        check(sili_fold_broadcast((const float*)dy, batch, out_dim, j0, width, n_folds, (float*)raw, (void*)stream));
    }, py::arg("dy"), py::arg("batch"), py::arg("out_dim"), py::arg("j0"), py::arg("width"), py::arg("n_folds"),
       py::arg("raw"), py::arg("stream") = 0);
    m.def("kernel_launches", []() { int64_t n = 0; sili_kernel_launches(&n); return n; });
    m.def("csr_union", [](iarr pa, iarr ia, farr va, iarr pb, iarr ib, farr vb, int n_rows, std::string prefer,
                          int num_cpus) {
        (void)num_cpus;
        const int code = prefer == "a" ? 0 : prefer == "b" ? 1 : prefer == "sum" ? 2 : -1;
        if (code < 0) throw py::value_error("prefer must be 'a', 'b', or 'sum'");
        if (pa.size() < (py::ssize_t)n_rows + 1 || pb.size() < (py::ssize_t)n_rows + 1)
            throw py::value_error("csr_union: ptrs shorter than n_rows + 1");
        const int na = pa.data()[n_rows], nb = pb.data()[n_rows];
        if (ia.size() < na || va.size() < na || ib.size() < nb || vb.size() < nb)
            throw py::value_error("csr_union: idx/vals shorter than ptrs[n_rows]");
        py::array_t<int> p((py::ssize_t)n_rows + 1);
        int64_t n = 0;
        check(sili_csr_union(pa.data(), ia.data(), va.data(), pb.data(), ib.data(), vb.data(), n_rows, code,
                             p.mutable_data(), nullptr, nullptr, &n, nullptr));
        py::array_t<int> i((py::ssize_t)n);
        py::array_t<float> v((py::ssize_t)n);
        check(sili_csr_union(pa.data(), ia.data(), va.data(), pb.data(), ib.data(), vb.data(), n_rows, code,
                             p.mutable_data(), i.mutable_data(), v.mutable_data(), &n, nullptr));
        return py::make_tuple(p, i, v);
    }, py::arg("ptrs_a"), py::arg("idx_a"), py::arg("vals_a"), py::arg("ptrs_b"), py::arg("idx_b"), py::arg("vals_b"),
       py::arg("n_rows"), py::arg("prefer") = "a", py::arg("num_cpus") = 4);
    // FoldedLayer.forward over its suffix layers in one call
    auto handles = [](py::list layers) {
        std::vector<sili_layer*> hs;
        for (auto o : layers) {
            if (py::isinstance<LayerT<true>>(o)) hs.push_back(o.cast<LayerT<true>&>().h);
            else if (py::isinstance<LayerT<false>>(o)) hs.push_back(o.cast<LayerT<false>&>().h);
            else if (py::isinstance<LayerT<true, SILI_SCALE_POLICY_NONE>>(o))
                hs.push_back(o.cast<LayerT<true, SILI_SCALE_POLICY_NONE>&>().h);
            else if (py::isinstance<LayerT<false, SILI_SCALE_POLICY_NONE>>(o))
                hs.push_back(o.cast<LayerT<false, SILI_SCALE_POLICY_NONE>&>().h);
            else if (py::isinstance<LayerT<true, SILI_SCALE_POLICY_RESYNC>>(o))
                hs.push_back(o.cast<LayerT<true, SILI_SCALE_POLICY_RESYNC>&>().h);
            else if (py::isinstance<LayerT<false, SILI_SCALE_POLICY_RESYNC>>(o))
                hs.push_back(o.cast<LayerT<false, SILI_SCALE_POLICY_RESYNC>&>().h);
            else throw py::type_error("folded_forward: layers must be this module's SparseLinearLayer objects");
        }
        if (hs.empty()) throw py::value_error("folded_forward: no layers");
        return hs;
    };
    m.def("folded_forward", [handles](py::list layers, farr x, int n_folds, int64_t out_dim, bool fold_sum) {
        auto hs = handles(layers);
        auto b = x.request();
        const int batch = b.ndim == 2 ? (int)b.shape[0] : 1;
        int64_t n_in = 0;
        {
            int64_t sz[6];
            check(sili_layer_sizes(hs[0], sz));
            n_in = sz[0];
        }
        if ((int64_t)b.size != (int64_t)batch * n_in) throw py::value_error("folded_forward: x must be [batch, n_inputs]");
        const int64_t w = fold_sum ? out_dim : (int64_t)n_folds * out_dim;
        py::array_t<float> y({(py::ssize_t)batch, (py::ssize_t)w});
        check(sili_folded_forward(hs.data(), (int)hs.size(), x.data(), batch, n_folds, out_dim, fold_sum ? 1 : 0,
                                  y.mutable_data(), nullptr));
        return y;
    }, py::arg("layers"), py::arg("x"), py::arg("n_folds"), py::arg("out_dim"), py::arg("fold_sum") = true);
    m.def("folded_forward_ptr", [handles](py::list layers, uintptr_t x, int batch, int n_folds, int64_t out_dim,
                                          bool fold_sum, uintptr_t y, uintptr_t stream) {
        auto hs = handles(layers);
        check(sili_folded_forward(hs.data(), (int)hs.size(), (const float*)x, batch, n_folds, out_dim,
                                  fold_sum ? 1 : 0, (float*)y, (void*)stream));
    }, py::arg("layers"), py::arg("x"), py::arg("batch"), py::arg("n_folds"), py::arg("out_dim"), py::arg("fold_sum"),
       py::arg("y"), py::arg("stream") = 0);
    // conversion-time CSR operations on device arrays (sili__new_b200.convert)
    m.def("prune_to_csr_ptr", [](uintptr_t w, int64_t rows, int64_t cols, float min_abs, uintptr_t ptrs, uintptr_t idx,
                                 uintptr_t vals, uintptr_t stream) {
        int64_t n = 0;
        check(sili_prune_to_csr((const float*)w, rows, cols, min_abs, (int*)ptrs, (int*)idx, (float*)vals, &n,
                                (void*)stream));
        return n;
    }, py::arg("w"), py::arg("rows"), py::arg("cols"), py::arg("min_abs"), py::arg("ptrs"), py::arg("idx") = 0,
       py::arg("vals") = 0, py::arg("stream") = 0);
    m.def("csr_transpose_ptr", [](uintptr_t p, uintptr_t i, uintptr_t v, int n_rows, int n_cols, uintptr_t op,
                                  uintptr_t oi, uintptr_t ov, uintptr_t stream) {
        check(sili_csr_transpose((const int*)p, (const int*)i, (const float*)v, n_rows, n_cols, (int*)op, (int*)oi,
                                 (float*)ov, (void*)stream));
    });
    m.def("csr_stack_vertical_ptr", [](std::vector<uintptr_t> p, std::vector<uintptr_t> i, std::vector<uintptr_t> v,
                                       std::vector<int> rows, uintptr_t op, uintptr_t oi, uintptr_t ov, uintptr_t stream) {
        if (p.size() != i.size() || p.size() != v.size() || p.size() != rows.size())
            throw py::value_error("csr_stack_vertical: one ptrs / idx / vals / rows entry per part");
        std::vector<const int*> pp(p.size()), ii(p.size());
        std::vector<const float*> vv(p.size());
        for (size_t k = 0; k < p.size(); ++k) { pp[k] = (const int*)p[k]; ii[k] = (const int*)i[k]; vv[k] = (const float*)v[k]; }
        check(sili_csr_stack_vertical((int)p.size(), pp.data(), ii.data(), vv.data(), rows.data(), (int*)op, (int*)oi,
                                      (float*)ov, (void*)stream));
    });
    m.def("fit_rank1_envelope_ptr", [](uintptr_t p, uintptr_t i, uintptr_t v, int n_rows, int n_cols, int n_iters,
                                       uintptr_t rs, uintptr_t cs, uintptr_t stream) {
        check(sili_fit_rank1_envelope((const int*)p, (const int*)i, (const float*)v, n_rows, n_cols, n_iters,
                                      (float*)rs, (float*)cs, (void*)stream));
    });
    m.def("fp4_row_rescale_ptr", [](uintptr_t p, uintptr_t i, uintptr_t v, int n_rows, int mode, uintptr_t cs,
                                    uintptr_t rs, uintptr_t stream) {
        check(sili_fp4_row_rescale((const int*)p, (const int*)i, (float*)v, n_rows, mode, (const float*)cs,
                                   (float*)rs, (void*)stream));
    });
    // attention.hpp's kernels with the reference's signatures (cpu_backend.cpp:3384-3468)
    auto td = [](const farr& a, const char* who) {
        auto b = a.request();
        if (b.ndim != 2) throw py::value_error(std::string(who) + ": q, k, v must be [T, d]");
        return std::make_pair((int64_t)b.shape[0], (int64_t)b.shape[1]);
    };
    m.def("banded_attention", [td](farr q, farr k, farr v, int64_t hbw, int num_cpus, bool causal) {
        (void)num_cpus;
        auto [T, d] = td(q, "banded_attention");
        auto [K, dk] = td(k, "banded_attention");
        if (dk != d || v.size() != K * d) throw py::value_error("banded_attention: k, v must be [K, d]");
        py::array_t<float> out({(py::ssize_t)T, (py::ssize_t)d});
        check(sili_banded_attention(q.data(), k.data(), v.data(), out.mutable_data(), 1, 1, T, K, d, hbw, 0, causal,
                                    nullptr));
        return out;
    }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("half_bandwidth"), py::arg("num_cpus") = 4,
       py::arg("causal") = false);
    m.def("sparse_banded_attention", [td](farr q, farr k, farr v, int64_t hbw, int64_t inner_k, int num_cpus,
                                          bool causal) {
        (void)num_cpus;
        auto [T, d] = td(q, "sparse_banded_attention");
        auto [K, dk] = td(k, "sparse_banded_attention");
        if (dk != d || v.size() != K * d) throw py::value_error("sparse_banded_attention: k, v must be [K, d]");
        py::array_t<float> out({(py::ssize_t)T, (py::ssize_t)d});
        check(sili_banded_attention(q.data(), k.data(), v.data(), out.mutable_data(), 1, 1, T, K, d, hbw, inner_k,
                                    causal, nullptr));
        return out;
    }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("half_bandwidth"), py::arg("inner_k") = 0,
       py::arg("num_cpus") = 4, py::arg("causal") = false);
    m.def("sparse_attention", [td](farr q, farr k, farr v, int64_t top_k, int num_cpus, bool causal) {
        (void)num_cpus;
        auto [T, d] = td(q, "sparse_attention");
        if (k.size() != T * d || v.size() != T * d) throw py::value_error("sparse_attention: q, k, v must be [T, d]");
        py::array_t<float> out({(py::ssize_t)T, (py::ssize_t)d});
        check(sili_sparse_attention(q.data(), k.data(), v.data(), out.mutable_data(), T, d, top_k, causal, nullptr));
        return out;
    }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("top_k") = 0, py::arg("num_cpus") = 4,
       py::arg("causal") = false);
    m.def("banded_attention_backward", [td](farr q, farr k, farr v, farr dO, int64_t hbw, int num_cpus, bool causal) {
        (void)num_cpus;
        auto [T, d] = td(q, "banded_attention_backward");
        auto [K, dk] = td(k, "banded_attention_backward");
        if (dk != d || v.size() != K * d || dO.size() != T * d)
            throw py::value_error("banded_attention_backward: k, v [K, d] and dO [T, d] expected");
        py::array_t<float> dQ({(py::ssize_t)T, (py::ssize_t)d}), dK({(py::ssize_t)K, (py::ssize_t)d}),
            dV({(py::ssize_t)K, (py::ssize_t)d});
        check(sili_banded_attention_backward(q.data(), k.data(), v.data(), dO.data(), dQ.mutable_data(),
                                             dK.mutable_data(), dV.mutable_data(), 1, 1, T, K, d, hbw, causal, nullptr));
        return py::make_tuple(dQ, dK, dV);
    }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("dO"), py::arg("half_bandwidth"), py::arg("num_cpus") = 4,
       py::arg("causal") = false);
    // device-pointer form over groups (heads x sequences), grouped-query KV
    m.def("banded_attention_ptr", [](uintptr_t q, uintptr_t k, uintptr_t v, uintptr_t out, int64_t groups,
                                     int64_t kv_groups, int64_t T, int64_t K, int64_t d, int64_t hbw, int64_t inner_k,
                                     bool causal, uintptr_t stream) {
        check(sili_banded_attention((const float*)q, (const float*)k, (const float*)v, (float*)out, groups, kv_groups,
                                    T, K, d, hbw, inner_k, causal, (void*)stream));
    }, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("groups"), py::arg("kv_groups"),
       py::arg("T"), py::arg("K"), py::arg("d"), py::arg("half_bandwidth"), py::arg("inner_k") = 0,
       py::arg("causal") = false, py::arg("stream") = 0);
    m.def("fp32_fma_peak", [](int device, int iters) {
        double tf = 0, ms = 0;
        check(sili_fp32_fma_peak(device, iters, &tf, &ms));
        return py::make_tuple(tf, ms);
    }, py::arg("device") = 0, py::arg("iters") = 4096);
    m.def("dense_to_csr", [](farr x, float thr) {
        auto b = x.request();
        const int rows = b.ndim == 2 ? (int)b.shape[0] : 1;
        const int cols = b.ndim == 2 ? (int)b.shape[1] : (int)b.shape[0];
        py::array_t<int> p((py::ssize_t)rows + 1);
        int64_t n = 0;
        check(sili_dense_to_csr(x.data(), rows, cols, thr, p.mutable_data(), nullptr, nullptr, &n, nullptr));
        py::array_t<int> i((py::ssize_t)n);
        py::array_t<float> v((py::ssize_t)n);
        check(sili_dense_to_csr(x.data(), rows, cols, thr, p.mutable_data(), i.mutable_data(), v.mutable_data(), &n, nullptr));
        return py::make_tuple(p, i, v);
    }, py::arg("x"), py::arg("threshold") = 1e-4f);
    m.def("dense_to_top_k_csr", [](farr x, int k, int num_threads) {
        (void)num_threads;
        auto b = x.request();
        const int rows = b.ndim == 2 ? (int)b.shape[0] : 1;
        const int cols = b.ndim == 2 ? (int)b.shape[1] : (int)b.shape[0];
        const int64_t kk = std::min<int64_t>(std::max(k, 0), (int64_t)rows * cols);
        py::array_t<int> p((py::ssize_t)rows + 1), i((py::ssize_t)kk);
        py::array_t<float> v((py::ssize_t)kk);
        check(sili_dense_to_top_k_csr(x.data(), rows, cols, kk, p.mutable_data(), i.mutable_data(), v.mutable_data(), nullptr));
        return py::make_tuple(p, i, v);
    }, py::arg("x"), py::arg("k"), py::arg("num_threads") = 4);
    m.def("fp4_quantize_array", [](farr v) {
        py::array_t<uint8_t> out((py::ssize_t)v.size());
        check(sili_fp4_quantize(v.data(), out.mutable_data(), (int64_t)v.size(), nullptr));
        return out;
    }, py::arg("vals"));
    m.def("seed_fp4_stochastic_rng", [](uint64_t seed) {
        std::lock_guard<std::mutex> g(g_live_mu);
        g_seed = seed;
        g_seeded = true;
        for (sili_layer* h : g_live) sili_layer_seed_rng(h, seed);
    }, py::arg("seed"));
}
