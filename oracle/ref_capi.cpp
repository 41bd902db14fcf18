// ref_capi.cpp -- extern "C" entry points into the reference's own code.
//
// TEST INFRASTRUCTURE ONLY. oracle/build_ref.sh compiles this file together
// with the UNMODIFIED reference sources (src/core, src/frontend, src/tape,
// src/tape/passes, src/backend/cpu of ayerofieiev-tt/tt_lazy) into
// oracle/_ref/libttref.so. tests/ use it to pin the C restatement (oracle.c)
// and bench.py's reference arm times it. Nothing on the product path loads it.
//
// Two kinds of entry point:
//  * ref_math_*  call `namespace math` directly (the backend seam,
//    src/backend/cpu/math_operations.hpp:6-31), the pattern of
//    tests/cpp/unit/math/test_math_ops.cpp.
//  * ref_lazy_*  build a graph with the frontend ops on constant tensors and
//    materialise it with to_vector() (the full tape path, call stack
//    Tensor.cpp:274 -> TapeEvaluationManager.cpp:18 -> OperationHandlers.cpp).
#include "Context.hpp"
#include "EvaluationManager.hpp"
#include "Tensor.hpp"
#include "math_operations.hpp"
#include "operations.hpp"

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <spdlog/spdlog.h>

namespace {
std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

std::vector<uint32_t> shp(const uint32_t* s, int rank) { return std::vector<uint32_t>(s, s + rank); }

Tensor materialized(const float* x, const uint32_t* s, int rank) {
    auto shape = shp(s, rank);
    size_t n = 1;
    for (auto d : shape) n *= d;
    return Tensor(shape, std::vector<float>(x, x + n));
}

// Constant tensor over caller memory: Tensor(void*, initializer_list) (Tensor.hpp:37).
Tensor constant(const float* x, const uint32_t* s, int rank) {
    void* p = const_cast<float*>(x);
    switch (rank) {
        case 1: return Tensor(p, {s[0]});
        case 2: return Tensor(p, {s[0], s[1]});
        case 3: return Tensor(p, {s[0], s[1], s[2]});
        default: return Tensor(p, {s[0], s[1], s[2], s[3]});
    }
}

void copy_out(const Tensor& t, float* out) {
    const float* d = t.const_data_ptr();
    std::memcpy(out, d, t.total_elements() * sizeof(float));
}

void fresh_graph() {
    Context::instance().clear();
    tt_lazy::get_evaluation_manager().clear_cache();
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

void ref_quiet() { spdlog::set_level(spdlog::level::off); }

int ref_math_relu(const float* x, const uint32_t* s, int rank, float* out) {
    return guarded([&] { copy_out(math::relu(materialized(x, s, rank)), out); });
}

int ref_math_add(const float* a, const uint32_t* as, int ar, const float* b, const uint32_t* bs, int br,
                 float* out) {
    return guarded([&] { copy_out(math::add(materialized(a, as, ar), materialized(b, bs, br)), out); });
}

int ref_math_multiply(const float* a, const uint32_t* as, int ar, const float* b, const uint32_t* bs, int br,
                      float* out) {
    return guarded([&] { copy_out(math::multiply(materialized(a, as, ar), materialized(b, bs, br)), out); });
}

int ref_math_matmul(const float* a, const uint32_t* as, const float* b, const uint32_t* bs, int ta, int tb,
                    float* out) {
    return guarded(
        [&] { copy_out(math::matmul(materialized(a, as, 2), materialized(b, bs, 2), ta != 0, tb != 0), out); });
}

int ref_math_fused_mlp(const float* x, const uint32_t* xs, const float* w, const uint32_t* ws, const float* b,
                       const uint32_t* bs, int has_relu, float* out) {
    return guarded([&] {
        copy_out(math::fused_mlp(materialized(x, xs, 2), materialized(w, ws, 2), materialized(b, bs, 2),
                                 has_relu != 0),
                 out);
    });
}

// Writes the reference result's element count to *out_numel (the reference
// keeps the input shape for dims={} and stores the sum in element 0).
int ref_math_reduce_sum(const float* x, const uint32_t* s, int rank, const int32_t* dims, int ndims,
                        int keepdim, float* out, size_t out_cap, size_t* out_numel) {
    return guarded([&] {
        Tensor r = math::reduce_sum(materialized(x, s, rank), std::vector<int32_t>(dims, dims + ndims),
                                    keepdim != 0);
        *out_numel = r.total_elements();
        if (r.total_elements() > out_cap) throw std::runtime_error("ref_math_reduce_sum: out too small");
        copy_out(r, out);
    });
}

int ref_math_transpose(const float* x, const uint32_t* s, int rank, float* out) {
    return guarded([&] { copy_out(math::transpose(materialized(x, s, rank)), out); });
}

// 1-D split (the only rank split.cpp implements): writes all chunks back to
// back into out.
int ref_math_split_1d(const float* x, uint32_t n, int64_t split_size, float* out) {
    return guarded([&] {
        uint32_t s = n;
        auto parts = math::split(materialized(x, &s, 1), split_size, 0);
        size_t off = 0;
        for (auto& p : parts) {
            copy_out(p, out + off);
            off += p.total_elements();
        }
    });
}

int ref_math_sigmoid_unavailable() { return -1; }  // no math::sigmoid in the reference

// Lazy path, element-wise chain of the README: w = (relu(x) + relu(x))^2 with
// y = relu(x), z = add(y, y), w = multiply(z, z). Evaluated by to_vector().
int ref_lazy_chain(const float* x, const uint32_t* s, int rank, float* w_out) {
    return guarded([&] {
        fresh_graph();
        Tensor xt = constant(x, s, rank);
        Tensor y = relu(xt);
        Tensor z = add(y, y);
        Tensor w = multiply(z, z);
        auto v = w.to_vector();
        std::memcpy(w_out, v.data(), v.size() * sizeof(float));
        fresh_graph();
    });
}

// Lazy path, two-layer MLP relu(x W1 + b1) W2 + b2 (test_mlp_demo.cpp:46-56).
int ref_lazy_mlp2(const float* x, const uint32_t* xs, const float* w1, const uint32_t* w1s, const float* b1,
                  const uint32_t* b1s, const float* w2, const uint32_t* w2s, const float* b2, const uint32_t* b2s,
                  float* out) {
    return guarded([&] {
        fresh_graph();
        Tensor X = constant(x, xs, 2), W1 = constant(w1, w1s, 2), B1 = constant(b1, b1s, 2);
        Tensor W2 = constant(w2, w2s, 2), B2 = constant(b2, b2s, 2);
        Tensor h = relu(add(matmul(X, W1), B1));
        Tensor y = add(matmul(h, W2), B2);
        auto v = y.to_vector();
        std::memcpy(out, v.data(), v.size() * sizeof(float));
        fresh_graph();
    });
}

// Lazy path, explicit fused op (operations.cpp:184-207 -> fused_ops.cpp).
int ref_lazy_fused_mlp(const float* x, const uint32_t* xs, const float* w, const uint32_t* ws, const float* b,
                       const uint32_t* bs, int has_relu, float* out) {
    return guarded([&] {
        fresh_graph();
        Tensor y = fused_mlp(constant(x, xs, 2), constant(w, ws, 2), constant(b, bs, 2), has_relu != 0);
        auto v = y.to_vector();
        std::memcpy(out, v.data(), v.size() * sizeof(float));
        fresh_graph();
    });
}

// ---- timed CPU baseline of the large MLP workload (bench.py --impl reference)
// Y = sigmoid(relu(X W1) W2), s = column sums of Y, for a row sample of X.
// The two matmuls and the relu are the reference's own math::matmul /
// math::relu (src/backend/cpu/matmul.cpp, eltwise.cpp); the reference has no
// sigmoid and no per-dim reduction on this path, so those two cheap steps
// follow the README formula (README.md:332) and a sequential column sum.
// Weights are wrapped once (ref_mlp_prepare) so every call times only the
// compute; calls on different rows may run concurrently.
namespace {
Tensor* g_w1 = nullptr;
Tensor* g_w2 = nullptr;
}  // namespace

int ref_mlp_prepare(const float* w1, const uint32_t* w1s, const float* w2, const uint32_t* w2s) {
    return guarded([&] {
        delete g_w1;
        delete g_w2;
        g_w1 = new Tensor(materialized(w1, w1s, 2));
        g_w2 = new Tensor(materialized(w2, w2s, 2));
    });
}

int ref_mlp_rows(const float* x, uint32_t rows, uint32_t k, float* colsum) {
    return guarded([&] {
        if (!g_w1 || !g_w2) throw std::runtime_error("ref_mlp_prepare not called");
        uint32_t xs[2] = {rows, k};
        Tensor h = math::relu(math::matmul(materialized(x, xs, 2), *g_w1));
        Tensor y = math::matmul(h, *g_w2);
        const float* yd = y.const_data_ptr();
        const uint32_t n = y.size(1);
        for (uint32_t j = 0; j < n; ++j) colsum[j] = 0.0f;
        for (uint32_t i = 0; i < rows; ++i)
            for (uint32_t j = 0; j < n; ++j) colsum[j] += 1.0f / (1.0f + std::exp(-yd[(size_t)i * n + j]));
    });
}

}  // extern "C"
