// Test entry points of the reference-side binding build
// (tests/native/build_reference_binding.sh): the reference's own, unmodified
// front end and tape, with tt_lazy_b200/binding/OperationHandlers.cpp as
// its handlers, driven through plain C functions so the GPU tests can call
// them with ctypes. Each builds the graph with the reference's public
// functions (relu / add / multiply / reduce_sum / matmul) over constant
// tensors and materialises the outputs with Tensor::to_vector(), which runs
// the reference's TapeEvaluationManager -> TapeGenerator -> TapeExecutor ->
// the binding's handlers -> libtt_cuda.so. Test infrastructure only.
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <spdlog/spdlog.h>

#include "Context.hpp"
#include "EvaluationManager.hpp"
#include "Tensor.hpp"
#include "operations.hpp"

namespace {
std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        spdlog::set_level(spdlog::level::off);
        Context::instance().clear();
        tt_lazy::get_evaluation_manager().clear_cache();
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

void copy_out(const Tensor& t, float* out, size_t n) {
    const std::vector<float> v = t.to_vector();
    if (v.size() < n) throw std::runtime_error("result has " + std::to_string(v.size()) + " elements, expected " +
                                               std::to_string(n));
    std::memcpy(out, v.data(), n * sizeof(float));
}
}  // namespace

extern "C" {

const char* rb_last_error(void) { return g_err.c_str(); }

// README chain: w = (relu(x) + relu(x))^2, s = reduce_sum(w) (dims = {}).
// w_out gets rows * cols values, s_out the total (element 0 of s).
int rb_readme_chain(const float* x, uint32_t rows, uint32_t cols, float* w_out, float* s_out) {
    return guarded([&] {
        Tensor X(const_cast<float*>(x), {rows, cols});
        Tensor y = relu(X);
        Tensor z = add(y, y);
        Tensor w = multiply(z, z);
        Tensor s = reduce_sum(w);
        copy_out(w, w_out, (size_t)rows * cols);
        copy_out(s, s_out, 1);
    });
}

// Two-layer MLP: y = relu(x W1 + b1) W2 + b2 (b rows of [1, n] broadcast).
int rb_mlp2(const float* x, uint32_t n, uint32_t d_in, const float* w1, uint32_t d_h, const float* b1,
            const float* w2, uint32_t d_out, const float* b2, float* y_out) {
    return guarded([&] {
        Tensor X(const_cast<float*>(x), {n, d_in});
        Tensor W1(const_cast<float*>(w1), {d_in, d_h});
        Tensor B1(const_cast<float*>(b1), {1, d_h});
        Tensor W2(const_cast<float*>(w2), {d_h, d_out});
        Tensor B2(const_cast<float*>(b2), {1, d_out});
        Tensor h = relu(add(matmul(X, W1), B1));
        Tensor y = add(matmul(h, W2), B2);
        copy_out(y, y_out, (size_t)n * d_out);
    });
}

// Row sums through the reduce handler: out[r] = sum_c x[r, c] (dims = {1}).
int rb_row_sums(const float* x, uint32_t rows, uint32_t cols, float* out) {
    return guarded([&] {
        Tensor X(const_cast<float*>(x), {rows, cols});
        Tensor r = reduce_sum(relu(X), {1});
        copy_out(r, out, rows);
    });
}

// A shape error raised by a handler reaches the caller as the reference's
// std::runtime_error (here: adding [n, m] and [n, 1]).
int rb_bad_broadcast(const float* a, uint32_t n, uint32_t m, const float* b) {
    return guarded([&] {
        Tensor A(const_cast<float*>(a), {n, m});
        Tensor B(const_cast<float*>(b), {n, 1});
        Tensor c = add(relu(A), B);
        c.to_vector();
    });
}

}  // extern "C"
