// OperationHandlers.cpp -- the reference tape's operation handlers on the
// B200 backend: a drop-in replacement for src/tape/OperationHandlers.cpp of
// the reference (ayerofieiev-tt/tt_lazy), built together with the
// reference's own, unmodified src/core, src/frontend and src/tape sources in
// place of its CPU library tt_math_lib (CMakeLists.txt:264-270 of the
// reference), calling only the C-ABI of include/tt_cuda.h.
//
// register_all_operations (TapeExecutor.hpp:46, OperationHandlers.cpp:224-232
// of the reference) installs one handler per op type, as the reference's
// does. Each handler gathers its operands in argument order from the node
// (lazy ones from the executor's results, constants as they are), uploads
// them, runs the op on the device and downloads the result into a new host
// Tensor that it hands to executor.set_result -- one host round trip per op,
// because the reference's Tensor holds host memory. Shape errors throw
// std::runtime_error with the reference's messages, and a non-zero C-ABI
// status throws with ttc_last_error().
//
// Differences from the reference handlers, all bug fixes:
// - matmul honours MatMulArgs::transpose_a / transpose_b (dropped at
//   OperationHandlers.cpp:61 of the reference);
// - reduce honours ReduceArgs::dims, keepdim and MEAN (the reference
//   hard-codes dims = {0}, OperationHandlers.cpp:90). Its result has the
//   element count of the lazy tensor the front end made (operations.cpp:96-103
//   of the reference: a dim counts as reduced only when listed, so dims = {}
//   keeps the input's shape), the reduced values first and zeros after, so
//   Tensor::eval_impl's copy of numel_ elements (Tensor.cpp:572 of the
//   reference) stays inside the result;
// - operands keep their argument order (the reference collects lazy
//   operands before constants).
// split stays as the reference has it (the whole input): the reference's
// evaluation manager keys results by node, so one split node cannot hold one
// result per chunk; the repository's own front end (tt_lazy_b200/host) keys
// them by (node, output index) and returns the chunks.
//
// The GEMM path follows TT_LAZY_GEMM (auto, tf32, tf32x3, ffma; read at
// every matmul); the device follows TT_LAZY_DEVICE (default 0).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "Context.hpp"
#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "operations.hpp"
#include "tt_cuda.h"

namespace {

void check(int rc) {
    if (rc != TTC_OK) throw std::runtime_error(ttc_last_error());
}

void backend_up() {
    static const bool up = [] {
        const char* e = std::getenv("TT_LAZY_DEVICE");
        check(ttc_init(e ? std::atoi(e) : 0));
        return true;
    }();
    (void)up;
}

int gemm_path() {
    const char* e = std::getenv("TT_LAZY_GEMM");
    if (!e) return TTC_GEMM_AUTO;
    const std::string s = e;
    if (s == "tf32") return TTC_GEMM_TF32;
    if (s == "tf32x3") return TTC_GEMM_TF32X3;
    if (s == "ffma") return TTC_GEMM_FFMA;
    return TTC_GEMM_AUTO;
}

// Device memory owned for the duration of one handler.
struct DeviceBuffer {
    float* ptr = nullptr;
    explicit DeviceBuffer(size_t n) { check(ttc_malloc(std::max<size_t>(n, 1) * sizeof(float), (void**)&ptr)); }
    ~DeviceBuffer() {
        if (ptr) ttc_free(ptr);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

std::vector<uint32_t> shape_of(const Tensor& t) { return std::vector<uint32_t>(t.shape(), t.shape() + t.rank()); }

std::unique_ptr<DeviceBuffer> upload(const Tensor& t) {
    const size_t n = t.total_elements();
    auto b = std::make_unique<DeviceBuffer>(n);
    if (n) check(ttc_memcpy_h2d(b->ptr, t.const_data_ptr(), n * sizeof(float)));
    return b;
}

std::shared_ptr<Tensor> download(const DeviceBuffer& b, const std::vector<uint32_t>& shape, size_t valid) {
    auto out = std::make_shared<Tensor>(shape);
    const size_t n = out->total_elements();
    if (valid) check(ttc_memcpy_d2h(out->data_ptr(), b.ptr, std::min(valid, n) * sizeof(float)));
    if (n > valid) std::memset(out->data_ptr() + valid, 0, (n - valid) * sizeof(float));
    return out;
}

// The node's operands in argument order.
std::vector<std::shared_ptr<Tensor>> operands(const TapeOperation& op, TapeExecutor& executor, size_t want,
                                              const char* what) {
    const Node* node = Context::instance().get_node(op.node_id);
    if (!node) throw std::runtime_error(std::string("Cannot find node for ") + what + " operation");
    std::vector<std::shared_ptr<Tensor>> in;
    for (const Tensor& t : node->inputs()) {
        if (t.is_lazy()) {
            auto r = executor.get_result(t.producer_node());
            if (!r) throw std::runtime_error(std::string("Missing lazy input tensor for ") + what + " operation");
            in.push_back(r);
        } else {
            in.push_back(std::make_shared<Tensor>(t));
        }
    }
    if (in.size() != want)
        throw std::runtime_error(std::string(what) + " operation requires exactly " + std::to_string(want) +
                                 " input" + (want == 1 ? "" : "s") + ", got " + std::to_string(in.size()));
    return in;
}

void finish(TapeOperation& op, TapeExecutor& executor, std::shared_ptr<Tensor> result) {
    executor.set_result(op.node_id, result);
    op.result = std::move(result);
}

ttc_instr ins(int op, int src = 0, int idx = 0) {
    ttc_instr i;
    i.op = (uint8_t)op;
    i.src = (uint8_t)src;
    i.idx = (uint8_t)idx;
    i.pad = 0;
    return i;
}

// One chain launch over `n` elements seen as [rows, cols].
ttc_chain_desc chain(int64_t rows, int64_t cols) {
    if (rows > INT32_MAX || cols > INT32_MAX) throw std::runtime_error("tensor too large for one chain launch");
    ttc_chain_desc d;
    std::memset(&d, 0, sizeof d);
    d.rows = (int32_t)rows;
    d.cols = (int32_t)cols;
    d.nseg = 1;
    return d;
}

void unary(TapeOperation& op, TapeExecutor& executor, int opcode, const char* what) {
    backend_up();
    auto in = operands(op, executor, 1, what);
    const size_t n = in[0]->total_elements();
    auto x = upload(*in[0]);
    DeviceBuffer y(n);
    if (n) {
        ttc_chain_desc d = chain(1, (int64_t)n);
        d.n_inputs = 1;
        d.inputs[0] = ttc_in_view{x->ptr, (int64_t)n, 1, 0};
        d.n_outputs = 1;
        d.outputs[0] = ttc_out_view{y.ptr, (int64_t)n, 0};
        d.n_instr = 3;
        d.program[0] = ins(TTC_OP_LOAD, TTC_SRC_INPUT, 0);
        d.program[1] = ins(opcode, 0, 0);
        d.program[2] = ins(TTC_OP_STORE, 0, 0);
        check(ttc_eltwise_chain(&d));
    }
    finish(op, executor, download(y, shape_of(*in[0]), n));
}

// add / multiply with the reference's broadcasting rules (eltwise.cpp:29-111):
// equal shapes, or for add a [N, M] + [1, M] bias.
void binary(TapeOperation& op, TapeExecutor& executor, int opcode, const char* what) {
    backend_up();
    auto in = operands(op, executor, 2, what);
    const auto as = shape_of(*in[0]), bs = shape_of(*in[1]);
    const bool is_add = opcode == TTC_OP_ADD;
    if (!Tensor::can_broadcast(as, bs))
        throw std::runtime_error(is_add ? "Cannot broadcast shapes for addition"
                                        : "Cannot broadcast shapes for multiplication");
    const bool bias = as != bs;
    if (bias && !(is_add && as.size() == 2 && bs.size() == 2 && bs[0] == 1 && as[1] == bs[1]))
        throw std::runtime_error(is_add ? "Broadcasting addition not implemented for these shapes"
                                        : "Broadcasting multiplication not fully implemented");
    const size_t n = in[0]->total_elements();
    const int64_t cols = bias ? as[1] : (int64_t)n, rows = bias ? as[0] : 1;
    auto a = upload(*in[0]);
    auto b = upload(*in[1]);
    DeviceBuffer y(n);
    if (n) {
        ttc_chain_desc d = chain(rows, cols);
        d.n_inputs = 2;
        d.inputs[0] = ttc_in_view{a->ptr, cols, 1, 0};
        d.inputs[1] = ttc_in_view{b->ptr, bias ? 0 : cols, 1, 0};  // row stride 0: the bias row for every row
        d.n_outputs = 1;
        d.outputs[0] = ttc_out_view{y.ptr, cols, 0};
        d.n_instr = 3;
        d.program[0] = ins(TTC_OP_LOAD, TTC_SRC_INPUT, 0);
        d.program[1] = ins(opcode, TTC_SRC_INPUT, 1);
        d.program[2] = ins(TTC_OP_STORE, 0, 0);
        check(ttc_eltwise_chain(&d));
    }
    finish(op, executor, download(y, as, n));
}

// C = act(op(A) op(B) [+ bias]) on the device; shapes per matmul.cpp:56-82 /
// fused_ops.cpp:15-25 of the reference.
std::shared_ptr<Tensor> gemm(const Tensor& A, const Tensor& B, bool ta, bool tb, const Tensor* bias, bool relu) {
    if (A.rank() < 2 || B.rank() < 2) throw std::runtime_error("Matrix multiplication requires at least 2D tensors");
    if (A.rank() > 2 || B.rank() > 2)
        throw std::runtime_error("Multi-dimensional matrix multiplication not fully implemented");
    const int64_t m = ta ? A.size(1) : A.size(0), k = ta ? A.size(0) : A.size(1);
    const int64_t kb = tb ? B.size(1) : B.size(0), n = tb ? B.size(0) : B.size(1);
    if (k != kb) throw std::runtime_error("Matrix dimension mismatch for multiplication");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) throw std::runtime_error("matmul dimension exceeds 2^31");
    if (bias && (bias->total_elements() != (size_t)n))
        throw std::runtime_error("Incompatible shapes for MLP: bias features don't match weight columns");
    auto a = upload(A);
    auto b = upload(B);
    std::unique_ptr<DeviceBuffer> bb;
    if (bias) bb = upload(*bias);
    DeviceBuffer c((size_t)(m * n));
    ttc_gemm_desc g;
    std::memset(&g, 0, sizeof g);
    g.M = (int32_t)m;
    g.N = (int32_t)n;
    g.K = (int32_t)k;
    g.a = a->ptr;
    g.lda = A.size(1);
    g.trans_a = ta;
    g.b = b->ptr;
    g.ldb = B.size(1);
    g.trans_b = tb;
    g.c = c.ptr;
    g.ldc = n;
    g.path = gemm_path();
    // epilogue over the accumulator: [+ bias row] [relu] store (none: store to c)
    ttc_chain_desc& epi = g.epilogue;
    int pc = 0;
    if (bias) {
        epi.n_inputs = 1;
        epi.inputs[0] = ttc_in_view{bb->ptr, 0, 1, 0};
        epi.program[pc++] = ins(TTC_OP_ADD, TTC_SRC_INPUT, 0);
    }
    if (relu) epi.program[pc++] = ins(TTC_OP_RELU, 0, 0);
    if (pc) {
        epi.n_outputs = 1;
        epi.outputs[0] = ttc_out_view{c.ptr, n, 0};
        epi.program[pc++] = ins(TTC_OP_STORE, 0, 0);
    }
    epi.n_instr = pc;
    if (m && n) check(ttc_gemm(&g));
    return download(c, {(uint32_t)m, (uint32_t)n}, (size_t)(m * n));
}

void handle_matmul(TapeOperation& op, TapeExecutor& executor) {
    backend_up();
    auto in = operands(op, executor, 2, "MatMul");
    const auto& args = Context::instance().get_node(op.node_id)->as<MatMulArgs>();
    finish(op, executor, gemm(*in[0], *in[1], args.transpose_a, args.transpose_b, nullptr, false));
}

void handle_fused_mlp(TapeOperation& op, TapeExecutor& executor) {
    backend_up();
    auto in = operands(op, executor, 3, "Fused MLP");
    const auto& args = Context::instance().get_node(op.node_id)->as<FusedMLPArgs>();
    if (in[0]->rank() == 2 && in[1]->rank() == 2 && in[0]->size(1) != in[1]->size(0))
        throw std::runtime_error("Incompatible shapes for MLP: input features don't match weight rows");
    finish(op, executor, gemm(*in[0], *in[1], false, false, in[2].get(), args.has_relu));
}

void handle_reduce(TapeOperation& op, TapeExecutor& executor) {
    backend_up();
    auto in = operands(op, executor, 1, "Reduce");
    const auto& args = Context::instance().get_node(op.node_id)->as<ReduceArgs>();
    if (args.type != ReduceArgs::Type::SUM && args.type != ReduceArgs::Type::MEAN)
        throw std::runtime_error("Reduce: only SUM and MEAN are implemented");
    const Tensor& x = *in[0];
    const int rank = x.rank();
    std::vector<int32_t> dims(args.dims.begin(), args.dims.end());
    size_t kept = 1;  // elements of the reduced result
    std::vector<bool> red(rank, dims.empty());
    for (int32_t d : dims) {
        const int dd = d < 0 ? d + rank : d;
        if (dd < 0 || dd >= rank) throw std::runtime_error("Reduce: dim out of range");
        red[dd] = true;
    }
    for (int i = 0; i < rank; ++i)
        if (!red[i]) kept *= x.size(i);
    // the shape the front end gave the lazy tensor (operations.cpp:96-103 of the reference)
    std::vector<uint32_t> lazy_shape;
    for (int i = 0; i < rank; ++i) {
        const bool listed = std::find(dims.begin(), dims.end(), i) != dims.end();
        if (!listed || args.keepdim) lazy_shape.push_back(listed ? 1 : x.size(i));
    }
    if (lazy_shape.empty()) lazy_shape.push_back(1);
    auto xd = upload(x);
    DeviceBuffer y(kept);
    if (x.total_elements()) {
        std::vector<uint32_t> shape = shape_of(x);
        check(ttc_reduce(xd->ptr, shape.data(), rank, dims.data(), (int)dims.size(),
                         args.type == ReduceArgs::Type::MEAN ? 1 : 0, y.ptr));
    } else {
        check(ttc_memset_zero(y.ptr, kept * sizeof(float)));
    }
    finish(op, executor, download(y, lazy_shape, kept));
}

void handle_split(TapeOperation& op, TapeExecutor& executor) {
    backend_up();
    auto in = operands(op, executor, 1, "Split");
    finish(op, executor, std::make_shared<Tensor>(*in[0]));
}

void handle_relu(TapeOperation& op, TapeExecutor& executor) { unary(op, executor, TTC_OP_RELU, "ReLU"); }
void handle_add(TapeOperation& op, TapeExecutor& executor) { binary(op, executor, TTC_OP_ADD, "Add"); }
void handle_multiply(TapeOperation& op, TapeExecutor& executor) { binary(op, executor, TTC_OP_MUL, "Multiply"); }

}  // namespace

void register_all_operations(TapeExecutor& executor) {
    executor.register_operation(SplitArgs::type_id(), handle_split);
    executor.register_operation(MatMulArgs::type_id(), handle_matmul);
    executor.register_operation(ReduceArgs::type_id(), handle_reduce);
    executor.register_operation(ReLUArgs::type_id(), handle_relu);
    executor.register_operation(AddArgs::type_id(), handle_add);
    executor.register_operation(MultiplyArgs::type_id(), handle_multiply);
    executor.register_operation(FusedMLPArgs::type_id(), handle_fused_mlp);
}
