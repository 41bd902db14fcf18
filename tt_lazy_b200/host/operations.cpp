// operations.cpp -- graph building (reference: src/frontend/operations.cpp)
// and the Context graph store (reference: src/core/Context.cpp).
//
// Shapes: every lazy output carries its true shape and rank, and the node
// records it (Node::output_shapes) for the backend. Shape errors that the
// reference only raises at evaluation time inside math::* are raised here
// with the reference's messages, at graph-build time.
#include "operations.hpp"

#include <algorithm>
#include <functional>
#include <iostream>
#include <queue>
#include <stdexcept>

// ------------------------------------------------------------------ Context
Context::Context() {
    nodes_.reserve(1024);
    id_to_index_.reserve(1024);
}

Node* Context::get_node(NodeId id) {
    auto it = id_to_index_.find(id);
    return it != id_to_index_.end() ? &nodes_[it->second] : nullptr;
}

const Node* Context::get_node(NodeId id) const {
    auto it = id_to_index_.find(id);
    return it != id_to_index_.end() ? &nodes_[it->second] : nullptr;
}

std::unordered_set<NodeId> Context::get_dependencies(const std::vector<Tensor>& outputs) const {
    std::unordered_set<NodeId> deps;
    std::vector<NodeId> stack;
    for (const auto& t : outputs)
        if (t.is_lazy() && t.producer_node() != 0) stack.push_back(t.producer_node());
    while (!stack.empty()) {
        const NodeId cur = stack.back();
        stack.pop_back();
        if (!deps.insert(cur).second) continue;
        if (const Node* n = get_node(cur))
            for (const auto& in : n->inputs())
                if (in.is_lazy() && in.producer_node() != 0) stack.push_back(in.producer_node());
    }
    return deps;
}

std::vector<NodeId> Context::topological_sort(const std::unordered_set<NodeId>& node_set) const {
    std::vector<NodeId> result;
    std::unordered_set<NodeId> done, active;
    std::function<void(NodeId)> visit = [&](NodeId id) {
        if (active.count(id)) throw std::runtime_error("Cycle detected in graph");
        if (done.count(id) || !node_set.count(id)) return;
        active.insert(id);
        if (const Node* n = get_node(id))
            for (const auto& in : n->inputs())
                if (in.is_lazy() && in.producer_node() != 0) visit(in.producer_node());
        active.erase(id);
        done.insert(id);
        result.push_back(id);
    };
    std::vector<NodeId> ids(node_set.begin(), node_set.end());
    std::sort(ids.begin(), ids.end());
    for (NodeId id : ids) visit(id);
    return result;
}

void Context::clear() {
    nodes_.clear();
    id_to_index_.clear();
    next_id_ = 1;
    ++epoch_;
}

void Context::print_stats() const {
    std::unordered_map<std::string, size_t> counts;
    for (const auto& n : nodes_) counts[std::string(n.op_name())]++;
    std::cout << "Graph statistics:\n  Total nodes: " << nodes_.size() << "\n";
    for (const auto& [name, c] : counts) std::cout << "    " << name << ": " << c << " nodes\n";
}

Context& Context::instance() {
    static Context ctx;
    return ctx;
}

// --------------------------------------------------------------- operations
namespace {
std::vector<uint32_t> shp(const Tensor& t) { return t.shape_vector(); }

template <typename ArgsT, size_t N>
Tensor make_node(const SmallVector<Tensor, N>& inputs, ArgsT&& args, const std::vector<uint32_t>& out_shape) {
    NodeId id = Context::instance().create_node(inputs, std::forward<ArgsT>(args));
    Context::instance().get_node(id)->set_output_shapes({out_shape});
    return Tensor(id, 0, out_shape);
}

// eltwise.cpp:29-83: same shape, or [N, M] + [1, M] only.
void check_add_shapes(const std::vector<uint32_t>& a, const std::vector<uint32_t>& b) {
    if (!Tensor::can_broadcast(a, b)) throw std::runtime_error("Cannot broadcast shapes for addition");
    if (a == b) return;
    if (a.size() == 2 && b.size() == 2 && b[0] == 1 && a[1] == b[1]) return;
    if (a.size() == 2 && b.size() == 2 && a[0] == 1 && a[1] == b[1]) return;  // [1,M] + [N,M]: commutative
    throw std::runtime_error("Broadcasting addition not implemented for these shapes");
}
}  // namespace

std::vector<Tensor> make_output_tensors(NodeId node_id, size_t num_outputs,
                                        const std::vector<std::vector<uint32_t>>& shapes) {
    std::vector<Tensor> out;
    out.reserve(num_outputs);
    for (size_t i = 0; i < num_outputs; ++i)
        out.emplace_back(node_id, (uint16_t)i, i < shapes.size() ? shapes[i] : std::vector<uint32_t>{1});
    return out;
}

std::vector<Tensor> split(const Tensor& input, int64_t split_size, int32_t dim) {
    if (dim < 0 || dim >= (int32_t)input.rank()) throw std::runtime_error("Invalid dimension for split operation");
    if (split_size <= 0) throw std::runtime_error("Split size must be positive");
    SplitArgs args;
    args.split_size = split_size;
    args.dim = dim;
    SmallVector<Tensor, 2> inputs{input};
    const NodeId id = Context::instance().create_node(inputs, std::move(args));
    const size_t size = input.size((size_t)dim);
    const size_t n = (size + (size_t)split_size - 1) / (size_t)split_size;
    std::vector<std::vector<uint32_t>> shapes;
    for (size_t i = 0; i < n; ++i) {
        auto s = shp(input);
        s[(size_t)dim] = (uint32_t)std::min<size_t>((size_t)split_size, size - i * (size_t)split_size);
        shapes.push_back(s);
    }
    Context::instance().get_node(id)->set_output_shapes(shapes);
    return make_output_tensors(id, n, shapes);
}

Tensor matmul(const Tensor& a, const Tensor& b, bool transpose_a, bool transpose_b) {
    if (a.rank() != 2 || b.rank() != 2) {
        if (a.rank() < 2 || b.rank() < 2)
            throw std::runtime_error("Matrix multiplication requires at least 2D tensors");
        throw std::runtime_error("Multi-dimensional matrix multiplication not fully implemented");
    }
    const uint32_t ar = transpose_a ? a.size(1) : a.size(0), ac = transpose_a ? a.size(0) : a.size(1);
    const uint32_t br = transpose_b ? b.size(1) : b.size(0), bc = transpose_b ? b.size(0) : b.size(1);
    if (ac != br) throw std::runtime_error("Matrix dimension mismatch for multiplication");
    MatMulArgs args;
    args.transpose_a = transpose_a;
    args.transpose_b = transpose_b;
    return make_node(SmallVector<Tensor, 2>{a, b}, std::move(args), {ar, bc});
}

std::vector<uint32_t> reduced_shape(const std::vector<uint32_t>& in, const std::vector<int32_t>& dims, bool keepdim) {
    const int r = (int)in.size();
    std::vector<bool> red((size_t)r, dims.empty());
    for (int32_t d : dims) {
        const int dd = d < 0 ? d + r : d;
        if (dd < 0 || dd >= r) throw std::runtime_error("reduce: dim out of range");
        red[(size_t)dd] = true;
    }
    std::vector<uint32_t> out;
    for (int i = 0; i < r; ++i) {
        if (!red[(size_t)i])
            out.push_back(in[(size_t)i]);
        else if (keepdim)
            out.push_back(1);
    }
    if (out.empty()) out.push_back(1);
    return out;
}

static Tensor reduce_op(const Tensor& input, const std::vector<int32_t>& dims, bool keepdim, ReduceArgs::Type type) {
    ReduceArgs args;
    for (int32_t d : dims) args.dims.push_back(d);
    args.keepdim = keepdim;
    args.type = type;
    const auto out = reduced_shape(shp(input), dims, keepdim);
    return make_node(SmallVector<Tensor, 2>{input}, std::move(args), out);
}

Tensor reduce_sum(const Tensor& input, const std::vector<int32_t>& dims, bool keepdim) {
    return reduce_op(input, dims, keepdim, ReduceArgs::Type::SUM);
}

Tensor reduce_mean(const Tensor& input, const std::vector<int32_t>& dims, bool keepdim) {
    return reduce_op(input, dims, keepdim, ReduceArgs::Type::MEAN);
}

Tensor relu(const Tensor& input) { return make_node(SmallVector<Tensor, 2>{input}, ReLUArgs{}, shp(input)); }

Tensor sigmoid(const Tensor& input) { return make_node(SmallVector<Tensor, 2>{input}, SigmoidArgs{}, shp(input)); }

Tensor add(const Tensor& a, const Tensor& b) {
    check_add_shapes(shp(a), shp(b));
    return make_node(SmallVector<Tensor, 2>{a, b}, AddArgs{}, Tensor::broadcast_shapes(shp(a), shp(b)));
}

Tensor multiply(const Tensor& a, const Tensor& b) {
    // eltwise.cpp:85-111: same shapes only.
    if (!Tensor::can_broadcast(shp(a), shp(b))) throw std::runtime_error("Cannot broadcast shapes for multiplication");
    if (shp(a) != shp(b)) throw std::runtime_error("Broadcasting multiplication not fully implemented");
    return make_node(SmallVector<Tensor, 2>{a, b}, MultiplyArgs{}, shp(a));
}

Tensor transpose(const Tensor& input) {
    if (input.rank() < 2) throw std::runtime_error("Transpose requires at least 2D tensor");
    auto s = shp(input);
    std::swap(s[s.size() - 1], s[s.size() - 2]);
    return make_node(SmallVector<Tensor, 2>{input}, TransposeArgs{}, s);
}

Tensor all_reduce_sum(const Tensor& input) {
    return make_node(SmallVector<Tensor, 2>{input}, AllReduceArgs{}, shp(input));
}

Tensor fused_mlp(const Tensor& input, const Tensor& weights, const Tensor& bias, bool has_relu) {
    if (input.rank() != 2 || weights.rank() != 2 || bias.rank() != 2)
        throw std::runtime_error("Fused MLP expects rank-2 input, weights and bias");
    if (weights.size(0) != input.size(1))
        throw std::runtime_error("Incompatible shapes for MLP: input features don't match weight rows");
    if (bias.size(1) != weights.size(1))
        throw std::runtime_error("Incompatible shapes for MLP: bias features don't match weight columns");
    FusedMLPArgs args;
    args.has_relu = has_relu;
    args.activation = has_relu ? 1 : 0;
    args.fusion_info = std::string("MatMul + Add") + (has_relu ? " + ReLU" : "");
    return make_node(SmallVector<Tensor, 3>{input, weights, bias}, std::move(args), {input.size(0), weights.size(1)});
}
