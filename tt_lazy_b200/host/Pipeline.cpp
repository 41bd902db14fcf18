// Pipeline.cpp -- row-chunked evaluation of a graph over one streamed batch.
//
// A graph whose batch input X [M, K] is streamed from host memory (an input
// batch that changes every run) or resident (a constant: the left operand of
// its matmuls) and whose every op up to a reduction over the batch dimension
// is row-local -- matmul with X's rows on the left,
// element-wise ops with row-broadcast [1, N] constants, reductions over
// non-batch dims -- is rebuilt as C copies over row chunks of X, whose
// batch-dim partial sums are added in chunk order, followed by what came
// after the reduction (the data-parallel all-reduce). Compiled into one tape,
// the chunks run one after the other on the library stream, while the upload
// of chunk c + 1 runs on the copy stream (ttc_h2d_prefetch): the host-to-
// device transfer of the batch overlaps the GEMMs instead of preceding them.
// A resident batch is cut into constant row views, uploaded once like the
// weights: the same work as the whole-batch plan in shorter GEMMs, which on a
// power-capped B200 hold higher clocks (the 65536-row MLP with the CTA-pair
// GEMM: 553-572 TFLOP/s in 8 chunks vs 477-513 as one batch, measured
// alternately in one process).
// No reference counterpart (the reference evaluates one host tensor at a time).
#include <map>
#include <set>
#include <stdexcept>

#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "operations.hpp"

namespace tt_lazy {

namespace {

using Key = std::pair<NodeId, uint16_t>;

struct Rebuilder {
    const float* x_host = nullptr;
    std::vector<uint32_t> x_shape;
    bool x_streamed = true;
    std::map<NodeId, bool> row_dep;  // node depends on X's rows
    Tensor chunk;                    // the current chunk of X
    std::map<Key, Tensor> memo;      // per chunk

    bool is_x(const Tensor& t) const {
        return !t.is_lazy() && t.host_data() == x_host && t.shape_vector() == x_shape;
    }

    bool depends(const Tensor& t) {
        if (!t.is_lazy()) return is_x(t);
        const NodeId id = t.producer_node();
        auto it = row_dep.find(id);
        if (it != row_dep.end()) return it->second;
        const Node* n = Context::instance().get_node(id);
        if (!n) throw std::runtime_error("pipelined plan: graph node missing");
        bool d = false;
        for (const auto& in : n->inputs()) d = depends(in) || d;
        row_dep[id] = d;
        return d;
    }

    static bool is_batch_reduce(const Node& n) {
        const auto* a = n.try_as<ReduceArgs>();
        if (!a || a->type != ReduceArgs::Type::SUM) return false;
        const auto& in = n.inputs()[0];
        const int r = (int)in.rank();
        if (r != 2) return false;
        return a->dims.size() == 1 && (a->dims[0] == 0 || a->dims[0] == -2);
    }

    // A row-region operand that does not depend on X must broadcast over rows.
    static void require_row_broadcast(const Tensor& t, const char* op) {
        const auto s = t.shape_vector();
        const bool ok = s.size() == 1 || (s.size() == 2 && s[0] == 1);
        if (!ok)
            throw std::runtime_error(std::string("pipelined plan: ") + op +
                                     " mixes the batch rows with a full-size tensor that is not row-chunked");
    }

    Tensor rebuild(const Tensor& t) {
        if (!t.is_lazy()) return is_x(t) ? chunk : t;
        if (!depends(t)) return t;
        const Key key{t.producer_node(), t.output_index()};
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
        const Node& n = *Context::instance().get_node(key.first);
        const auto& in = n.inputs();
        Tensor out;
        if (const auto* a = n.try_as<MatMulArgs>()) {
            if (!depends(in[0]) || depends(in[1]) || a->transpose_a)
                throw std::runtime_error("pipelined plan: matmul must take the batch rows as its left operand");
            out = matmul(rebuild(in[0]), in[1], a->transpose_a, a->transpose_b);
        } else if (n.is<ReLUArgs>()) {
            out = relu(rebuild(in[0]));
        } else if (n.is<SigmoidArgs>()) {
            out = sigmoid(rebuild(in[0]));
        } else if (n.is<AddArgs>() || n.is<MultiplyArgs>()) {
            for (const auto& x : in)
                if (!depends(x)) require_row_broadcast(x, "an element-wise op");
            out = n.is<AddArgs>() ? add(rebuild(in[0]), rebuild(in[1])) : multiply(rebuild(in[0]), rebuild(in[1]));
        } else if (const auto* f = n.try_as<FusedMLPArgs>()) {
            if (!depends(in[0]) || depends(in[1]) || depends(in[2]))
                throw std::runtime_error("pipelined plan: fused_mlp must take the batch rows as its input");
            require_row_broadcast(in[2], "fused_mlp");
            out = fused_mlp(rebuild(in[0]), in[1], in[2], f->has_relu);
        } else if (const auto* r = n.try_as<ReduceArgs>()) {
            for (int32_t d : r->dims)
                if (d == 0 || d == -(int32_t)in[0].rank())
                    throw std::runtime_error("pipelined plan: a reduction over the batch rows must end the row region");
            if (r->dims.empty()) throw std::runtime_error("pipelined plan: full reduction inside the row region");
            const std::vector<int32_t> dims(r->dims.begin(), r->dims.end());
            out = r->type == ReduceArgs::Type::MEAN ? reduce_mean(rebuild(in[0]), dims, r->keepdim)
                                                    : reduce_sum(rebuild(in[0]), dims, r->keepdim);
        } else {
            throw std::runtime_error(std::string("pipelined plan: op ") + std::string(n.op_name()) +
                                     " is not row-local");
        }
        memo[key] = out;
        return out;
    }
};

// The batch input: the streamed rank-2 tensor the outputs depend on (exactly
// one), or, with none streamed, the one rank-2 constant that is the left
// operand of a matmul / fused_mlp (the weights are right operands).
void find_batch_input(const std::vector<Tensor>& outputs, Rebuilder& rb) {
    std::set<NodeId> seen;
    std::vector<NodeId> stack;
    for (const auto& t : outputs)
        if (t.is_lazy()) stack.push_back(t.producer_node());
    int found = 0;
    std::set<std::pair<const float*, std::vector<uint32_t>>> resident;
    while (!stack.empty()) {
        const NodeId id = stack.back();
        stack.pop_back();
        if (!seen.insert(id).second) continue;
        const Node* n = Context::instance().get_node(id);
        if (!n) continue;
        const bool left_operand_op = n->is<MatMulArgs>() || n->is<FusedMLPArgs>();
        for (size_t i = 0; i < n->inputs().size(); ++i) {
            const auto& in = n->inputs()[i];
            if (in.is_lazy()) {
                stack.push_back(in.producer_node());
            } else if (in.is_streamed()) {
                if (found && (in.host_data() != rb.x_host || in.shape_vector() != rb.x_shape))
                    throw std::runtime_error("pipelined plan: more than one streamed input");
                rb.x_host = in.host_data();
                rb.x_shape = in.shape_vector();
                found = 1;
            } else if (left_operand_op && i == 0 && in.rank() == 2 && in.is_constant() && in.host_data()) {
                // a constant's caller-owned memory outlives the plan's row views of it
                resident.insert({in.host_data(), in.shape_vector()});
            }
        }
    }
    if (!found && resident.size() == 1) {
        rb.x_host = resident.begin()->first;
        rb.x_shape = resident.begin()->second;
        rb.x_streamed = false;
        found = 1;
    }
    if (!found || rb.x_shape.size() != 2)
        throw std::runtime_error(
            "pipelined plan: needs exactly one streamed rank-2 batch input (or, with none, one resident "
            "rank-2 constant as the left operand of the matmuls)");
}

}  // namespace

std::vector<Tensor> build_row_pipeline(const std::vector<Tensor>& outputs, int chunks) {
    Rebuilder rb;
    find_batch_input(outputs, rb);
    const uint32_t M = rb.x_shape[0], K = rb.x_shape[1];
    if (chunks < 2 || (uint32_t)chunks > M) throw std::runtime_error("pipelined plan: chunks must be in [2, rows]");
    // each output: a batch-dim sum of the row region, or an all-reduce of one
    struct Out {
        Tensor reduced_input;  // the row-region tensor the batch reduction reads
        bool keepdim = false;
        bool all_reduce = false;
    };
    std::vector<Out> plan;
    for (const auto& t : outputs) {
        if (!t.is_lazy()) throw std::runtime_error("pipelined plan: outputs must be lazy");
        const Node* n = Context::instance().get_node(t.producer_node());
        Out o;
        if (n->is<AllReduceArgs>()) {
            o.all_reduce = true;
            const auto& in = n->inputs()[0];
            n = in.is_lazy() ? Context::instance().get_node(in.producer_node()) : nullptr;
        }
        if (!n || !Rebuilder::is_batch_reduce(*n) || !rb.depends(n->inputs()[0]))
            throw std::runtime_error(
                "pipelined plan: every output must be reduce_sum over the batch rows (optionally all-reduced)");
        o.reduced_input = n->inputs()[0];
        o.keepdim = n->as<ReduceArgs>().keepdim;
        plan.push_back(o);
    }
    std::vector<Tensor> totals(plan.size());
    const uint32_t rows = (M + (uint32_t)chunks - 1) / (uint32_t)chunks;
    // Row ranges. A streamed batch's first chunk of 4096 rows or more is cut
    // into 1/8, 1/8, 1/4 and 1/2 of it: nothing computes until the first
    // upload lands, so a small first piece shortens that wait (1024 rows of
    // a 4096-wide fp32 batch: 16 MiB instead of 128), and the uploads, faster
    // than the GEMMs consume rows, stay ahead from then on.
    std::vector<std::pair<uint32_t, uint32_t>> ranges;
    uint32_t start = 0;
    if (rb.x_streamed && rows >= 4096) {
        for (uint32_t part : {rows / 8, rows / 8, rows / 4, rows - rows / 8 - rows / 8 - rows / 4}) {
            ranges.push_back({start, part});
            start += part;
        }
    }
    for (; start < M; start += rows) ranges.push_back({start, std::min(rows, M - start)});
    for (const auto& [r0, rc] : ranges) {
        rb.chunk = Tensor(const_cast<float*>(rb.x_host) + (size_t)r0 * K, std::vector<uint32_t>{rc, K});
        rb.chunk.set_streamed(rb.x_streamed);
        rb.memo.clear();
        for (size_t i = 0; i < plan.size(); ++i) {
            Tensor part = reduce_sum(rb.rebuild(plan[i].reduced_input), {0}, plan[i].keepdim);
            totals[i] = r0 == 0 ? part : add(totals[i], part);
        }
    }
    for (size_t i = 0; i < plan.size(); ++i)
        if (plan[i].all_reduce) totals[i] = all_reduce_sum(totals[i]);
    return totals;
}

}  // namespace tt_lazy
