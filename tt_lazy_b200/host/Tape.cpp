// Tape.cpp -- tape, tape generation and the optimisation passes.
//
// Generation follows the reference (src/tape/TapeGenerator.cpp:20-74):
// collect the dependencies of the outputs, topologically sort them (Kahn),
// build one TapeOperation per node, run the passes by priority. Differences:
// no logging on the hot path (the reference prints through spdlog on every
// generation), a deterministic topological order (ties broken by node id),
// operands kept in argument order, materialized non-constant inputs kept
// (the reference drops them, TapeGenerator.cpp:159-170, so relu(Tensor(...))
// fails), and real output shapes.
#include <algorithm>
#include <functional>
#include <map>
#include <queue>
#include <set>
#include <sstream>
#include <stdexcept>

#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "operations.hpp"
#include "tt_cuda.h"

// --------------------------------------------------------------------- Tape
void Tape::add_operation(std::unique_ptr<TapeOperation> op) {
    operations_.push_back(std::move(op));
    build_node_map();
}

void Tape::build_node_map() {
    node_to_op_.clear();
    for (const auto& op : operations_) {
        node_to_op_[op->node_id] = op.get();
        for (NodeId n : op->output_nodes) node_to_op_[n] = op.get();
        if (op->plan) {
            for (const auto& m : op->plan->members) node_to_op_[m.node] = op.get();
            for (const auto& seg : op->plan->seg_nodes)
                for (NodeId s : seg) node_to_op_[s] = op.get();
            if (op->plan->has_matmul) node_to_op_[op->plan->matmul_node] = op.get();
        }
    }
}

TapeOperation* Tape::find_operation(NodeId node_id) {
    auto it = node_to_op_.find(node_id);
    return it != node_to_op_.end() ? it->second : nullptr;
}

const TapeOperation* Tape::find_operation(NodeId node_id) const {
    auto it = node_to_op_.find(node_id);
    return it != node_to_op_.end() ? it->second : nullptr;
}

TapeOperation* Tape::producer_of(NodeId id) { return find_operation(id); }

std::vector<NodeId> Tape::get_dependencies(NodeId node_id) const {
    const TapeOperation* op = find_operation(node_id);
    return op ? op->input_nodes : std::vector<NodeId>{};
}

bool Tape::is_valid() const {
    for (const auto& op : operations_)
        for (NodeId in : op->input_nodes)
            if (!find_operation(in)) return false;
    return true;
}

void Tape::validate() const {
    if (!is_valid()) throw std::runtime_error("Invalid tape: missing dependencies");
}

void Tape::print_tape(std::ostream& os) const {
    os << "Tape with " << operations_.size() << " operations:\n";
    for (size_t i = 0; i < operations_.size(); ++i) {
        const auto& op = operations_[i];
        os << "  " << i << ": Node " << op->node_id << " (op_type: " << op->op_type << ")";
        if (op->plan) os << " fused: " << op->plan->describe();
        os << "\n    Inputs:";
        for (NodeId in : op->input_nodes) os << " " << in;
        os << "\n    Outputs:";
        for (NodeId out : op->output_nodes) os << " " << out;
        os << "\n";
    }
}

void Tape::print_tape() const { print_tape(std::cout); }

std::string FusionPlan::describe() const {
    static const char* names[] = {"relu", "sigmoid", "add", "multiply", "reduce"};
    std::ostringstream o;
    if (has_matmul) o << "matmul" << (members.empty() ? "" : " -> ");
    for (size_t i = 0; i < members.size(); ++i) o << (i ? " -> " : "") << names[members[i].op];
    if (nseg > 1) o << " x" << nseg << " segments";
    return o.str();
}

// ---------------------------------------------------------------- generator
bool TapeGenerator::default_passes_registered_ = false;

std::vector<std::unique_ptr<TapeOptimizationPass>>& TapeGenerator::passes() {
    static std::vector<std::unique_ptr<TapeOptimizationPass>> p;
    return p;
}

void TapeGenerator::register_optimization_pass(std::unique_ptr<TapeOptimizationPass> pass) {
    passes().push_back(std::move(pass));
}

void TapeGenerator::register_default_passes() {
    if (default_passes_registered_) return;
    register_optimization_pass(std::make_unique<DeadCodeEliminationPass>());
    register_optimization_pass(std::make_unique<MLPFusionPass>());
    register_optimization_pass(std::make_unique<EltwiseFusionPass>());
    register_optimization_pass(std::make_unique<SegmentFusionPass>());
    default_passes_registered_ = true;
}

void TapeGenerator::clear_passes() {
    passes().clear();
    default_passes_registered_ = false;
}

std::unique_ptr<Tape> TapeGenerator::generate_tape(const Tensor& output) {
    return generate_tape(std::vector<Tensor>{output});
}

std::unique_ptr<Tape> TapeGenerator::generate_tape(const std::vector<Tensor>& outputs) {
    auto tape = std::make_unique<Tape>();
    tape->set_outputs(outputs);
    const auto deps = collect_dependencies(outputs);
    const auto order = topological_sort(deps);
    auto& ctx = Context::instance();
    for (NodeId id : order)
        if (const Node* n = ctx.get_node(id)) tape->operations_.push_back(create_tape_operation(*n));
    tape->build_node_map();
    if (optimization_enabled_) {
        if (!default_passes_registered_) register_default_passes();
        std::vector<TapeOptimizationPass*> ps;
        for (auto& p : passes()) ps.push_back(p.get());
        std::stable_sort(ps.begin(), ps.end(), [](auto* a, auto* b) {
            if (a->priority() != b->priority()) return a->priority() < b->priority();
            return a->name() < b->name();
        });
        for (auto* p : ps) p->apply(*tape, outputs);
    }
    return tape;
}

std::vector<NodeId> TapeGenerator::collect_dependencies(const std::vector<Tensor>& outputs) {
    const auto set = Context::instance().get_dependencies(outputs);
    return std::vector<NodeId>(set.begin(), set.end());
}

// Kahn's algorithm; among ready nodes the smallest id goes first, so the
// order (and every cache keyed on it) is reproducible.
std::vector<NodeId> TapeGenerator::topological_sort(const std::vector<NodeId>& nodes) {
    auto& ctx = Context::instance();
    std::unordered_set<NodeId> in_set(nodes.begin(), nodes.end());
    std::unordered_map<NodeId, int> indeg;
    std::unordered_map<NodeId, std::vector<NodeId>> users;
    for (NodeId id : nodes) {
        indeg[id];
        if (const Node* n = ctx.get_node(id))
            for (const auto& in : n->inputs())
                if (in.is_lazy() && in_set.count(in.producer_node())) {
                    users[in.producer_node()].push_back(id);
                    indeg[id]++;
                }
    }
    std::priority_queue<NodeId, std::vector<NodeId>, std::greater<NodeId>> ready;
    for (auto& [id, d] : indeg)
        if (d == 0) ready.push(id);
    std::vector<NodeId> out;
    while (!ready.empty()) {
        const NodeId cur = ready.top();
        ready.pop();
        out.push_back(cur);
        for (NodeId u : users[cur])
            if (--indeg[u] == 0) ready.push(u);
    }
    if (out.size() != nodes.size()) throw std::runtime_error("Cycle detected in graph");
    return out;
}

std::unique_ptr<TapeOperation> TapeGenerator::create_tape_operation(const Node& node) {
    auto op = std::make_unique<TapeOperation>(node.id(), node.type_id());
    for (const auto& in : node.inputs()) {
        if (in.is_lazy()) {
            op->input_nodes.push_back(in.producer_node());
            op->operands.push_back(OperandRef::of_node(in.producer_node(), in.output_index()));
        } else {
            op->constant_inputs.push_back(in);
            op->operands.push_back(OperandRef::of_tensor(in));
        }
    }
    op->output_nodes.push_back(node.id());
    op->output_shapes = node.output_shapes();
    return op;
}

// --------------------------------------------------------------- DCE pass
int DeadCodeEliminationPass::apply(Tape& tape, const std::vector<Tensor>& outputs) {
    auto& ops = get_operations(tape);
    std::unordered_map<NodeId, TapeOperation*> by_node;
    for (auto& op : ops) by_node[op->node_id] = op.get();
    std::unordered_set<NodeId> live;
    std::vector<NodeId> stack;
    for (const auto& t : outputs)
        if (t.is_lazy()) stack.push_back(t.producer_node());
    while (!stack.empty()) {
        const NodeId n = stack.back();
        stack.pop_back();
        if (!live.insert(n).second) continue;
        auto it = by_node.find(n);
        if (it != by_node.end())
            for (NodeId in : it->second->input_nodes) stack.push_back(in);
    }
    const size_t before = ops.size();
    ops.erase(std::remove_if(ops.begin(), ops.end(), [&](const auto& op) { return !live.count(op->node_id); }),
              ops.end());
    rebuild_node_map(tape);
    return (int)(before - ops.size());
}

// ------------------------------------------------------------ fusion helpers
namespace {

struct TapeIndex {
    // consumers[(node, idx)] = tape positions reading that result
    std::map<std::pair<NodeId, uint16_t>, std::vector<size_t>> consumers;
    std::set<std::pair<NodeId, uint16_t>> outputs;
    std::unordered_map<NodeId, size_t> pos;
};

TapeIndex index_tape(const std::vector<std::unique_ptr<TapeOperation>>& ops, const std::vector<Tensor>& outputs) {
    TapeIndex ix;
    for (size_t i = 0; i < ops.size(); ++i) {
        ix.pos[ops[i]->node_id] = i;
        for (const auto& o : ops[i]->operands)
            if (o.lazy) ix.consumers[{o.node, o.index}].push_back(i);
    }
    for (const auto& t : outputs)
        if (t.is_lazy()) ix.outputs.insert({t.producer_node(), t.output_index()});
    return ix;
}

enum class Kind { OTHER, RELU, SIGMOID, ADD, MUL, REDUCE, MATMUL };

Kind kind_of(const TapeOperation& op) {
    if (op.plan) return Kind::OTHER;
    if (op.op_type == ReLUArgs::type_id()) return Kind::RELU;
    if (op.op_type == SigmoidArgs::type_id()) return Kind::SIGMOID;
    if (op.op_type == AddArgs::type_id()) return Kind::ADD;
    if (op.op_type == MultiplyArgs::type_id()) return Kind::MUL;
    if (op.op_type == ReduceArgs::type_id()) return Kind::REDUCE;
    if (op.op_type == MatMulArgs::type_id()) return Kind::MATMUL;
    return Kind::OTHER;
}

FusionPlan::MemberOp member_op(Kind k) {
    switch (k) {
        case Kind::RELU: return FusionPlan::RELU;
        case Kind::SIGMOID: return FusionPlan::SIGMOID;
        case Kind::ADD: return FusionPlan::ADD;
        case Kind::MUL: return FusionPlan::MUL;
        default: return FusionPlan::REDUCE;
    }
}

std::vector<uint32_t> out_shape(const TapeOperation& op) {
    return op.output_shapes.empty() ? std::vector<uint32_t>{} : op.output_shapes[0];
}

// A reduction can end a fused chain when its reduced dims are a prefix or a
// suffix of the input's dims (one kernel mode: over rows or over columns).
bool reduce_fusable(const std::vector<uint32_t>& in, const ReduceArgs& a) {
    if (a.type != ReduceArgs::Type::SUM && a.type != ReduceArgs::Type::MEAN) return false;
    const int r = (int)in.size();
    if (r == 0) return false;
    std::vector<bool> red((size_t)r, a.dims.empty());
    for (int32_t d : a.dims) {
        const int dd = d < 0 ? d + r : d;
        if (dd < 0 || dd >= r) return false;
        red[(size_t)dd] = true;
    }
    int first = -1, last = -1, count = 0;
    for (int i = 0; i < r; ++i)
        if (red[(size_t)i]) {
            if (first < 0) first = i;
            last = i;
            ++count;
        }
    if (count == 0) return false;
    if (last - first + 1 != count) return false;  // not contiguous
    return first == 0 || last == r - 1;
}

// Rebuilds the operation list with `fused` ops replacing their members.
// Emits in an order where every op follows the ops it reads (Kahn over the
// contracted graph, ties by original position).
// Returns false (and leaves `ops` untouched) when contracting the groups
// would create a cycle.
bool rebuild(std::vector<std::unique_ptr<TapeOperation>>& ops, std::vector<std::unique_ptr<TapeOperation>>& fused,
             const std::vector<int>& group_of) {
    const size_t n = ops.size();
    // units: original ops not in a group, and the fused ops
    struct Unit {
        TapeOperation* op;
        bool is_fused;
        size_t index;  // into ops or fused
        size_t first;
    };
    std::vector<Unit> units;
    std::vector<int> unit_of_group(fused.size(), -1);
    for (size_t i = 0; i < n; ++i) {
        if (group_of[i] >= 0) {
            int& u = unit_of_group[(size_t)group_of[i]];
            if (u < 0) {
                u = (int)units.size();
                units.push_back({fused[(size_t)group_of[i]].get(), true, (size_t)group_of[i], i});
            }
        } else {
            units.push_back({ops[i].get(), false, i, i});
        }
    }
    std::unordered_map<NodeId, int> unit_of_node;
    for (size_t u = 0; u < units.size(); ++u) {
        auto& op = *units[u].op;
        unit_of_node[op.node_id] = (int)u;
        for (NodeId o : op.output_nodes) unit_of_node[o] = (int)u;
        if (op.plan) {
            for (auto& m : op.plan->members) unit_of_node[m.node] = (int)u;
            for (const auto& seg : op.plan->seg_nodes)
                for (NodeId s : seg) unit_of_node[s] = (int)u;
            if (op.plan->has_matmul) unit_of_node[op.plan->matmul_node] = (int)u;
        }
    }
    std::vector<int> indeg(units.size(), 0);
    std::vector<std::vector<int>> users(units.size());
    for (size_t u = 0; u < units.size(); ++u) {
        std::set<int> deps;
        for (NodeId in : units[u].op->input_nodes) {
            auto it = unit_of_node.find(in);
            if (it != unit_of_node.end() && it->second != (int)u) deps.insert(it->second);
        }
        for (int d : deps) {
            users[(size_t)d].push_back((int)u);
            indeg[u]++;
        }
    }
    std::priority_queue<std::pair<size_t, int>, std::vector<std::pair<size_t, int>>, std::greater<>> ready;
    for (size_t u = 0; u < units.size(); ++u)
        if (indeg[u] == 0) ready.push({units[u].first, (int)u});
    std::vector<int> order;
    while (!ready.empty()) {
        const int u = ready.top().second;
        ready.pop();
        order.push_back(u);
        for (int v : users[(size_t)u])
            if (--indeg[(size_t)v] == 0) ready.push({units[(size_t)v].first, v});
    }
    if (order.size() != units.size()) return false;
    std::vector<std::unique_ptr<TapeOperation>> out;
    for (int u : order) {
        const Unit& un = units[(size_t)u];
        out.push_back(un.is_fused ? std::move(fused[un.index]) : std::move(ops[un.index]));
    }
    ops = std::move(out);
    return true;
}

// Lazy input nodes (dedup, order of first use) of a fused op's externals.
void set_inputs(TapeOperation& op, const FusionPlan& plan) {
    std::set<NodeId> seen;
    for (const auto& e : plan.externals) {
        if (e.lazy) {
            if (seen.insert(e.node).second) op.input_nodes.push_back(e.node);
        } else {
            op.constant_inputs.push_back(e.tensor);
        }
    }
    op.operands = plan.externals;
}

}  // namespace

// ------------------------------------------------------------- MLP fusion
// Pattern (rank-2): MatMul -> [Add(bias [1,N] or same-shape tensor)] ->
// [relu | sigmoid | Add | Multiply ...], every absorbed intermediate read by
// exactly the next op only and not requested as an output. The explicit
// FusedMLP op of the frontend is lowered the same way.
int MLPFusionPass::apply(Tape& tape, const std::vector<Tensor>& outputs) {
    auto& ops = get_operations(tape);
    const size_t n = ops.size();
    TapeIndex ix = index_tape(ops, outputs);
    std::vector<int> group_of(n, -1);
    std::vector<std::unique_ptr<TapeOperation>> fused;
    auto single_private_use = [&](NodeId node) -> long {
        auto it = ix.consumers.find({node, 0});
        if (it == ix.consumers.end() || it->second.size() != 1) return -1;
        if (ix.outputs.count({node, 0})) return -1;
        return (long)it->second[0];
    };
    for (size_t i = 0; i < n; ++i) {
        TapeOperation& mm = *ops[i];
        if (group_of[i] >= 0) continue;
        const bool explicit_mlp = !mm.plan && mm.op_type == FusedMLPArgs::type_id();
        if (kind_of(mm) != Kind::MATMUL && !explicit_mlp) continue;
        auto plan = std::make_shared<FusionPlan>();
        plan->has_matmul = true;
        plan->matmul_node = mm.node_id;
        plan->matmul_shape = out_shape(mm);
        plan->externals = {mm.operands[0], mm.operands[1]};
        NodeId last = mm.node_id;
        std::vector<size_t> absorbed = {i};
        if (explicit_mlp) {
            const Node* node = Context::instance().get_node(mm.node_id);
            const auto& a = node->as<FusedMLPArgs>();
            plan->matmul_node = 0;  // the explicit op is one node: its id names the final result
            FusionPlan::Member bias;
            bias.node = mm.node_id;
            bias.op = FusionPlan::ADD;
            bias.args = {FusionPlan::kProduct, -3};
            plan->externals.push_back(mm.operands[2]);
            bias.shape = out_shape(mm);
            const int act = a.activation >= 0 ? a.activation : (a.has_relu ? 1 : 0);
            if (act == 0) {
                plan->members.push_back(bias);
            } else {
                bias.node = 0;
                plan->members.push_back(bias);
                FusionPlan::Member m;
                m.node = mm.node_id;
                m.op = act == 1 ? FusionPlan::RELU : FusionPlan::SIGMOID;
                m.args = {0};
                m.shape = out_shape(mm);
                plan->members.push_back(m);
            }
        } else {
            plan->transpose_a = Context::instance().get_node(mm.node_id)->as<MatMulArgs>().transpose_a;
            plan->transpose_b = Context::instance().get_node(mm.node_id)->as<MatMulArgs>().transpose_b;
            // absorb the element-wise ops that follow
            for (;;) {
                const long nxt = single_private_use(last);
                if (nxt < 0 || group_of[(size_t)nxt] >= 0) break;
                TapeOperation& op = *ops[(size_t)nxt];
                const Kind k = kind_of(op);
                if (k != Kind::RELU && k != Kind::SIGMOID && k != Kind::ADD && k != Kind::MUL) break;
                if (out_shape(op) != plan->matmul_shape) break;
                FusionPlan::Member m;
                m.node = op.node_id;
                m.op = member_op(k);
                m.shape = out_shape(op);
                bool ok = true;
                for (const auto& o : op.operands) {
                    if (o.lazy && o.node == last) {
                        m.args.push_back(plan->members.empty() ? FusionPlan::kProduct : (int)plan->members.size() - 1);
                    } else {
                        // a second operand: bias [1,N] or a same-shape tensor, computed before the matmul
                        if (o.lazy) {
                            auto p = ix.pos.find(o.node);
                            if (p == ix.pos.end() || p->second > i) {
                                ok = false;
                                break;
                            }
                        }
                        plan->externals.push_back(o);
                        m.args.push_back(-(int)plan->externals.size());
                    }
                }
                if (!ok || plan->externals.size() > 2 + TTC_CHAIN_MAX_INPUTS) break;
                plan->members.push_back(m);
                absorbed.push_back((size_t)nxt);
                last = op.node_id;
            }
            if (plan->members.empty()) continue;  // a lone matmul stays a matmul
        }
        if (!plan->members.empty() && plan->members.back().node == 0) plan->members.back().node = last;
        plan->members.back().escapes = true;
        std::vector<uint32_t> out_shape_of_op = plan->matmul_shape;
        // A batch-dim (row) reduce_sum / reduce_mean that alone reads the
        // final value becomes the epilogue's column sum: the [M, N] value is
        // then never written to memory.
        const long red = single_private_use(last);
        if (red >= 0 && group_of[(size_t)red] < 0 && kind_of(*ops[(size_t)red]) == Kind::REDUCE &&
            plan->matmul_shape.size() == 2) {
            TapeOperation& rop = *ops[(size_t)red];
            const auto& ra = Context::instance().get_node(rop.node_id)->as<ReduceArgs>();
            const bool rows_only = ra.dims.size() == 1 && (ra.dims[0] == 0 || ra.dims[0] == -2);
            if (rows_only && (ra.type == ReduceArgs::Type::SUM || ra.type == ReduceArgs::Type::MEAN)) {
                plan->members.back().escapes = false;
                FusionPlan::Member r;
                r.node = rop.node_id;
                r.op = FusionPlan::REDUCE;
                r.args = {(int)plan->members.size() - 1};
                r.shape = out_shape(rop);
                r.dims.assign(ra.dims.begin(), ra.dims.end());
                r.keepdim = ra.keepdim;
                r.mean = ra.type == ReduceArgs::Type::MEAN;
                r.escapes = true;
                plan->members.push_back(r);
                absorbed.push_back((size_t)red);
                last = rop.node_id;
                out_shape_of_op = r.shape;
            }
        }
        auto op = std::make_unique<TapeOperation>(last, FusedGemmArgs::type_id());
        op->output_nodes = {last};
        op->output_shapes = {out_shape_of_op};
        set_inputs(*op, *plan);
        op->plan = plan;
        const int g = (int)fused.size();
        for (size_t a : absorbed) group_of[a] = g;
        fused.push_back(std::move(op));
    }
    if (fused.empty()) return 0;
    const int count = (int)fused.size();
    if (!rebuild(ops, fused, group_of)) return 0;  // would be cyclic: keep the unfused tape
    rebuild_node_map(tape);
    return count;
}

// --------------------------------------------------------- element-wise fusion
// Greedy grouping in tape order. An element-wise op joins the group(s) that
// produce its operands when shapes match and the contracted graph stays
// acyclic; an op reading two open groups merges them (union-find). A
// reduction whose dims are a prefix or suffix closes the group as its tail.
int EltwiseFusionPass::apply(Tape& tape, const std::vector<Tensor>& outputs) {
    auto& ops = get_operations(tape);
    const size_t n = ops.size();
    TapeIndex ix = index_tape(ops, outputs);
    std::vector<int> group_of(n, -1);
    struct Group {
        std::vector<size_t> members;
        std::vector<uint32_t> shape;
        std::set<std::pair<NodeId, uint16_t>> ext;  // distinct external lazy operands
        int n_const = 0;
        bool closed = false;  // a reduce ended it
    };
    std::vector<Group> groups;
    std::vector<int> parent;
    auto find = [&](int g) {
        while (parent[(size_t)g] != g) g = parent[(size_t)g] = parent[(size_t)parent[(size_t)g]];
        return g;
    };
    auto gof = [&](size_t pos) { return group_of[pos] < 0 ? -1 : find(group_of[pos]); };
    // groups each op depends on (raw ids; map through find), and groups each
    // group depends on through its external operands (transitive)
    std::vector<std::set<int>> dep_groups(n);
    std::vector<std::set<int>> gdeps;
    auto resolved = [&](const std::set<int>& s) {
        std::set<int> r;
        for (int g : s) r.insert(find(g));
        return r;
    };
    auto depends_on = [&](const std::set<int>& D, int g) {
        for (int d : resolved(D)) {
            if (d == g) return true;
            for (int e : resolved(gdeps[(size_t)d]))
                if (e == g) return true;
        }
        return false;
    };
    auto absorb_deps = [&](int g, const TapeOperation& op) {
        for (const auto& o : op.operands) {
            if (!o.lazy) continue;
            auto p = ix.pos.find(o.node);
            if (p == ix.pos.end()) continue;
            const int og = gof(p->second);
            if (og == g) continue;
            std::set<int> add = resolved(dep_groups[p->second]);
            if (og >= 0) add.insert(og);
            for (int d : std::set<int>(add)) {
                auto r = resolved(gdeps[(size_t)d]);
                add.insert(r.begin(), r.end());
            }
            add.erase(g);
            gdeps[(size_t)g].insert(add.begin(), add.end());
        }
    };
    auto ext_count = [&](const Group& G) { return (int)G.ext.size() + G.n_const; };
    for (size_t i = 0; i < n; ++i) {
        TapeOperation& op = *ops[i];
        for (const auto& o : op.operands) {
            if (!o.lazy) continue;
            auto p = ix.pos.find(o.node);
            if (p == ix.pos.end()) continue;
            const size_t j = p->second;
            dep_groups[i].insert(dep_groups[j].begin(), dep_groups[j].end());
            if (group_of[j] >= 0) dep_groups[i].insert(group_of[j]);
        }
        const Kind k = kind_of(op);
        const bool elt = k == Kind::RELU || k == Kind::SIGMOID || k == Kind::ADD || k == Kind::MUL;
        if (!elt && k != Kind::REDUCE) continue;
        // open groups producing this op's operands
        std::vector<int> cand;
        for (const auto& o : op.operands) {
            if (!o.lazy) continue;
            auto p = ix.pos.find(o.node);
            if (p == ix.pos.end()) continue;
            const int g = gof(p->second);
            if (g >= 0 && !groups[(size_t)g].closed && std::find(cand.begin(), cand.end(), g) == cand.end())
                cand.push_back(g);
        }
        // merge a second candidate group into the first when that is safe
        if (cand.size() == 2 && elt) {
            int g1 = cand[0], g2 = cand[1];
            Group &A = groups[(size_t)g1], &B = groups[(size_t)g2];
            const bool same = A.shape == B.shape && A.shape == out_shape(op);
            const bool independent = !resolved(gdeps[(size_t)g1]).count(g2) && !resolved(gdeps[(size_t)g2]).count(g1);
            std::set<std::pair<NodeId, uint16_t>> ext = A.ext;
            ext.insert(B.ext.begin(), B.ext.end());
            const bool small = A.members.size() + B.members.size() + 1 <= 12 &&
                               (int)ext.size() + A.n_const + B.n_const <= TTC_CHAIN_MAX_INPUTS;
            if (same && independent && small) {
                for (size_t m : B.members) A.members.push_back(m);
                std::sort(A.members.begin(), A.members.end());
                A.ext = ext;
                A.n_const += B.n_const;
                // members of either group are no longer external to the merged one
                for (size_t m : A.members) A.ext.erase({ops[m]->node_id, 0});
                gdeps[(size_t)g1].insert(gdeps[(size_t)g2].begin(), gdeps[(size_t)g2].end());
                B.members.clear();
                parent[(size_t)g2] = g1;
                gdeps[(size_t)g1].erase(g1);
                gdeps[(size_t)g1].erase(g2);
                cand = {g1};
            }
        }
        const int target = cand.empty() ? -1 : cand[0];
        auto joinable = [&](int g) {
            Group& G = groups[(size_t)g];
            if (k == Kind::REDUCE) {
                // the reduce must read the group's last member
                const size_t lastm = G.members.back();
                const auto& o = op.operands[0];
                if (!o.lazy || o.node != ops[lastm]->node_id) return false;
                const Node* node = Context::instance().get_node(op.node_id);
                if (!reduce_fusable(G.shape, node->as<ReduceArgs>())) return false;
            } else if (out_shape(op) != G.shape) {
                return false;
            }
            int new_ext = 0;
            for (const auto& o : op.operands) {
                if (!o.lazy) {
                    ++new_ext;
                    continue;
                }
                auto p = ix.pos.find(o.node);
                if (p != ix.pos.end() && gof(p->second) == g) continue;
                if (p != ix.pos.end()) {
                    // the operand must not depend on g, directly or through another group
                    if (depends_on(dep_groups[p->second], g)) return false;
                    const int og = gof(p->second);
                    if (og >= 0 && resolved(gdeps[(size_t)og]).count(g)) return false;
                }
                if (!G.ext.count({o.node, o.index})) ++new_ext;
            }
            if (ext_count(G) + new_ext > TTC_CHAIN_MAX_INPUTS) return false;
            if (G.members.size() + 1 > 12) return false;  // program length / slot budget
            return true;
        };
        if (target >= 0 && joinable(target)) {
            Group& G = groups[(size_t)target];
            G.members.push_back(i);
            for (const auto& o : op.operands) {
                if (!o.lazy) {
                    G.n_const++;
                    continue;
                }
                auto p = ix.pos.find(o.node);
                if (p != ix.pos.end() && gof(p->second) == target) continue;
                G.ext.insert({o.node, o.index});
            }
            if (k == Kind::REDUCE) G.closed = true;
            absorb_deps(target, op);
            group_of[i] = target;
            continue;
        }
        if (k == Kind::REDUCE) continue;  // a lone reduce runs as itself
        Group G;
        G.members.push_back(i);
        G.shape = out_shape(op);
        for (const auto& o : op.operands) {
            if (o.lazy)
                G.ext.insert({o.node, o.index});
            else
                G.n_const++;
        }
        const int ng = (int)groups.size();
        groups.push_back(G);
        gdeps.emplace_back();
        parent.push_back(ng);
        absorb_deps(ng, op);
        group_of[i] = ng;
    }
    for (auto& g : group_of)
        if (g >= 0) g = find(g);
    // Lower each group to a FusionPlan.
    std::vector<std::unique_ptr<TapeOperation>> fused;
    std::vector<int> gmap(groups.size(), -1);
    int fused_count = 0;
    for (size_t g = 0; g < groups.size(); ++g) {
        const Group& G = groups[g];
        if (G.members.empty()) continue;  // merged into another group
        auto plan = std::make_shared<FusionPlan>();
        std::unordered_map<NodeId, int> member_idx;
        std::map<std::pair<NodeId, uint16_t>, int> ext_idx;
        for (size_t mi = 0; mi < G.members.size(); ++mi) {
            const TapeOperation& op = *ops[G.members[mi]];
            FusionPlan::Member m;
            m.node = op.node_id;
            m.op = member_op(kind_of(op));
            m.shape = out_shape(op);
            if (m.op == FusionPlan::REDUCE) {
                const auto& a = Context::instance().get_node(op.node_id)->as<ReduceArgs>();
                m.dims.assign(a.dims.begin(), a.dims.end());
                m.keepdim = a.keepdim;
                m.mean = a.type == ReduceArgs::Type::MEAN;
            }
            for (const auto& o : op.operands) {
                if (o.lazy && member_idx.count(o.node)) {
                    m.args.push_back(member_idx[o.node]);
                } else if (o.lazy) {
                    auto key = std::make_pair(o.node, o.index);
                    if (!ext_idx.count(key)) {
                        ext_idx[key] = (int)plan->externals.size();
                        plan->externals.push_back(o);
                    }
                    m.args.push_back(-(ext_idx[key] + 1));
                } else {
                    plan->externals.push_back(o);
                    m.args.push_back(-(int)plan->externals.size());
                }
            }
            // escapes: read outside the group or requested
            bool esc = ix.outputs.count({op.node_id, 0}) > 0;
            auto cit = ix.consumers.find({op.node_id, 0});
            if (cit != ix.consumers.end())
                for (size_t c : cit->second)
                    if (group_of[c] != (int)g) esc = true;
            m.escapes = esc;
            member_idx[op.node_id] = (int)mi;
            plan->members.push_back(m);
        }
        const NodeId last = plan->members.back().node;
        auto op = std::make_unique<TapeOperation>(last, FusedChainArgs::type_id());
        for (const auto& m : plan->members)
            if (m.escapes) op->output_nodes.push_back(m.node);
        op->output_shapes = {plan->members.back().shape};
        set_inputs(*op, *plan);
        op->plan = plan;
        gmap[g] = (int)fused.size();
        fused.push_back(std::move(op));
        if (G.members.size() > 1) ++fused_count;
    }
    if (fused.empty()) return 0;
    for (auto& gi : group_of)
        if (gi >= 0) gi = gmap[(size_t)gi];
    if (!rebuild(ops, fused, group_of)) return 0;  // would be cyclic: keep the unfused tape
    rebuild_node_map(tape);
    return fused_count;
}

// ------------------------------------------------------------- segment fusion
int SegmentFusionPass::apply(Tape& tape, const std::vector<Tensor>& outputs) {
    (void)outputs;
    auto& ops = get_operations(tape);
    const size_t n = ops.size();
    auto is_split = [](NodeId id) {
        const Node* nd = Context::instance().get_node(id);
        return nd && nd->is<SplitArgs>();
    };
    // (signature, split node) -> [(chunk index, tape position)]
    std::map<std::pair<std::string, NodeId>, std::vector<std::pair<int, size_t>>> groups;
    for (size_t i = 0; i < n; ++i) {
        const TapeOperation& op = *ops[i];
        if (!op.plan || op.plan->has_matmul || op.plan->nseg != 1 || op.op_type != FusedChainArgs::type_id())
            continue;
        const FusionPlan& P = *op.plan;
        std::ostringstream sig;
        for (const auto& m : P.members) {
            sig << m.op << "(";
            for (int a : m.args) sig << a << ",";
            sig << ")" << m.escapes << m.keepdim << m.mean << "[";
            for (auto d : m.shape) sig << d << ",";
            sig << "]{";
            for (auto d : m.dims) sig << d << ",";
            sig << "};";
        }
        NodeId split = 0;
        int chunk = -1;
        bool ok = true;
        for (const auto& e : P.externals) {
            if (e.lazy && is_split(e.node)) {
                if (split == 0) {
                    split = e.node;
                    chunk = e.index;
                } else if (e.node != split || e.index != chunk) {
                    ok = false;  // every varying operand must read the same chunk
                    break;
                }
                // the chunk's own shape (a ragged last chunk differs)
                const auto& shapes = Context::instance().get_node(e.node)->output_shapes();
                sig << "S[";
                if (e.index < shapes.size())
                    for (auto d : shapes[e.index]) sig << d << ",";
                sig << "];";
            } else if (e.lazy) {
                sig << "L" << e.node << ":" << e.index << ";";
            } else {
                const void* id = e.tensor.host_data();
                if (!id && e.tensor.has_device()) id = e.tensor.device().ptr();
                if (!id) {
                    ok = false;
                    break;
                }
                sig << "C" << id << ":" << e.tensor.total_elements() << ";";
            }
        }
        if (!ok || split == 0) continue;
        groups[{sig.str(), split}].push_back({chunk, i});
    }
    std::vector<int> group_of(n, -1);
    std::vector<std::unique_ptr<TapeOperation>> fused;
    for (auto& [key, v] : groups) {
        std::sort(v.begin(), v.end());
        size_t a = 0;
        while (a < v.size()) {
            size_t b = a + 1;
            while (b < v.size() && v[b].first == v[b - 1].first + 1) ++b;
            if (b - a >= 2) {
                const TapeOperation& first = *ops[v[a].second];
                auto plan = std::make_shared<FusionPlan>(*first.plan);
                plan->nseg = (int)(b - a);
                plan->ext_seg_index.clear();
                for (const auto& e : plan->externals)
                    plan->ext_seg_index.push_back(e.lazy && e.node == key.second ? (int)e.index : -1);
                auto op = std::make_unique<TapeOperation>(ops[v[b - 1].second]->node_id, FusedChainArgs::type_id());
                for (size_t s = a; s < b; ++s) {
                    const TapeOperation& seg = *ops[v[s].second];
                    std::vector<NodeId> nodes;
                    for (const auto& m : seg.plan->members) nodes.push_back(m.node);
                    plan->seg_nodes.push_back(nodes);
                    for (NodeId o : seg.output_nodes) op->output_nodes.push_back(o);
                    group_of[v[s].second] = (int)fused.size();
                }
                op->output_shapes = first.output_shapes;
                op->input_nodes = first.input_nodes;
                op->constant_inputs = first.constant_inputs;
                // operands: every segment's chunk (keeps them alive until this op ran)
                op->operands = plan->externals;
                for (int s = 1; s < plan->nseg; ++s)
                    for (size_t k = 0; k < plan->externals.size(); ++k)
                        if (plan->ext_seg_index[k] >= 0) {
                            OperandRef r = plan->externals[k];
                            r.index = (uint16_t)(plan->ext_seg_index[k] + s);
                            op->operands.push_back(r);
                        }
                op->plan = plan;
                fused.push_back(std::move(op));
            }
            a = b;
        }
    }
    if (fused.empty()) return 0;
    const int count = (int)fused.size();
    if (!rebuild(ops, fused, group_of)) return 0;
    rebuild_node_map(tape);
    return count;
}
