// Tape.hpp -- the execution tape: a linear, topologically ordered list of
// operations (interfaces of the reference's src/tape/TapeOperation.hpp:9-27
// and src/tape/Tape.hpp:15-49).
//
// A TapeOperation keeps the reference fields (input_nodes for lazy inputs,
// constant_inputs for materialized ones) and adds what the B200 backend
// needs: every operand in argument order (the reference's split into two
// lists loses the order, so matmul(constant, lazy) swaps its operands), and
// the fusion plan of a fused operation.
#pragma once
#include <iostream>
#include <memory>
#include <unordered_map>
#include <vector>

#include "Tensor.hpp"
#include "common.hpp"

// An input of a tape operation: output `index` of lazy node `node`, or a
// constant / materialized tensor.
struct OperandRef {
    bool lazy = true;
    NodeId node = 0;
    uint16_t index = 0;
    Tensor tensor;
    static OperandRef of_node(NodeId n, uint16_t i) {
        OperandRef r;
        r.lazy = true;
        r.node = n;
        r.index = i;
        return r;
    }
    static OperandRef of_tensor(const Tensor& t) {
        OperandRef r;
        r.lazy = false;
        r.tensor = t;
        return r;
    }
};

// What a fused tape operation computes (built by MLPFusionPass and
// EltwiseFusionPass, lowered by the FusedChain / FusedMLP handlers).
struct FusionPlan {
    enum MemberOp { RELU, SIGMOID, ADD, MUL, REDUCE };
    struct Member {
        NodeId node = 0;
        MemberOp op = RELU;
        // operand sources: >= 0 member index; < 0 external -(k + 1)
        std::vector<int> args;
        bool escapes = false;  // result needed outside the fused op
        std::vector<uint32_t> shape;
        std::vector<int32_t> dims;  // REDUCE
        bool keepdim = false, mean = false;
    };
    // operand source meaning "the matmul product" (the epilogue's entry value)
    static constexpr int kProduct = -1000;
    bool has_matmul = false;  // externals 0 and 1 are the matmul operands
    NodeId matmul_node = 0;
    bool transpose_a = false, transpose_b = false;
    std::vector<uint32_t> matmul_shape;
    bool matmul_escapes = false;
    std::vector<Member> members;
    std::vector<OperandRef> externals;
    // Segmented chain (SegmentFusionPass): the same chain over `nseg`
    // consecutive chunks of one split. External k reads split output
    // ext_seg_index[k] + s in segment s (or is shared when -1); member m of
    // segment s is graph node seg_nodes[s][m].
    int nseg = 1;
    std::vector<int> ext_seg_index;
    std::vector<std::vector<NodeId>> seg_nodes;
    std::string describe() const;
};

struct TapeOperation {
    NodeId node_id;
    OpTypeId op_type;
    std::vector<NodeId> input_nodes;
    std::vector<Tensor> constant_inputs;
    std::vector<NodeId> output_nodes;
    std::vector<std::vector<uint32_t>> output_shapes;
    bool is_constant = false;
    bool is_evaluated = false;
    std::shared_ptr<Tensor> result;

    std::vector<OperandRef> operands;
    std::shared_ptr<const FusionPlan> plan;

    TapeOperation(NodeId node_id, OpTypeId op_type) : node_id(node_id), op_type(op_type) {}
};

class TapeOptimizationPass;
class TapeExecutor;

class Tape {
   public:
    Tape() = default;
    void add_operation(std::unique_ptr<TapeOperation> op);
    const std::vector<std::unique_ptr<TapeOperation>>& operations() const { return operations_; }

    friend class TapeOptimizationPass;
    friend class TapeGenerator;

    TapeOperation* find_operation(NodeId node_id);
    const TapeOperation* find_operation(NodeId node_id) const;
    std::vector<NodeId> get_dependencies(NodeId node_id) const;
    bool is_valid() const;
    void validate() const;
    void print_tape(std::ostream& os) const;
    void print_tape() const;
    size_t size() const { return operations_.size(); }

    // The tensors this tape was generated for (their results are kept).
    const std::vector<Tensor>& outputs() const { return outputs_; }
    void set_outputs(const std::vector<Tensor>& o) { outputs_ = o; }
    // Op that produces lazy node `id` (a fused op answers for every node it
    // absorbed).
    TapeOperation* producer_of(NodeId id);

   private:
    std::vector<std::unique_ptr<TapeOperation>> operations_;
    std::unordered_map<NodeId, TapeOperation*> node_to_op_;
    std::vector<Tensor> outputs_;
    void build_node_map();
};

// -------------------------------------------------------------- generator
class TapeGenerator {
   public:
    TapeGenerator() : optimization_enabled_(true) {}
    std::unique_ptr<Tape> generate_tape(const std::vector<Tensor>& outputs);
    std::unique_ptr<Tape> generate_tape(const Tensor& output);
    void set_optimization_enabled(bool enabled) { optimization_enabled_ = enabled; }
    bool is_optimization_enabled() const { return optimization_enabled_; }

    static void register_optimization_pass(std::unique_ptr<TapeOptimizationPass> pass);
    static void register_default_passes();
    static void clear_passes();

   private:
    std::vector<NodeId> collect_dependencies(const std::vector<Tensor>& outputs);
    std::vector<NodeId> topological_sort(const std::vector<NodeId>& nodes);
    std::unique_ptr<TapeOperation> create_tape_operation(const Node& node);
    bool optimization_enabled_ = false;
    static std::vector<std::unique_ptr<TapeOptimizationPass>>& passes();
    static bool default_passes_registered_;
};

// ------------------------------------------------------------------ passes
class TapeOptimizationPass {
   public:
    virtual ~TapeOptimizationPass() = default;
    TapeOptimizationPass(const TapeOptimizationPass&) = delete;
    TapeOptimizationPass& operator=(const TapeOptimizationPass&) = delete;
    virtual int apply(Tape& tape, const std::vector<Tensor>& outputs) = 0;
    virtual std::string name() const = 0;
    static constexpr int DEFAULT_PRIORITY = 100;
    virtual int priority() const { return DEFAULT_PRIORITY; }

   protected:
    TapeOptimizationPass() = default;
    std::vector<std::unique_ptr<TapeOperation>>& get_operations(Tape& tape) { return tape.operations_; }
    void rebuild_node_map(Tape& tape) { tape.build_node_map(); }
};

// Drops operations unreachable from the outputs (reference:
// src/tape/passes/DeadCodeEliminationPass.cpp:12-58, priority 10).
class DeadCodeEliminationPass : public TapeOptimizationPass {
   public:
    int apply(Tape& tape, const std::vector<Tensor>& outputs) override;
    std::string name() const override { return "DeadCodeElimination"; }
    static constexpr int EARLY_PRIORITY = 10;
    int priority() const override { return EARLY_PRIORITY; }
};

// MatMul [+ bias] [-> relu | sigmoid ...] -> one GEMM with the bias and
// activations in its epilogue (reference: src/tape/passes/MLPFusionPass.cpp,
// disabled there at :101-103; here enabled, and the fused op answers for the
// node id of the last op it absorbs so get_result() keeps working).
class MLPFusionPass : public TapeOptimizationPass {
   public:
    int apply(Tape& tape, const std::vector<Tensor>& outputs) override;
    std::string name() const override { return "MLPFusion"; }
    static constexpr int MLP_FUSION_PRIORITY = 50;
    int priority() const override { return MLP_FUSION_PRIORITY; }
};

// Groups relu / sigmoid / add / multiply operations over the same element
// space (with an optional tail reduce_sum / reduce_mean) into one fused
// chain operation: one kernel, intermediates in registers. No reference
// counterpart (its README's "single fused kernel" claim, README.md:92).
class EltwiseFusionPass : public TapeOptimizationPass {
   public:
    int apply(Tape& tape, const std::vector<Tensor>& outputs) override;
    std::string name() const override { return "EltwiseFusion"; }
    static constexpr int ELTWISE_FUSION_PRIORITY = 60;
    int priority() const override { return ELTWISE_FUSION_PRIORITY; }
};

// Merges fused chains that run the same program on consecutive chunks of
// one split (e.g. a per-chunk chain after transpose -> split) into one
// segmented chain: one kernel launch over all chunks instead of one each.
class SegmentFusionPass : public TapeOptimizationPass {
   public:
    int apply(Tape& tape, const std::vector<Tensor>& outputs) override;
    std::string name() const override { return "SegmentFusion"; }
    static constexpr int SEGMENT_FUSION_PRIORITY = 70;
    int priority() const override { return SEGMENT_FUSION_PRIORITY; }
};

// Internal op types of fused tape operations.
DEFINE_OP_ARGS(FusedChain, );
DEFINE_OP_ARGS(FusedGemm, );
