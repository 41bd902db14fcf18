// Node.hpp / Context.hpp -- graph nodes and the global graph store
// (interfaces of the reference's src/core/Node.hpp:7-90 and
// src/core/Context.hpp:12-95).
//
// A Node owns its typed arguments through a shared pointer instead of the
// reference's 256-byte placement-new buffer (Node.hpp:87-88), so argument
// objects with heap members (FusedMLPArgs::fusion_info) are destroyed
// correctly; is<T>() / as<T>() / try_as<T>() behave the same.
#pragma once
#include <memory>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "Tensor.hpp"
#include "common.hpp"

class Node {
   public:
    template <typename ArgsT, size_t N>
    Node(NodeId id, const SmallVector<Tensor, N>& inputs, ArgsT&& args)
        : id_(id),
          type_id_(detail::get_op_id<std::decay_t<ArgsT>>()),
          inputs_(inputs.begin(), inputs.end()),
          args_(std::make_shared<std::decay_t<ArgsT>>(std::forward<ArgsT>(args))) {}

    NodeId id() const { return id_; }
    OpTypeId type_id() const { return type_id_; }

    template <typename T>
    bool is() const {
        return type_id_ == detail::get_op_id<T>();
    }
    template <typename T>
    const T& as() const {
        assert(is<T>());
        return *static_cast<const T*>(args_.get());
    }
    template <typename T>
    T& as() {
        assert(is<T>());
        return *static_cast<T*>(args_.get());
    }
    template <typename T>
    const T* try_as() const {
        return is<T>() ? static_cast<const T*>(args_.get()) : nullptr;
    }
    template <typename T>
    T* try_as() {
        return is<T>() ? static_cast<T*>(args_.get()) : nullptr;
    }

    OpArgsBase* args_base() { return args_.get(); }
    const OpArgsBase* args_base() const { return args_.get(); }
    std::string_view op_name() const { return args_->op_name(); }

    const SmallVector<Tensor, 4>& inputs() const { return inputs_; }
    const SmallVector<NodeId, 2>& output_nodes() const { return output_nodes_; }
    void add_output_node(NodeId node_id) { output_nodes_.push_back(node_id); }

    // Shapes of this node's outputs (one per output index), recorded by the
    // frontend op that created it. The reference leaves tape output shapes as
    // a dummy {1,1,1,1} (TapeGenerator.cpp:175-177); the B200 backend sizes
    // device buffers from these.
    const std::vector<std::vector<uint32_t>>& output_shapes() const { return output_shapes_; }
    void set_output_shapes(std::vector<std::vector<uint32_t>> s) { output_shapes_ = std::move(s); }

   private:
    NodeId id_;
    OpTypeId type_id_;
    SmallVector<Tensor, 4> inputs_;
    SmallVector<NodeId, 2> output_nodes_;
    std::shared_ptr<OpArgsBase> args_;
    std::vector<std::vector<uint32_t>> output_shapes_;
};

class Context {
   public:
    Context();

    Node* get_node(NodeId id);
    const Node* get_node(NodeId id) const;
    const std::vector<Node>& get_all_nodes() const { return nodes_; }
    std::vector<Node>& get_all_nodes() { return nodes_; }

    std::unordered_set<NodeId> get_dependencies(const std::vector<Tensor>& outputs) const;
    std::vector<NodeId> topological_sort(const std::unordered_set<NodeId>& node_set) const;

    size_t size() const { return nodes_.size(); }
    // Drops every node. Also advances epoch(), which invalidates evaluation
    // caches keyed by node id (ids restart at 1 after a clear).
    void clear();
    uint64_t epoch() const { return epoch_; }

    void print_stats() const;
    static Context& instance();

    template <typename ArgsT, size_t N>
    NodeId create_node(const SmallVector<Tensor, N>& inputs, ArgsT&& args) {
        NodeId id = next_id_++;
        id_to_index_[id] = nodes_.size();
        nodes_.emplace_back(id, inputs, std::forward<ArgsT>(args));
        for (const auto& input : inputs) {
            if (!input.is_constant() && input.is_lazy() && input.producer_node() != 0) {
                if (Node* producer = get_node(input.producer_node())) producer->add_output_node(id);
            }
        }
        return id;
    }

    template <typename ArgsT>
    std::vector<const Node*> find_nodes() const {
        std::vector<const Node*> result;
        const OpTypeId target = detail::get_op_id<ArgsT>();
        for (const auto& node : nodes_)
            if (node.type_id() == target) result.push_back(&node);
        return result;
    }

   private:
    std::vector<Node> nodes_;
    std::unordered_map<NodeId, size_t> id_to_index_;
    NodeId next_id_ = 1;
    uint64_t epoch_ = 1;
};
