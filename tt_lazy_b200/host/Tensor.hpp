// Tensor.hpp -- the unified lazy / materialized tensor of the tt_lazy front
// end (public interface of the reference's src/core/Tensor.hpp:17-131).
//
// Differences from the reference, all deliberate:
//  * lazy tensors keep the true rank of their op (the reference pads relu /
//    add / multiply / reduce outputs to rank 4, operations.cpp:125-135, which
//    later breaks broadcasting of a [N,M,1,1] result against a [1,M] bias);
//  * a tensor can be device-resident: evaluation results live in HBM
//    (DeviceView) and data_ptr() / to_vector() do the one device-to-host copy
//    (the memcpy of the reference's Tensor::eval_impl, Tensor.cpp:572);
//  * host storage of large tensors is pinned, so that copy runs at full
//    PCIe / C2C bandwidth.
#pragma once
#include <atomic>
#include <functional>
#include <memory>
#include <ostream>
#include <string>
#include <vector>

#include "common.hpp"

namespace tt_lazy {
class DeviceBuffer;  // MemoryManager.hpp
}

// A strided window of a device buffer (element units).
struct DeviceView {
    std::shared_ptr<tt_lazy::DeviceBuffer> buf;
    int64_t offset = 0;
    int64_t strides[4] = {0, 0, 0, 0};
    float* ptr() const;
    bool valid() const { return buf != nullptr; }
};

class Tensor {
   public:
    enum class State { LAZY, MATERIALIZED };

    Tensor();
    Tensor(NodeId producer_node_id, uint16_t output_index, std::initializer_list<uint32_t> shape);
    Tensor(NodeId producer_node_id, uint16_t output_index, const std::vector<uint32_t>& shape);
    Tensor(std::initializer_list<uint32_t> shape);
    Tensor(const std::vector<uint32_t>& shape);
    Tensor(const std::vector<uint32_t>& shape, const std::vector<float>& data);
    Tensor(void* data, std::initializer_list<uint32_t> shape);  // constant over caller memory
    Tensor(void* data, const std::vector<uint32_t>& shape);

    Tensor(const Tensor& other);
    Tensor(Tensor&& other) noexcept;
    Tensor& operator=(const Tensor& other);
    Tensor& operator=(Tensor&& other) noexcept;
    ~Tensor();

    State state() const { return state_; }
    bool is_lazy() const { return state_ == State::LAZY; }
    bool is_evaluated() const { return state_ == State::MATERIALIZED; }
    bool is_constant() const { return is_constant_; }
    bool is_null() const;
    explicit operator bool() const;

    NodeId producer_node() const;
    uint16_t output_index() const;

    const uint32_t* shape() const;
    uint16_t rank() const;
    uint32_t size(size_t dim) const;
    size_t total_elements() const;
    bool is_scalar() const;
    std::vector<uint32_t> shape_vector() const;

    // Data access (materialises a lazy tensor; a device-resident tensor is
    // copied to host memory once).
    float* data_ptr();
    const float* const_data_ptr() const;
    std::vector<float> to_vector() const;
    void eval();

    std::string to_string() const;
    void print_graph(std::ostream& os, int indent = 0) const;
    void print_graph(int indent = 0) const;

    struct GraphNode {
        NodeId id{};
        std::string op_name;
        std::vector<std::string> args;
        std::vector<GraphNode> inputs;
        int depth{};
    };
    static constexpr int DEFAULT_MAX_DEPTH = 10;
    GraphNode build_graph_node(int max_depth = DEFAULT_MAX_DEPTH) const;

    void fill(float value);
    void print() const;
    Tensor reshape(const std::vector<uint32_t>& new_shape) const;

    static std::vector<uint32_t> broadcast_shapes(const std::vector<uint32_t>& shape1,
                                                  const std::vector<uint32_t>& shape2);
    static bool can_broadcast(const std::vector<uint32_t>& shape1, const std::vector<uint32_t>& shape2);

    // ---- device residency (backend use) ----
    static Tensor on_device(const std::vector<uint32_t>& shape, DeviceView view);
    bool has_device() const { return device_.valid(); }
    const DeviceView& device() const { return device_; }
    // Host data pointer without triggering evaluation (constants and
    // materialized tensors; nullptr for lazy or device-only tensors).
    const float* host_data() const;
    // A constant whose caller-owned data changes between evaluations (a batch
    // of inputs): uploaded on every evaluation instead of cached like weights.
    void set_streamed(bool s) { streamed_ = s; }
    bool is_streamed() const { return streamed_; }

   private:
    State state_;
    NodeId producer_node_;
    uint16_t output_index_;
    uint16_t rank_;
    uint32_t shape_[4];
    std::shared_ptr<float> data_;  // host storage (pinned when large)
    size_t numel_;
    bool is_constant_;
    bool streamed_ = false;
    void* constant_data_;
    DeviceView device_;
    mutable std::atomic<bool> evaluation_in_progress_;

    void set_shape(const uint32_t* s, size_t rank);
    void allocate_data();
    void copy_from_device();
    void eval_impl() const;
    void assign(const Tensor& other, bool deep);
};

std::ostream& operator<<(std::ostream& os, const Tensor& tensor);
