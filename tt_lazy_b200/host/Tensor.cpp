// Tensor.cpp -- see Tensor.hpp. Graph printing, broadcasting and reshape
// follow the reference's behaviour (src/core/Tensor.cpp); storage and
// materialisation are the B200 backend's.
#include "Tensor.hpp"

#include <algorithm>
#include <cstring>
#include <sstream>
#include <stdexcept>

#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "tt_cuda.h"

float* DeviceView::ptr() const { return buf ? buf->ptr() + offset : nullptr; }

Tensor::Tensor()
    : state_(State::LAZY),
      producer_node_(0),
      output_index_(0),
      rank_(0),
      shape_{1, 1, 1, 1},
      numel_(0),
      is_constant_(false),
      constant_data_(nullptr),
      evaluation_in_progress_(false) {}

void Tensor::set_shape(const uint32_t* s, size_t rank) {
    if (rank > 4) throw std::runtime_error("Tensor rank must be <= 4");
    rank_ = (uint16_t)rank;
    for (int i = 0; i < 4; ++i) shape_[i] = i < (int)rank ? s[i] : 1;
    numel_ = 1;
    for (size_t i = 0; i < rank; ++i) numel_ *= shape_[i];
}

Tensor::Tensor(NodeId id, uint16_t idx, std::initializer_list<uint32_t> shape) : Tensor() {
    producer_node_ = id;
    output_index_ = idx;
    set_shape(shape.begin(), shape.size());
}

Tensor::Tensor(NodeId id, uint16_t idx, const std::vector<uint32_t>& shape) : Tensor() {
    producer_node_ = id;
    output_index_ = idx;
    set_shape(shape.data(), shape.size());
}

Tensor::Tensor(std::initializer_list<uint32_t> shape) : Tensor() {
    state_ = State::MATERIALIZED;
    set_shape(shape.begin(), shape.size());
    allocate_data();
}

Tensor::Tensor(const std::vector<uint32_t>& shape) : Tensor() {
    state_ = State::MATERIALIZED;
    set_shape(shape.data(), shape.size());
    allocate_data();
}

Tensor::Tensor(const std::vector<uint32_t>& shape, const std::vector<float>& data) : Tensor(shape) {
    if (data.size() != numel_) throw std::runtime_error("Tensor data size does not match its shape");
    std::copy(data.begin(), data.end(), data_.get());
}

Tensor::Tensor(void* data, std::initializer_list<uint32_t> shape) : Tensor() {
    state_ = State::MATERIALIZED;
    is_constant_ = true;
    constant_data_ = data;
    set_shape(shape.begin(), shape.size());
}

Tensor::Tensor(void* data, const std::vector<uint32_t>& shape) : Tensor() {
    state_ = State::MATERIALIZED;
    is_constant_ = true;
    constant_data_ = data;
    set_shape(shape.data(), shape.size());
}

void Tensor::assign(const Tensor& o, bool deep) {
    state_ = o.state_;
    producer_node_ = o.producer_node_;
    output_index_ = o.output_index_;
    rank_ = o.rank_;
    std::copy(o.shape_, o.shape_ + 4, shape_);
    numel_ = o.numel_;
    is_constant_ = o.is_constant_;
    streamed_ = o.streamed_;
    constant_data_ = o.constant_data_;
    device_ = o.device_;
    if (deep && o.data_) {
        // Materialized data is copied, as in the reference (Tensor.cpp:586-601):
        // a node keeps the values its inputs had when the graph was built.
        data_ = tt_lazy::MemoryManager::host_buffer(numel_);
        std::memcpy(data_.get(), o.data_.get(), numel_ * sizeof(float));
    } else {
        data_ = o.data_;
    }
}

Tensor::Tensor(const Tensor& o) : Tensor() { assign(o, true); }
Tensor::Tensor(Tensor&& o) noexcept : Tensor() {
    assign(o, false);
    o = Tensor();
}
Tensor& Tensor::operator=(const Tensor& o) {
    if (this != &o) assign(o, true);
    return *this;
}
Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this != &o) {
        assign(o, false);
        o.state_ = State::LAZY;
        o.producer_node_ = 0;
        o.output_index_ = 0;
        o.rank_ = 0;
        o.numel_ = 0;
        o.is_constant_ = false;
        o.constant_data_ = nullptr;
        o.data_.reset();
        o.device_ = DeviceView();
        std::fill(o.shape_, o.shape_ + 4, 1);
    }
    return *this;
}
Tensor::~Tensor() = default;

bool Tensor::is_null() const { return state_ == State::LAZY && producer_node_ == 0; }
Tensor::operator bool() const { return !is_null(); }
NodeId Tensor::producer_node() const { return producer_node_; }
uint16_t Tensor::output_index() const { return output_index_; }
const uint32_t* Tensor::shape() const { return shape_; }
uint16_t Tensor::rank() const { return rank_; }
uint32_t Tensor::size(size_t dim) const { return dim < rank_ ? shape_[dim] : 1; }
size_t Tensor::total_elements() const { return numel_; }
bool Tensor::is_scalar() const { return numel_ == 1; }
std::vector<uint32_t> Tensor::shape_vector() const { return std::vector<uint32_t>(shape_, shape_ + rank_); }

Tensor Tensor::on_device(const std::vector<uint32_t>& shape, DeviceView view) {
    Tensor t;
    t.state_ = State::MATERIALIZED;
    t.set_shape(shape.data(), shape.size());
    t.device_ = std::move(view);
    return t;
}

const float* Tensor::host_data() const {
    if (is_constant_) return static_cast<const float*>(constant_data_);
    return data_.get();
}

void Tensor::allocate_data() {
    if (numel_ > 0) data_ = tt_lazy::MemoryManager::host_buffer(numel_);
}

// The single device-to-host copy of a materialised result. A strided view
// (e.g. a transposed result) is copied contiguous on the device first.
void Tensor::copy_from_device() {
    if (!device_.valid() || data_) return;
    allocate_data();
    if (numel_ == 0) return;
    const int r = rank_;
    bool contiguous = true;
    int64_t expect = 1;
    for (int i = r - 1; i >= 0; --i) {
        if (shape_[i] != 1 && device_.strides[i] != expect) contiguous = false;
        expect *= shape_[i];
    }
    if (contiguous) {
        if (ttc_memcpy_d2h(data_.get(), device_.ptr(), numel_ * sizeof(float)) != TTC_OK)
            throw std::runtime_error(ttc_last_error());
        return;
    }
    // strided view (transpose / split chunk): densify on the device, then one copy
    const DeviceView dense = tt_lazy::dense_view(device_, shape_vector());
    if (ttc_memcpy_d2h(data_.get(), dense.ptr(), numel_ * sizeof(float)) != TTC_OK)
        throw std::runtime_error(ttc_last_error());
}

float* Tensor::data_ptr() {
    if (state_ == State::LAZY) eval();
    if (is_constant_) return static_cast<float*>(constant_data_);
    if (!data_ && device_.valid()) copy_from_device();
    return data_.get();
}

const float* Tensor::const_data_ptr() const { return const_cast<Tensor*>(this)->data_ptr(); }

std::vector<float> Tensor::to_vector() const {
    const float* d = const_data_ptr();
    if (!d) return {};
    return std::vector<float>(d, d + numel_);
}

void Tensor::eval() {
    if (state_ == State::MATERIALIZED) return;
    eval_impl();
}

void Tensor::eval_impl() const {
    if (state_ == State::MATERIALIZED || evaluation_in_progress_.load()) return;
    evaluation_in_progress_.store(true);
    try {
        auto evaluated = tt_lazy::get_evaluation_manager().evaluate(*this);
        if (!evaluated) throw std::runtime_error("Failed to evaluate tensor");
        if (evaluated->total_elements() != numel_)
            throw std::runtime_error("evaluated result has " + std::to_string(evaluated->total_elements()) +
                                     " elements, the lazy tensor expects " + std::to_string(numel_));
        Tensor* self = const_cast<Tensor*>(this);
        self->state_ = State::MATERIALIZED;
        self->device_ = evaluated->device_;
        if (!device_.valid() && evaluated->host_data()) {
            self->allocate_data();
            std::memcpy(self->data_.get(), evaluated->host_data(), numel_ * sizeof(float));
        } else {
            self->copy_from_device();
        }
    } catch (...) {
        evaluation_in_progress_.store(false);
        throw;
    }
    evaluation_in_progress_.store(false);
}

static std::string shape_str(const uint32_t* s, int rank) {
    std::ostringstream o;
    o << "shape=[";
    for (int i = 0; i < rank; ++i) o << (i ? ", " : "") << s[i];
    o << "]";
    return o.str();
}

Tensor::GraphNode Tensor::build_graph_node(int max_depth) const {
    GraphNode node;
    if (is_constant()) {
        node.op_name = "CONSTANT";
        node.args.push_back(shape_str(shape_, rank_));
        return node;
    }
    if (is_null()) {
        node.op_name = "NULL";
        return node;
    }
    if (state_ == State::MATERIALIZED) {
        node.op_name = "MATERIALIZED";
        node.args.push_back(shape_str(shape_, rank_));
        return node;
    }
    const Node* producer = Context::instance().get_node(producer_node_);
    node.id = producer_node_;
    if (!producer) {
        node.op_name = "UNKNOWN";
        return node;
    }
    node.op_name = std::string(producer->op_name());
    node.args.push_back("type_id=" + std::to_string(producer->type_id()));
    node.args.push_back(shape_str(shape_, rank_));
    if (max_depth > 0) {
        for (const auto& input : producer->inputs()) {
            if (input.is_constant() || input.is_null()) continue;
            GraphNode child = input.build_graph_node(max_depth - 1);
            child.depth = node.depth + 1;
            node.inputs.push_back(child);
        }
    }
    return node;
}

std::string Tensor::to_string() const {
    std::ostringstream oss;
    print_graph(oss, 0);
    return oss.str();
}

void Tensor::print_graph(std::ostream& os, int indent) const {
    std::function<void(const GraphNode&, int)> rec = [&](const GraphNode& n, int ind) {
        os << std::string((size_t)ind * 2, ' ') << "[" << n.id << "] " << n.op_name;
        if (!n.args.empty()) {
            os << "(";
            for (size_t i = 0; i < n.args.size(); ++i) os << (i ? ", " : "") << n.args[i];
            os << ")";
        }
        os << "\n";
        for (const auto& c : n.inputs) rec(c, ind + 1);
    };
    rec(build_graph_node(), indent);
}

void Tensor::print_graph(int indent) const { print_graph(std::cout, indent); }

void Tensor::fill(float value) {
    float* d = data_ptr();
    if (d) std::fill(d, d + numel_, value);
}

void Tensor::print() const {
    if (state_ == State::LAZY) {
        print_graph();
        return;
    }
    const float* d = const_data_ptr();
    std::cout << "Tensor " << shape_str(shape_, rank_) << "\n";
    if (!d) return;
    if (numel_ <= 16) {
        std::cout << "Data: [";
        for (size_t i = 0; i < numel_; ++i) std::cout << (i ? ", " : "") << d[i];
        std::cout << "]\n";
    } else {
        std::cout << "Data: [too large to display]\n";
    }
}

Tensor Tensor::reshape(const std::vector<uint32_t>& new_shape) const {
    size_t n = 1;
    for (uint32_t d : new_shape) n *= d;
    if (n != numel_) throw std::runtime_error("Reshape: total elements mismatch");
    Tensor r = *this;
    r.set_shape(new_shape.data(), new_shape.size());
    if (r.device_.valid()) {
        int64_t s = 1;
        for (int i = (int)new_shape.size() - 1; i >= 0; --i) {
            r.device_.strides[i] = s;
            s *= new_shape[i];
        }
    }
    return r;
}

std::vector<uint32_t> Tensor::broadcast_shapes(const std::vector<uint32_t>& a, const std::vector<uint32_t>& b) {
    const size_t r = std::max(a.size(), b.size());
    std::vector<uint32_t> out(r);
    for (size_t i = 0; i < r; ++i) {
        const uint32_t da = i < a.size() ? a[a.size() - 1 - i] : 1;
        const uint32_t db = i < b.size() ? b[b.size() - 1 - i] : 1;
        if (da != db && da != 1 && db != 1) throw std::runtime_error("Incompatible shapes for broadcasting");
        out[r - 1 - i] = std::max(da, db);
    }
    return out;
}

bool Tensor::can_broadcast(const std::vector<uint32_t>& a, const std::vector<uint32_t>& b) {
    try {
        broadcast_shapes(a, b);
        return true;
    } catch (...) {
        return false;
    }
}

std::ostream& operator<<(std::ostream& os, const Tensor& t) {
    t.print_graph(os, 0);
    return os;
}
