// Executor.cpp -- tape execution on the B200 backend: the memory manager,
// constant uploads, the operation handlers (lowering every tape operation,
// fused or not, to tt_cuda C-ABI calls) and the evaluation manager.
//
// The handlers replace the reference's src/tape/OperationHandlers.cpp, which
// gathered host tensors and called namespace math. Here every result stays
// in device memory as a DeviceView; transpose and split produce views (no
// copy), and a view is folded into its consumer's strides (a transposed
// matmul operand becomes the GEMM's transpose flag, a transposed chain input
// flips the chain's iteration order). Errors from the backend come back as
// std::runtime_error with the backend's message, as the reference's math
// functions threw.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <stdexcept>
#include <tuple>

#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "operations.hpp"
#include "tt_cuda.h"

namespace tt_lazy {

namespace {
bool g_ready = false;

void check(int rc) {
    if (rc != TTC_OK) throw std::runtime_error(ttc_last_error());
}
}  // namespace

void backend_init() {
    if (g_ready) return;
    int device = 0;
    if (const char* e = getenv("TT_LAZY_DEVICE"))
        device = atoi(e);
    else if (const char* l = getenv("LOCAL_RANK"))
        device = atoi(l);
    int count = 0;
    if (ttc_device_count(&count) != TTC_OK || count == 0)
        throw std::runtime_error(std::string("tt_lazy: no CUDA device available for the B200 backend: ") +
                                 ttc_last_error());
    if (device >= count) device = device % count;
    check(ttc_init(device));
    g_ready = true;
}

bool backend_ready() { return g_ready; }

namespace {
int g_gemm_path = -1;  // -1: from TT_LAZY_GEMM on first use
}
void set_gemm_path(int path) { g_gemm_path = path; }
int get_gemm_path() { return g_gemm_path; }

// ------------------------------------------------------------ memory manager
DeviceBuffer::~DeviceBuffer() { MemoryManager::instance().release(ptr_, bytes_); }

MemoryManager& MemoryManager::instance() {
    static MemoryManager* m = new MemoryManager();  // never destroyed: buffers may outlive statics
    return *m;
}

static size_t bucket(size_t bytes) {
    if (bytes <= (1u << 20)) return (bytes + 255) & ~(size_t)255;
    return (bytes + (2u << 20) - 1) & ~((size_t)(2u << 20) - 1);
}

namespace {
// 256-byte guard pattern written after a buffer in canary mode
const unsigned char* canary_pattern() {
    static unsigned char p[256];
    static bool init = [] {
        for (int i = 0; i < 256; ++i) p[i] = (unsigned char)(0xA5 ^ i);
        return true;
    }();
    (void)init;
    return p;
}
}  // namespace

bool MemoryManager::canaries() {
    if (canaries_ < 0) {
        const char* e = getenv("TT_LAZY_CANARY");
        canaries_ = (e && e[0] == '1') ? 1 : 0;
    }
    return canaries_ == 1;
}

bool MemoryManager::band_intact(float* ptr, size_t bytes) {
    unsigned char h[256];
    if (ttc_memcpy_d2h(h, (const char*)ptr + bytes - 256, 256) != TTC_OK) return false;
    return std::memcmp(h, canary_pattern(), 256) == 0;
}

std::vector<std::string> MemoryManager::check_canaries(const std::string& where) {
    std::vector<std::string> out = std::move(violations_);
    violations_.clear();
    for (const auto& [ptr, bytes] : guarded_)
        if (!band_intact(ptr, bytes))
            out.push_back("guard band of the " + std::to_string(bytes - 256) + "-byte buffer at " +
                          std::to_string((uintptr_t)ptr) + " overwritten (" + where + ")");
    return out;
}

long long MemoryManager::canary_offset(const float* ptr) const {
    auto it = guarded_.find(const_cast<float*>(ptr));
    return it == guarded_.end() ? -1 : (long long)it->second - 256;
}

std::shared_ptr<DeviceBuffer> MemoryManager::allocate(size_t bytes) {
    backend_init();
    const bool guard = canaries();
    const size_t b = bucket(std::max<size_t>(bytes, 4) + (guard ? 256 : 0));
    float* p = nullptr;
    auto& fl = free_[b];
    if (!fl.empty()) {
        p = fl.back();
        fl.pop_back();
        stats_.reuses++;
        stats_.bytes_cached -= b;
    } else {
        void* d = nullptr;
        if (ttc_malloc(b, &d) != TTC_OK) {
            trim();  // give cached blocks back and retry once
            check(ttc_malloc(b, &d));
        }
        p = static_cast<float*>(d);
    }
    stats_.allocations++;
    stats_.bytes_live += b;
    stats_.bytes_peak = std::max(stats_.bytes_peak, stats_.bytes_live);
    if (recording_) recorded_.emplace_back(p, b);
    if (guard) {  // the band is the bucket's last 256 bytes: past every request of this bucket
        check(ttc_memcpy_h2d((char*)p + b - 256, canary_pattern(), 256));
        guarded_[p] = b;
    } else {
        guarded_.erase(p);
    }
    return std::make_shared<DeviceBuffer>(p, b);
}

std::shared_ptr<DeviceBuffer> MemoryManager::claim(float* ptr, size_t bytes) {
    auto it = free_.find(bytes);
    if (it == free_.end()) return nullptr;
    auto& v = it->second;
    auto pos = std::find(v.begin(), v.end(), ptr);
    if (pos == v.end()) return nullptr;
    v.erase(pos);
    stats_.bytes_cached -= bytes;
    stats_.bytes_live += bytes;
    return std::make_shared<DeviceBuffer>(ptr, bytes);
}

void MemoryManager::release(float* ptr, size_t bytes) {
    if (!ptr) return;
    auto g = guarded_.find(ptr);
    if (g != guarded_.end()) {  // (runs from a destructor: report later, never throw)
        if (!band_intact(ptr, bytes))
            violations_.push_back("guard band of a released " + std::to_string(bytes - 256) +
                                  "-byte buffer overwritten");
        guarded_.erase(g);
    }
    free_[bytes].push_back(ptr);
    stats_.bytes_live -= bytes;
    stats_.bytes_cached += bytes;
}

void MemoryManager::trim() {
    for (auto& [b, v] : free_) {
        for (float* p : v) ttc_free(p);
        stats_.bytes_cached -= b * v.size();
        v.clear();
    }
}

std::shared_ptr<float> MemoryManager::host_buffer(size_t n) {
    const size_t bytes = std::max<size_t>(n, 1) * sizeof(float);
    if (g_ready && bytes >= (1u << 20)) {
        void* h = nullptr;
        if (ttc_host_alloc(bytes, &h) == TTC_OK) {
            std::memset(h, 0, bytes);
            return std::shared_ptr<float>(static_cast<float*>(h), [](float* p) { ttc_host_free(p); });
        }
    }
    return std::shared_ptr<float>(new float[std::max<size_t>(n, 1)](), std::default_delete<float[]>());
}

// ------------------------------------------------------------ constant cache
namespace {
std::map<std::pair<const void*, size_t>, DeviceView>& constant_cache() {
    static auto* c = new std::map<std::pair<const void*, size_t>, DeviceView>();
    return *c;
}

void set_contiguous_strides(DeviceView& v, const std::vector<uint32_t>& shape) {
    int64_t s = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        v.strides[i] = s;
        s *= shape[(size_t)i];
    }
}
}  // namespace

// Streamed inputs whose upload a pipelined plan started on the copy stream:
// (host pointer, elements) -> (device view, prefetch ticket).
std::map<std::pair<const void*, size_t>, std::pair<DeviceView, int>>& prefetched() {
    static auto* m = new std::map<std::pair<const void*, size_t>, std::pair<DeviceView, int>>();
    return *m;
}

DeviceView upload(const Tensor& t) {
    if (t.has_device()) return t.device();
    const float* host = t.host_data();
    if (!host) throw std::runtime_error("tt_lazy: input tensor has no data");
    const size_t n = t.total_elements();
    if (t.is_streamed()) {
        auto it = prefetched().find(std::make_pair((const void*)host, n));
        if (it != prefetched().end()) {  // kernels from here on wait for that copy
            check(ttc_wait_ticket(it->second.second));
            return it->second.first;
        }
    }
    const bool cached = t.is_constant() && !t.is_streamed();
    if (cached) {
        auto key = std::make_pair((const void*)host, n);
        auto it = constant_cache().find(key);
        if (it != constant_cache().end()) return it->second;
    }
    DeviceView v;
    v.buf = MemoryManager::instance().allocate(n * sizeof(float));
    set_contiguous_strides(v, t.shape_vector());
    check(ttc_memcpy_h2d(v.buf->ptr(), host, n * sizeof(float)));
    if (cached) constant_cache()[std::make_pair((const void*)host, n)] = v;
    return v;
}

void clear_constant_cache() { constant_cache().clear(); }

}  // namespace tt_lazy

using tt_lazy::DeviceBuffer;
using tt_lazy::MemoryManager;

// ==================================================================== executor
void TapeExecutor::register_operation(OpTypeId op_type, OperationHandler handler) {
    if (op_type >= operation_handlers_.size()) operation_handlers_.resize(op_type + 1);
    operation_handlers_[op_type] = std::move(handler);
}

bool TapeExecutor::is_registered(OpTypeId op_type) const {
    return op_type < operation_handlers_.size() && operation_handlers_[op_type] != nullptr;
}

size_t TapeExecutor::get_num_registered_operations() const { return operation_handlers_.size(); }

std::shared_ptr<Tensor> TapeExecutor::get_result(NodeId node_id) const { return get_result(node_id, 0); }

std::shared_ptr<Tensor> TapeExecutor::get_result(NodeId node_id, uint16_t idx) const {
    auto it = results_.find({node_id, idx});
    return it != results_.end() ? it->second : nullptr;
}

void TapeExecutor::set_result(NodeId node_id, std::shared_ptr<Tensor> r) { set_result(node_id, 0, std::move(r)); }

void TapeExecutor::set_result(NodeId node_id, uint16_t idx, std::shared_ptr<Tensor> r) {
    results_[{node_id, idx}] = std::move(r);
}

void TapeExecutor::clear_results() { results_.clear(); }

size_t TapeExecutor::memory_usage() const {
    size_t total = 0;
    for (const auto& [k, t] : results_)
        if (t) total += t->total_elements() * sizeof(float);
    return total;
}

void TapeExecutor::execute_operation(TapeOperation& op) {
    if (op.is_evaluated) return;
    if (!is_registered(op.op_type)) throw std::runtime_error("Unknown operation type: " + std::to_string(op.op_type));
    operation_handlers_[op.op_type](op, *this);
    op.is_evaluated = true;
    ++ops_executed_;
}

namespace tt_lazy {
namespace {
int g_profiling = -1;  // -1: from TT_LAZY_PROFILE on first use
std::vector<OpProfile> g_last_profile;
}  // namespace

void set_profiling(bool on) { g_profiling = on ? 1 : 0; }
bool profiling() {
    if (g_profiling < 0) {
        const char* e = getenv("TT_LAZY_PROFILE");
        g_profiling = (e && e[0] == '1') ? 1 : 0;
    }
    return g_profiling == 1;
}
std::vector<OpProfile> last_profile() { return g_last_profile; }

std::string op_label(const TapeOperation& op) {
    if (op.plan)
        return std::string(op.plan->has_matmul ? "FusedGemm" : "FusedChain") + "[" + op.plan->describe() + "]";
    const Node* n = Context::instance().get_node(op.node_id);
    return n ? std::string(n->op_name()) : std::string("?");
}
}  // namespace tt_lazy

void TapeExecutor::execute_tape(Tape& tape) {
    const auto& ops = tape.operations();
    const bool prof = tt_lazy::profiling();
    std::vector<std::pair<int, int>> marks;
    std::vector<std::string> labels;
    std::map<std::pair<NodeId, uint16_t>, size_t> last_use;
    for (size_t i = 0; i < ops.size(); ++i)
        for (const auto& o : ops[i]->operands)
            if (o.lazy) last_use[{o.node, o.index}] = i;
    std::set<std::pair<NodeId, uint16_t>> keep;
    for (const auto& t : tape.outputs())
        if (t.is_lazy()) keep.insert({t.producer_node(), t.output_index()});
    // an op's own handle on its first output (TapeOperation::result) is dropped
    // with the executor's, so a released result goes back to the pool at once
    std::map<NodeId, TapeOperation*> producer;
    for (const auto& op : ops) producer[op->node_id] = op.get();
    for (size_t i = 0; i < ops.size(); ++i) {
        if (prof) {
            labels.push_back(tt_lazy::op_label(*ops[i]));
            int m0 = -1;
            if (ttc_timer_mark(&m0) != TTC_OK) throw std::runtime_error(ttc_last_error());
            ttc_range_push(labels.back().c_str());
            marks.push_back({m0, -1});
        }
        execute_operation(*ops[i]);
        if (prof) {
            ttc_range_pop();
            if (ttc_timer_mark(&marks.back().second) != TTC_OK) throw std::runtime_error(ttc_last_error());
        }
        if (tt_lazy::MemoryManager::instance().canaries()) {
            const auto bad = tt_lazy::MemoryManager::instance().check_canaries("after " + tt_lazy::op_label(*ops[i]));
            if (!bad.empty()) throw std::runtime_error("tt_lazy: " + bad.front());
        }
        // release operands whose last reader just ran
        for (const auto& o : ops[i]->operands) {
            if (!o.lazy) continue;
            const auto key = std::make_pair(o.node, o.index);
            if (last_use[key] != i || keep.count(key)) continue;
            results_.erase(key);
            if (key.second == 0) {
                auto p = producer.find(key.first);
                if (p != producer.end()) p->second->result.reset();
            }
        }
    }
    if (prof) {
        std::vector<tt_lazy::OpProfile> p;
        for (size_t i = 0; i < marks.size(); ++i) {
            float ms = 0.0f;
            if (ttc_timer_elapsed(marks[i].first, marks[i].second, &ms) != TTC_OK)
                throw std::runtime_error(ttc_last_error());
            p.push_back({labels[i], (double)ms});
        }
        tt_lazy::g_last_profile = std::move(p);
    }
}

// =================================================================== handlers
namespace {

using tt_lazy::upload;

void check(int rc) {
    if (rc != TTC_OK) throw std::runtime_error(ttc_last_error());
}

struct Operand {
    DeviceView view;
    std::vector<uint32_t> shape;
};

Operand resolve(const OperandRef& o, TapeExecutor& ex, const char* what) {
    Operand r;
    if (o.lazy) {
        auto t = ex.get_result(o.node, o.index);
        if (!t) throw std::runtime_error(std::string("Missing lazy input tensor for ") + what + " operation");
        r.view = t->device();
        r.shape = t->shape_vector();
    } else {
        r.view = upload(o.tensor);
        r.shape = o.tensor.shape_vector();
    }
    return r;
}

int64_t numel(const std::vector<uint32_t>& s) {
    int64_t n = 1;
    for (auto d : s) n *= d;
    return n;
}

// A dense row-major buffer for `copies` tensors of `shape` (the view covers
// the first; copy s starts at element s * numel(shape)).
DeviceView new_buffer(const std::vector<uint32_t>& shape, int copies = 1) {
    DeviceView v;
    v.buf = MemoryManager::instance().allocate((size_t)std::max<int64_t>(numel(shape) * copies, 1) * sizeof(float));
    int64_t s = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
        v.strides[i] = s;
        s *= shape[(size_t)i];
    }
    return v;
}

void set_output(TapeExecutor& ex, TapeOperation& op, NodeId node, uint16_t idx, const std::vector<uint32_t>& shape,
                DeviceView v) {
    auto t = std::make_shared<Tensor>(Tensor::on_device(shape, std::move(v)));
    ex.set_result(node, idx, t);
    if (node == op.node_id && idx == 0) op.result = t;
}

bool is_contiguous(const Operand& o) {
    int64_t expect = 1;
    for (int i = (int)o.shape.size() - 1; i >= 0; --i) {
        if (o.shape[(size_t)i] != 1 && o.view.strides[i] != expect) return false;
        expect *= o.shape[(size_t)i];
    }
    return true;
}

// Dense row-major copy of an operand (used only when a consumer cannot fold
// the operand's strides).
// Dense copy of a window whose innermost dim has stride 1: dims (outer...,
// rows, cols) with strides (..., rs, 1) into dst (row-major). Dims before the
// last two become chain segments (one launch per extra outer index).
void copy_rows(const float* src, const std::vector<int64_t>& sh, const std::vector<int64_t>& st, float* dst) {
    const int r = (int)sh.size();
    const int64_t cols = sh[(size_t)r - 1], rows = r >= 2 ? sh[(size_t)r - 2] : 1;
    const int64_t rs = r >= 2 ? st[(size_t)r - 2] : cols;
    const int64_t nseg = r >= 3 ? sh[(size_t)r - 3] : 1, ss = r >= 3 ? st[(size_t)r - 3] : 0;
    const int64_t outer = r >= 4 ? sh[0] : 1, os = r >= 4 ? st[0] : 0;
    if (r > 4 || nseg > 65535 || rows > INT32_MAX || cols > INT32_MAX)
        throw std::runtime_error("tt_lazy: view too large to densify");
    for (int64_t o = 0; o < outer; ++o) {
        ttc_chain_desc d;
        std::memset(&d, 0, sizeof d);
        d.rows = (int32_t)rows;
        d.cols = (int32_t)cols;
        d.nseg = (int32_t)nseg;
        d.n_inputs = 1;
        d.inputs[0] = ttc_in_view{src + o * os, rs, 1, ss};
        d.n_outputs = 1;
        d.outputs[0] = ttc_out_view{dst + o * nseg * rows * cols, cols, rows * cols};
        d.n_instr = 2;
        d.program[0] = ttc_instr{TTC_OP_LOAD, TTC_SRC_INPUT, 0, 0};
        d.program[1] = ttc_instr{TTC_OP_STORE, TTC_SRC_ACC, 0, 0};
        check(ttc_eltwise_chain(&d));
    }
}

// Dense row-major copy of a strided view of rank <= 4 (transposes and split
// chunks, and compositions of them): the innermost dim with stride 1 is
// copied with 128-bit accesses; a view whose stride-1 dim is the
// second-to-last (a transposed window) is packed that way and then
// transposed by the tiled transpose kernel.
Operand contiguous(const Operand& o) {
    if (is_contiguous(o)) return o;
    Operand r;
    r.shape = o.shape;
    r.view = new_buffer(o.shape);
    // collapse dims of size 1 and dims whose strides nest
    std::vector<int64_t> sh, st;
    for (size_t i = 0; i < o.shape.size(); ++i) {
        if (o.shape[i] == 1) continue;
        const int64_t n = o.shape[i], s = o.view.strides[i];
        if (!sh.empty() && st.back() == n * s) {
            sh.back() *= n;
            st.back() = s;
        } else {
            sh.push_back(n);
            st.push_back(s);
        }
    }
    const size_t k = sh.size();
    if (k >= 1 && st[k - 1] == 1) {
        copy_rows(o.view.ptr(), sh, st, r.view.ptr());
    } else if (k >= 2 && st[k - 2] == 1) {
        // pack as [..., cols, rows] (stride 1 innermost), then transpose the last two dims
        std::vector<int64_t> psh = sh, pst = st;
        std::swap(psh[k - 1], psh[k - 2]);
        std::swap(pst[k - 1], pst[k - 2]);
        int64_t batch = 1;
        for (size_t i = 0; i + 2 < k; ++i) batch *= sh[i];
        DeviceView packed = new_buffer({(uint32_t)(batch * psh[k - 2]), (uint32_t)psh[k - 1]});
        copy_rows(o.view.ptr(), psh, pst, packed.ptr());
        check(ttc_transpose(packed.ptr(), r.view.ptr(), batch, psh[k - 2], psh[k - 1]));
    } else {
        std::string s;
        for (size_t i = 0; i < o.shape.size(); ++i) s += (i ? ", " : "") + std::to_string(o.view.strides[i]);
        throw std::runtime_error("tt_lazy: cannot densify a view with strides (" + s + ")");
    }
    return r;
}

}  // namespace

DeviceView tt_lazy::dense_view(const DeviceView& v, const std::vector<uint32_t>& shape) {
    Operand o;
    o.view = v;
    o.shape = shape;
    return contiguous(o).view;
}

namespace {

// --------------------------------------------------------- program builder
// Lowers a member DAG (element-wise ops over one element space, optional tail
// reduce) to the accumulator machine of ttc_eltwise_chain / the GEMM
// epilogue: acc holds the current value, four slots hold values that are
// read again later.
struct ProgramBuilder {
    ttc_chain_desc d;
    std::map<int, int> input_of_ext;  // external index -> chain input index
    int acc = INT32_MIN;              // value id in acc (INT32_MIN = none)
    int slot_val[TTC_CHAIN_SLOTS] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
    std::map<int, int> uses;  // remaining reads of each value id
    // value ids: member m -> m; external k -> -(k + 1); product -> kProduct
    ProgramBuilder() { std::memset(&d, 0, sizeof d); }

    void emit(uint8_t op, uint8_t src = TTC_SRC_ACC, uint8_t idx = 0) {
        if (d.n_instr >= TTC_CHAIN_MAX_INSTR) throw std::length_error("fused program too long");
        d.program[d.n_instr++] = ttc_instr{op, src, idx, 0};
    }
    int slot_of(int v) const {
        for (int s = 0; s < TTC_CHAIN_SLOTS; ++s)
            if (slot_val[s] == v) return s;
        return -1;
    }
    void free_dead_slots() {
        for (int s = 0; s < TTC_CHAIN_SLOTS; ++s)
            if (slot_val[s] != INT32_MIN && uses[slot_val[s]] <= 0) slot_val[s] = INT32_MIN;
    }
    // Keep acc's value alive before acc is overwritten.
    void spill_acc() {
        // externals reload from their input; members and the GEMM product
        // live only in registers and need a slot while still to be read
        if (acc == INT32_MIN || is_external(acc) || uses[acc] <= 0 || slot_of(acc) >= 0) return;
        for (int s = 0; s < TTC_CHAIN_SLOTS; ++s)
            if (slot_val[s] == INT32_MIN) {
                slot_val[s] = acc;
                emit(TTC_OP_SAVE, TTC_SRC_ACC, (uint8_t)s);
                return;
            }
        throw std::length_error("fused program needs more than 4 live values");
    }
    int input_index(int ext) {
        auto it = input_of_ext.find(ext);
        if (it == input_of_ext.end()) throw std::logic_error("external without a view");
        return it->second;
    }
    bool is_external(int v) const { return v < 0 && v != FusionPlan::kProduct; }
    void to_acc(int v) {
        if (acc == v) return;
        spill_acc();
        if (is_external(v)) {
            emit(TTC_OP_LOAD, TTC_SRC_INPUT, (uint8_t)input_index(-v - 1));
        } else {
            const int s = slot_of(v);
            if (s < 0) throw std::logic_error("fused value lost before its last use");
            emit(TTC_OP_LOAD, TTC_SRC_SLOT, (uint8_t)s);
        }
        acc = v;
    }
    // source operand of a binary op while acc holds `x`
    void binary(uint8_t op, int x, int y) {
        if (y == x) {
            emit(op, TTC_SRC_ACC);
        } else if (is_external(y)) {
            emit(op, TTC_SRC_INPUT, (uint8_t)input_index(-y - 1));
        } else {
            const int s = slot_of(y);
            if (s < 0) throw std::logic_error("fused operand not available");
            emit(op, TTC_SRC_SLOT, (uint8_t)s);
        }
    }
};

// Builds the program for `plan` (members up to `nmembers`). `entry` is the
// value acc holds at entry (kProduct for a GEMM epilogue, INT32_MIN for a
// chain). Escaping members are stored to consecutive outputs in member
// order; returns their member indices.
std::vector<int> build_program(ProgramBuilder& pb, const FusionPlan& plan, size_t nmembers, int entry) {
    pb.acc = entry;
    for (size_t m = 0; m < nmembers; ++m)
        for (int a : plan.members[m].args) pb.uses[a]++;
    std::vector<int> stored;
    for (size_t m = 0; m < nmembers; ++m) {
        const auto& mem = plan.members[m];
        if (mem.op == FusionPlan::REDUCE) {
            pb.to_acc(mem.args[0]);
            pb.uses[mem.args[0]]--;
            break;  // the reduction is the chain's tail (reduce mode of the desc)
        }
        int x = mem.args[0];
        if (mem.args.size() == 2 && pb.acc == mem.args[1]) x = mem.args[1];  // add / mul commute exactly
        const int y = mem.args.size() == 2 ? (x == mem.args[0] ? mem.args[1] : mem.args[0]) : x;
        pb.to_acc(x);
        pb.uses[x]--;
        if (mem.args.size() == 2) pb.uses[y]--;
        // acc is about to become member m; keep x if it is read again
        if (pb.uses[x] > 0) pb.spill_acc();
        switch (mem.op) {
            case FusionPlan::RELU: pb.emit(TTC_OP_RELU); break;
            case FusionPlan::SIGMOID: pb.emit(TTC_OP_SIGMOID); break;
            case FusionPlan::ADD: pb.binary(TTC_OP_ADD, x, y); break;
            case FusionPlan::MUL: pb.binary(TTC_OP_MUL, x, y); break;
            default: break;
        }
        pb.acc = (int)m;
        pb.free_dead_slots();
        if (mem.escapes) {
            pb.emit(TTC_OP_STORE, TTC_SRC_ACC, (uint8_t)stored.size());
            stored.push_back((int)m);
        }
    }
    return stored;
}

// Element space of a chain and how each operand maps onto it.
struct Space {
    bool transposed = false;  // iterate the physical (column-major) order
    int64_t rows = 0, cols = 0;
};

// ttc_in_view of an operand of shape `s` over the chain space `out` (rank-2
// [R, C] or flattened), or false when it needs a dense copy first.
bool operand_view(const Operand& o, const std::vector<uint32_t>& out, const Space& sp, ttc_in_view* v) {
    const int64_t n = numel(o.shape), full = numel(out);
    v->ptr = o.view.ptr();
    v->seg_stride = 0;
    if (n == full && o.shape == out) {
        if (is_contiguous(o)) {
            if (sp.transposed) return false;
            v->row_stride = sp.cols;
            v->col_stride = 1;
            return true;
        }
        if (out.size() == 2) {
            const int64_t rs = o.view.strides[0], cs = o.view.strides[1];
            if (!sp.transposed && cs == 1) {
                v->row_stride = rs;
                v->col_stride = 1;
                return true;
            }
            if (sp.transposed && rs == 1) {
                v->row_stride = cs;  // physical rows are logical columns
                v->col_stride = 1;
                return true;
            }
        }
        return false;
    }
    // [1, C] bias over [R, C]
    if (out.size() == 2 && o.shape.size() == 2 && o.shape[0] == 1 && o.shape[1] == out[1] && is_contiguous(o)) {
        if (!sp.transposed) {
            v->row_stride = 0;
            v->col_stride = 1;
        } else {
            v->row_stride = 1;  // physical row = logical column
            v->col_stride = 0;
        }
        return true;
    }
    if (n == full && is_contiguous(o) && !sp.transposed) {  // same element count, different rank
        v->row_stride = sp.cols;
        v->col_stride = 1;
        return true;
    }
    return false;
}

// Thrown when a segmented chain cannot address its segments with one stride
// per operand; the caller then runs the segments one by one.
struct SegmentLayoutError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Runs a fused chain plan. A segmented plan (nseg > 1) runs all segments in
// one launch: `ext` holds segment 0's operands and seg_strides[k] the element
// distance between consecutive segments of operand k (0 when shared).
void run_chain_plan(TapeOperation& op, TapeExecutor& ex, const FusionPlan& plan, std::vector<Operand> ext,
                    const std::vector<int64_t>* seg_strides = nullptr) {
    const int nseg = seg_strides ? plan.nseg : 1;
    const auto& members = plan.members;
    const bool has_reduce = members.back().op == FusionPlan::REDUCE;
    const size_t n_elt = has_reduce ? members.size() - 1 : members.size();
    // element space: the shape of the element-wise members (the reduce input)
    const std::vector<uint32_t> space_shape =
        n_elt > 0 ? members[n_elt - 1].shape
                  : (members.back().args[0] < 0 ? ext[(size_t)(-members.back().args[0] - 1)].shape
                                                : members[(size_t)members.back().args[0]].shape);
    const int rank = (int)space_shape.size();
    Space sp;
    sp.cols = rank ? space_shape[(size_t)rank - 1] : 1;
    sp.rows = numel(space_shape) / std::max<int64_t>(sp.cols, 1);
    // Transposed iteration when every full-size operand is a transposed view
    // (column stride != 1, row stride 1): no copy of the transpose is made.
    if (rank == 2) {
        bool any_full = false, all_t = true;
        for (const auto& o : ext) {
            if (o.shape != space_shape) continue;
            any_full = true;
            if (!(o.view.strides[0] == 1 && o.view.strides[1] != 1)) all_t = false;
        }
        sp.transposed = any_full && all_t;
    }
    ProgramBuilder pb;
    auto& d = pb.d;
    d.nseg = nseg;
    d.rows = (int32_t)(sp.transposed ? sp.cols : sp.rows);
    d.cols = (int32_t)(sp.transposed ? sp.rows : sp.cols);
    // inputs
    for (size_t k = 0; k < ext.size(); ++k) {
        ttc_in_view v;
        const int64_t ss = nseg > 1 ? (*seg_strides)[k] : 0;
        if (!operand_view(ext[k], space_shape, sp, &v)) {
            if (ss != 0) throw SegmentLayoutError("segment operand needs a dense copy");
            ext[k] = contiguous(ext[k]);
            if (!operand_view(ext[k], space_shape, sp, &v))
                throw std::runtime_error("Broadcasting addition not implemented for these shapes");
        }
        v.seg_stride = ss;
        pb.input_of_ext[(int)k] = d.n_inputs;
        d.inputs[d.n_inputs++] = v;
    }
    const auto stored = build_program(pb, plan, members.size(), INT32_MIN);
    // outputs of escaping element-wise members (all segments in one buffer)
    std::vector<DeviceView> outs;
    for (int m : stored) {
        DeviceView v = new_buffer(members[(size_t)m].shape, nseg);
        if (sp.transposed) {  // allocate physical [C, R]; expose as a transposed view
            v.strides[0] = 1;
            v.strides[1] = sp.rows;
        }
        d.outputs[d.n_outputs++] = ttc_out_view{v.ptr(), d.cols, numel(members[(size_t)m].shape)};
        outs.push_back(v);
    }
    DeviceView red_out;
    if (has_reduce) {
        const auto& r = members.back();
        // mode: all dims -> ALL; suffix -> over cols (ROWS); prefix -> over rows (COLS)
        std::vector<bool> red((size_t)rank, r.dims.empty());
        for (int32_t dd : r.dims) red[(size_t)(dd < 0 ? dd + rank : dd)] = true;
        int first = rank, last = -1;
        for (int i = 0; i < rank; ++i)
            if (red[(size_t)i]) {
                first = std::min(first, i);
                last = std::max(last, i);
            }
        int mode;
        int64_t R = 1, C = 1;
        if (first == 0 && last == rank - 1) {
            mode = TTC_REDUCE_ALL;
            R = sp.rows;
            C = sp.cols;
        } else if (last == rank - 1) {  // reduce a suffix: over columns of [prefix, suffix]
            for (int i = 0; i < first; ++i) R *= space_shape[(size_t)i];
            for (int i = first; i < rank; ++i) C *= space_shape[(size_t)i];
            mode = TTC_REDUCE_ROWS;
        } else {  // prefix
            for (int i = 0; i <= last; ++i) R *= space_shape[(size_t)i];
            for (int i = last + 1; i < rank; ++i) C *= space_shape[(size_t)i];
            mode = TTC_REDUCE_COLS;
        }
        if (sp.transposed) {
            if (mode == TTC_REDUCE_ROWS)
                mode = TTC_REDUCE_COLS;
            else if (mode == TTC_REDUCE_COLS)
                mode = TTC_REDUCE_ROWS;
            std::swap(R, C);
        } else if (mode != TTC_REDUCE_ALL && (R != d.rows || C != d.cols)) {
            // re-factor the element space for a reduction over a multi-dim prefix / suffix
            if (d.n_outputs > 0) throw std::logic_error("stored outputs need the natural element space");
            for (int k = 0; k < d.n_inputs; ++k) {
                if (d.inputs[k].row_stride != d.cols || d.inputs[k].col_stride != 1)
                    throw std::runtime_error("tt_lazy: reduction over this view needs a dense input");
                d.inputs[k].row_stride = C;
            }
            d.rows = (int32_t)R;
            d.cols = (int32_t)C;
        }
        d.reduce = mode;
        d.reduce_mean = r.mean ? 1 : 0;
        red_out = new_buffer(r.shape, nseg);
        d.reduce_out = red_out.ptr();
        d.reduce_seg_stride = numel(r.shape);
    }
    check(ttc_eltwise_chain(&d));
    // segment s of every result sits s * numel(shape) elements into its buffer
    auto seg_view = [](DeviceView v, const std::vector<uint32_t>& shape, int s) {
        v.offset += (int64_t)s * numel(shape);
        return v;
    };
    auto node_of = [&](size_t m, int s) { return nseg > 1 ? plan.seg_nodes[(size_t)s][m] : members[m].node; };
    for (int s = 0; s < nseg; ++s) {
        for (size_t j = 0; j < stored.size(); ++j) {
            const auto& m = members[(size_t)stored[j]];
            set_output(ex, op, node_of((size_t)stored[j], s), 0, m.shape, seg_view(outs[j], m.shape, s));
        }
        if (has_reduce)
            set_output(ex, op, node_of(members.size() - 1, s), 0, members.back().shape,
                       seg_view(red_out, members.back().shape, s));
    }
}

// matmul operand -> (ptr, ld, transposed) for ttc_gemm, folding a transposed view.
void gemm_operand(Operand& o, bool want_t, const float** ptr, int64_t* ld, int32_t* trans) {
    if (o.shape.size() != 2) throw std::runtime_error("Multi-dimensional matrix multiplication not fully implemented");
    const int64_t rs = o.view.strides[0], cs = o.view.strides[1];
    if (cs == 1 && rs >= (int64_t)o.shape[1]) {
        *ptr = o.view.ptr();
        *ld = rs;
        *trans = want_t ? 1 : 0;
    } else if (rs == 1 && cs >= (int64_t)o.shape[0]) {
        *ptr = o.view.ptr();
        *ld = cs;
        *trans = want_t ? 0 : 1;
    } else {
        o = contiguous(o);
        *ptr = o.view.ptr();
        *ld = o.shape[1];
        *trans = want_t ? 1 : 0;
    }
}

int gemm_path() {
    int p = tt_lazy::get_gemm_path();
    if (p < 0) {
        const char* e = getenv("TT_LAZY_GEMM");
        const std::string v = e ? e : "";
        p = v == "ffma" ? (int)TTC_GEMM_FFMA
            : v == "tf32" ? (int)TTC_GEMM_TF32
            : v == "tf32x3" ? (int)TTC_GEMM_TF32X3
                            : (int)TTC_GEMM_AUTO;
        tt_lazy::set_gemm_path(p);
    }
    return p;
}

void run_gemm_plan(TapeOperation& op, TapeExecutor& ex, const FusionPlan& plan, std::vector<Operand> ext) {
    Operand& A = ext[0];
    Operand& B = ext[1];
    ttc_gemm_desc g;
    std::memset(&g, 0, sizeof g);
    gemm_operand(A, plan.transpose_a, &g.a, &g.lda, &g.trans_a);
    gemm_operand(B, plan.transpose_b, &g.b, &g.ldb, &g.trans_b);
    const int64_t M = plan.transpose_a ? A.shape[1] : A.shape[0];
    const int64_t K = plan.transpose_a ? A.shape[0] : A.shape[1];
    const int64_t N = plan.transpose_b ? B.shape[0] : B.shape[1];
    const int64_t Kb = plan.transpose_b ? B.shape[1] : B.shape[0];
    if (K != Kb) throw std::runtime_error("Matrix dimension mismatch for multiplication");
    g.M = (int32_t)M;
    g.N = (int32_t)N;
    g.K = (int32_t)K;
    g.path = gemm_path();
    const std::vector<uint32_t> out_shape = {(uint32_t)M, (uint32_t)N};
    auto fit_path = [&]() {
        // "tf32" asks for the tensor-core path where it applies; shapes or
        // layouts the tcgen05 kernel does not take run on the fp32 path.
        if (g.path == TTC_GEMM_TF32 && ttc_gemm_select_path(&g) != TTC_GEMM_TF32) g.path = TTC_GEMM_FFMA;
    };
    ProgramBuilder pb;
    Space sp;
    sp.rows = M;
    sp.cols = N;
    for (size_t k = 2; k < ext.size(); ++k) {
        ttc_in_view v;
        if (!operand_view(ext[k], out_shape, sp, &v)) {
            ext[k] = contiguous(ext[k]);
            if (!operand_view(ext[k], out_shape, sp, &v))
                throw std::runtime_error("Broadcasting addition not implemented for these shapes");
        }
        pb.input_of_ext[(int)k] = pb.d.n_inputs;
        pb.d.inputs[pb.d.n_inputs++] = v;
    }
    std::vector<int> stored;
    DeviceView out, red_out;
    const bool has_reduce = !plan.members.empty() && plan.members.back().op == FusionPlan::REDUCE;
    if (plan.members.empty()) {
        out = new_buffer(out_shape);
        g.c = out.ptr();
        g.ldc = N;
    } else {
        stored = build_program(pb, plan, plan.members.size(), FusionPlan::kProduct);
        if (stored.size() != (has_reduce ? 0u : 1u))
            throw std::logic_error("fused GEMM must store exactly its final value");
        if (!has_reduce) {
            out = new_buffer(out_shape);
            pb.d.outputs[pb.d.n_outputs++] = ttc_out_view{out.ptr(), N, 0};
        } else {  // the batch-dim sum of the final value, reduced in the epilogue
            const auto& r = plan.members.back();
            red_out = new_buffer(r.shape);
            pb.d.reduce = TTC_REDUCE_COLS;
            pb.d.reduce_mean = r.mean ? 1 : 0;
            pb.d.reduce_out = red_out.ptr();
        }
        g.epilogue = pb.d;
    }
    fit_path();
    check(ttc_gemm(&g));
    if (has_reduce) {
        set_output(ex, op, plan.members.back().node, 0, plan.members.back().shape, red_out);
        return;
    }
    const NodeId node = plan.members.empty() ? op.node_id : plan.members[(size_t)stored[0]].node;
    set_output(ex, op, node, 0, out_shape, out);
}

std::vector<Operand> resolve_all(TapeOperation& op, TapeExecutor& ex, const char* what) {
    std::vector<Operand> r;
    for (const auto& o : op.operands) r.push_back(resolve(o, ex, what));
    return r;
}

// A single element-wise op as a one-member chain.
void single_eltwise(TapeOperation& op, TapeExecutor& ex, FusionPlan::MemberOp kind, const char* what,
                    size_t arity) {
    auto ext = resolve_all(op, ex, what);
    if (ext.size() != arity)
        throw std::runtime_error(std::string(what) + " operation requires exactly " + std::to_string(arity) +
                                 " input" + (arity > 1 ? "s" : "") + ", got " + std::to_string(ext.size()));
    FusionPlan plan;
    FusionPlan::Member m;
    m.node = op.node_id;
    m.op = kind;
    m.escapes = true;
    m.shape = op.output_shapes.at(0);
    for (size_t k = 0; k < arity; ++k) m.args.push_back(-(int)(k + 1));
    plan.members.push_back(m);
    run_chain_plan(op, ex, plan, ext);
}

void handle_relu(TapeOperation& op, TapeExecutor& ex) { single_eltwise(op, ex, FusionPlan::RELU, "ReLU", 1); }
void handle_sigmoid(TapeOperation& op, TapeExecutor& ex) {
    single_eltwise(op, ex, FusionPlan::SIGMOID, "Sigmoid", 1);
}
void handle_add(TapeOperation& op, TapeExecutor& ex) { single_eltwise(op, ex, FusionPlan::ADD, "Add", 2); }
void handle_multiply(TapeOperation& op, TapeExecutor& ex) {
    single_eltwise(op, ex, FusionPlan::MUL, "Multiply", 2);
}

void handle_reduce(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "reduce");
    if (ext.size() != 1)
        throw std::runtime_error("Reduce operation requires exactly 1 input, got " + std::to_string(ext.size()));
    const auto& args = Context::instance().get_node(op.node_id)->as<ReduceArgs>();
    if (args.type != ReduceArgs::Type::SUM && args.type != ReduceArgs::Type::MEAN)
        throw std::runtime_error("reduce: only SUM and MEAN are implemented");
    Operand in = contiguous(ext[0]);
    DeviceView out = new_buffer(op.output_shapes.at(0));
    std::vector<uint32_t> shape = in.shape;
    std::vector<int32_t> dims(args.dims.begin(), args.dims.end());
    check(ttc_reduce(in.view.ptr(), shape.data(), (int)shape.size(), dims.data(), (int)dims.size(),
                     args.type == ReduceArgs::Type::MEAN ? 1 : 0, out.ptr()));
    set_output(ex, op, op.node_id, 0, op.output_shapes.at(0), out);
}

// transpose(x): a view with the last two strides swapped; no kernel runs.
void handle_transpose(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "transpose");
    if (ext.size() != 1)
        throw std::runtime_error("Transpose operation requires exactly 1 input, got " + std::to_string(ext.size()));
    DeviceView v = ext[0].view;
    const int r = (int)ext[0].shape.size();
    if (r < 2) throw std::runtime_error("Transpose requires at least 2D tensor");
    std::swap(v.strides[r - 1], v.strides[r - 2]);
    set_output(ex, op, op.node_id, 0, op.output_shapes.at(0), v);
}

// split(x): one view per chunk (offset along `dim`); no kernel runs.
void handle_split(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "split");
    if (ext.size() != 1)
        throw std::runtime_error("Split operation requires exactly 1 input, got " + std::to_string(ext.size()));
    const auto& args = Context::instance().get_node(op.node_id)->as<SplitArgs>();
    const auto& in = ext[0];
    const int64_t size = in.shape.at((size_t)args.dim);
    for (size_t i = 0; i < op.output_shapes.size(); ++i) {
        DeviceView v = in.view;
        v.offset += (int64_t)i * args.split_size * in.view.strides[args.dim];
        (void)size;
        set_output(ex, op, op.node_id, (uint16_t)i, op.output_shapes[i], v);
    }
}

void handle_matmul(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "matmul");
    if (ext.size() != 2)
        throw std::runtime_error("MatMul operation requires exactly 2 inputs, got " + std::to_string(ext.size()));
    const auto& a = Context::instance().get_node(op.node_id)->as<MatMulArgs>();
    FusionPlan plan;
    plan.has_matmul = true;
    plan.transpose_a = a.transpose_a;
    plan.transpose_b = a.transpose_b;
    run_gemm_plan(op, ex, plan, ext);
}

void handle_fused_mlp(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "fused MLP");
    if (ext.size() != 3)
        throw std::runtime_error("Fused MLP operation requires exactly 3 inputs (input, weights, bias), got " +
                                 std::to_string(ext.size()));
    const auto& a = Context::instance().get_node(op.node_id)->as<FusedMLPArgs>();
    FusionPlan plan;
    plan.has_matmul = true;
    FusionPlan::Member bias;
    bias.op = FusionPlan::ADD;
    bias.args = {FusionPlan::kProduct, -3};
    bias.shape = op.output_shapes.at(0);
    plan.members.push_back(bias);
    const int act = a.activation >= 0 ? a.activation : (a.has_relu ? 1 : 0);
    if (act != 0) {
        FusionPlan::Member m;
        m.op = act == 1 ? FusionPlan::RELU : FusionPlan::SIGMOID;
        m.args = {0};
        m.shape = bias.shape;
        plan.members.push_back(m);
    }
    plan.members.back().node = op.node_id;
    plan.members.back().escapes = true;
    run_gemm_plan(op, ex, plan, ext);
}

// Segment s of a segmented plan as a plain chain plan.
FusionPlan segment_plan(const FusionPlan& p, int s) {
    FusionPlan q = p;
    q.nseg = 1;
    q.seg_nodes.clear();
    q.ext_seg_index.clear();
    for (size_t m = 0; m < q.members.size(); ++m) q.members[m].node = p.seg_nodes[(size_t)s][m];
    for (size_t k = 0; k < q.externals.size(); ++k)
        if (p.ext_seg_index[k] >= 0) q.externals[k].index = (uint16_t)(p.ext_seg_index[k] + s);
    return q;
}

void run_chain_unsegmented(TapeOperation& op, TapeExecutor& ex, const FusionPlan& plan);

void handle_fused_chain(TapeOperation& op, TapeExecutor& ex) {
    const FusionPlan& plan = *op.plan;
    if (plan.nseg <= 1) {
        run_chain_unsegmented(op, ex, plan);
        return;
    }
    // Segment k of a split operand must sit a fixed stride after segment k-1
    // in the same buffer with the same strides (equal chunks of one split).
    std::vector<Operand> ext;
    std::vector<int64_t> seg_strides;
    bool uniform = true;
    for (size_t k = 0; k < plan.externals.size(); ++k) {
        ext.push_back(resolve(plan.externals[k], ex, "fused chain"));
        int64_t stride = 0;
        if (plan.ext_seg_index[k] >= 0) {
            for (int s = 1; s < plan.nseg && uniform; ++s) {
                OperandRef r = plan.externals[k];
                r.index = (uint16_t)(plan.ext_seg_index[k] + s);
                const Operand o = resolve(r, ex, "fused chain");
                const int64_t dist = o.view.offset - ext[k].view.offset;
                if (s == 1) stride = dist;
                uniform = o.view.buf == ext[k].view.buf && o.shape == ext[k].shape && dist == s * stride &&
                          std::equal(o.view.strides, o.view.strides + 4, ext[k].view.strides) && stride != 0;
            }
        }
        seg_strides.push_back(stride);
    }
    if (uniform) {
        try {
            run_chain_plan(op, ex, plan, ext, &seg_strides);
            return;
        } catch (const SegmentLayoutError&) {
        } catch (const std::length_error&) {
        }
    }
    for (int s = 0; s < plan.nseg; ++s) run_chain_unsegmented(op, ex, segment_plan(plan, s));
}

void run_chain_unsegmented(TapeOperation& op, TapeExecutor& ex, const FusionPlan& plan) {
    std::vector<Operand> ext;
    for (const auto& o : plan.externals) ext.push_back(resolve(o, ex, "fused chain"));
    try {
        run_chain_plan(op, ex, plan, ext);
    } catch (const std::length_error&) {
        // Program over the register budget: run the members one by one.
        std::vector<Operand> vals(plan.members.size());
        for (size_t m = 0; m < plan.members.size(); ++m) {
            FusionPlan one;
            FusionPlan::Member mem = plan.members[m];
            std::vector<Operand> args;
            for (size_t j = 0; j < mem.args.size(); ++j) {
                const int a = mem.args[j];
                args.push_back(a < 0 ? ext[(size_t)(-a - 1)] : vals[(size_t)a]);
                mem.args[j] = -(int)(j + 1);
            }
            mem.escapes = mem.op != FusionPlan::REDUCE;
            one.members.push_back(mem);
            TapeExecutor scratch;
            TapeOperation tmp(mem.node, op.op_type);
            run_chain_plan(tmp, scratch, one, args);
            auto r = scratch.get_result(mem.node);
            vals[m].view = r->device();
            vals[m].shape = r->shape_vector();
            if (plan.members[m].escapes) set_output(ex, op, mem.node, 0, vals[m].shape, vals[m].view);
        }
    }
}

void handle_fused_gemm(TapeOperation& op, TapeExecutor& ex) {
    std::vector<Operand> ext;
    for (const auto& o : op.plan->externals) ext.push_back(resolve(o, ex, "fused MLP"));
    run_gemm_plan(op, ex, *op.plan, ext);
}

// all_reduce_sum(x): the cross-shard exchange of data parallelism. The sum
// is taken in a fresh buffer (results are immutable once produced).
void handle_all_reduce(TapeOperation& op, TapeExecutor& ex) {
    auto ext = resolve_all(op, ex, "all-reduce");
    if (ext.size() != 1)
        throw std::runtime_error("AllReduce operation requires exactly 1 input, got " + std::to_string(ext.size()));
    Operand in = contiguous(ext[0]);
    DeviceView out = new_buffer(in.shape);
    const size_t n = (size_t)numel(in.shape);
    check(ttc_memcpy_d2d(out.ptr(), in.view.ptr(), n * sizeof(float)));
    check(ttc_allreduce_sum(out.ptr(), n, tt_lazy::comm_timeout_ms()));
    set_output(ex, op, op.node_id, 0, in.shape, out);
}

}  // namespace

void register_all_operations(TapeExecutor& executor) {
    executor.register_operation(SplitArgs::type_id(), handle_split);
    executor.register_operation(MatMulArgs::type_id(), handle_matmul);
    executor.register_operation(ReduceArgs::type_id(), handle_reduce);
    executor.register_operation(ReLUArgs::type_id(), handle_relu);
    executor.register_operation(SigmoidArgs::type_id(), handle_sigmoid);
    executor.register_operation(AddArgs::type_id(), handle_add);
    executor.register_operation(MultiplyArgs::type_id(), handle_multiply);
    executor.register_operation(TransposeArgs::type_id(), handle_transpose);
    executor.register_operation(FusedMLPArgs::type_id(), handle_fused_mlp);
    executor.register_operation(FusedChainArgs::type_id(), handle_fused_chain);
    executor.register_operation(FusedGemmArgs::type_id(), handle_fused_gemm);
    executor.register_operation(AllReduceArgs::type_id(), handle_all_reduce);
}

// ========================================================= evaluation manager
namespace tt_lazy {

TapeEvaluationManager::TapeEvaluationManager() { register_all_operations(executor_); }

std::shared_ptr<Tensor> TapeEvaluationManager::evaluate(const Tensor& tensor) {
    if (tensor.is_evaluated()) {
        stats_.cache_hits++;
        return std::make_shared<Tensor>(tensor);
    }
    return evaluate_many({tensor}).at(0);
}

std::vector<std::shared_ptr<Tensor>> TapeEvaluationManager::evaluate_many(const std::vector<Tensor>& tensors) {
    const uint64_t epoch = Context::instance().epoch();
    std::vector<std::shared_ptr<Tensor>> out(tensors.size());
    std::vector<Tensor> todo;
    for (size_t i = 0; i < tensors.size(); ++i) {
        const Tensor& t = tensors[i];
        if (!t.is_lazy()) {
            out[i] = std::make_shared<Tensor>(t);
            continue;
        }
        auto it = cache_.find({epoch, t.producer_node(), t.output_index()});
        if (it != cache_.end()) {
            stats_.cache_hits++;
            out[i] = it->second;
        } else {
            todo.push_back(t);
        }
    }
    if (!todo.empty()) {
        stats_.cache_misses++;
        backend_init();
        ttc_memory_stats before;
        ttc_get_memory_stats(&before);
        auto tape = generator_.generate_tape(todo);
        executor_.clear_results();
        executor_.execute_tape(*tape);
        size_t fused = 0;
        for (const auto& op : tape->operations())
            if (op->plan && (op->plan->members.size() + (op->plan->has_matmul ? 1 : 0)) > 1) ++fused;
        for (const auto& t : todo) {
            auto r = executor_.get_result(t.producer_node(), t.output_index());
            if (!r) throw std::runtime_error("Failed to evaluate tensor");
            cache_[{epoch, t.producer_node(), t.output_index()}] = r;
        }
        ttc_memory_stats after;
        ttc_get_memory_stats(&after);
        stats_.operations_executed += tape->size();
        stats_.fused_operations = fused;
        stats_.kernels_launched = (size_t)(after.kernels_launched - before.kernels_launched);
        stats_.device_peak_bytes = MemoryManager::instance().stats().bytes_peak;
        executor_.clear_results();
        for (size_t i = 0; i < tensors.size(); ++i)
            if (!out[i])
                out[i] = cache_.at({epoch, tensors[i].producer_node(), tensors[i].output_index()});
    }
    for (const auto& r : out)
        if (r) stats_.memory_allocated += r->total_elements() * sizeof(float);
    return out;
}

void TapeEvaluationManager::clear_cache() {
    cache_.clear();
    clear_constant_cache();
    stats_ = EvaluationStats{};
}

EvaluationManager& get_evaluation_manager() {
    static TapeEvaluationManager* instance = new TapeEvaluationManager();
    return *instance;
}

CompiledTape::CompiledTape(const std::vector<Tensor>& outputs, int pipeline_chunks) : outputs_(outputs) {
    for (const auto& t : outputs)
        if (!t.is_lazy()) throw std::runtime_error("CompiledTape: outputs must be lazy tensors");
    if (pipeline_chunks > 1) outputs_ = build_row_pipeline(outputs, pipeline_chunks);
    TapeGenerator gen;
    tape_ = gen.generate_tape(outputs_);
    register_all_operations(executor_);
    if (pipeline_chunks > 1) {
        // the row chunks of the streamed batch, in the order the tape reads them
        std::set<std::pair<const void*, size_t>> seen;
        for (const auto& op : tape_->operations()) {
            std::vector<OperandRef> refs = op->operands;
            if (op->plan) refs.insert(refs.end(), op->plan->externals.begin(), op->plan->externals.end());
            for (const auto& o : refs)
                if (!o.lazy && o.tensor.is_streamed() &&
                    seen.insert({(const void*)o.tensor.host_data(), o.tensor.total_elements()}).second)
                    prefetch_.push_back(o.tensor);
        }
    }
}

CompiledTape::~CompiledTape() {
    if (graph_) ttc_graph_destroy(graph_);
}

void CompiledTape::run() {
    backend_init();
    if (graph_) {
        check(ttc_graph_launch(graph_));
        return;  // results_ and kernels_ are those of the captured run
    }
    ttc_memory_stats before;
    ttc_get_memory_stats(&before);
    execute();
    ttc_memory_stats after;
    ttc_get_memory_stats(&after);
    kernels_ = (size_t)(after.kernels_launched - before.kernels_launched);
}

void CompiledTape::capture() {
    if (graph_) return;
    for (const auto& op : tape_->operations())
        if (op->op_type == AllReduceArgs::type_id())
            throw std::runtime_error(
                "Plan.capture: a plan with an all-reduce is not captured (its completion is checked on the host "
                "against the communicator's deadline, which a graph replay would bypass)");
    run();  // warm: specialised kernels compiled, scratch grown, buffer pool filled
    check(ttc_synchronize());
    auto& mm = MemoryManager::instance();
    mm.begin_record();
    const auto mm0 = mm.stats();
    ttc_memory_stats before;
    ttc_get_memory_stats(&before);
    const bool prof = profiling(), guard = MemoryManager::instance().canaries();
    set_profiling(false);  // event waits and guard-band reads cannot be recorded into a graph
    MemoryManager::instance().set_canaries(false);
    struct Restore {
        bool prof, guard;
        ~Restore() {
            set_profiling(prof);
            MemoryManager::instance().set_canaries(guard);
        }
    } restore{prof, guard};
    check(ttc_capture_begin());
    void* exec = nullptr;
    try {
        execute();
    } catch (...) {
        ttc_capture_end(&exec);  // ends the (now invalid) capture
        ttc_graph_destroy(exec);
        mm.end_record();
        throw;
    }
    const int rc = ttc_capture_end(&exec);
    const auto used = mm.end_record();
    check(rc);
    // every buffer of the recorded run must come from the pool the warm run
    // filled: a fresh stream-ordered allocation would belong to the graph
    const auto mm1 = mm.stats();
    if (mm1.allocations - mm0.allocations != mm1.reuses - mm0.reuses) {
        ttc_graph_destroy(exec);
        throw std::runtime_error("Plan.capture: the recorded run needed new device memory; run it uncaptured");
    }
    // Buffers the recorded run released (intermediates, reused within the
    // graph in stream order) leave the pool for good; the rest are the
    // results, which this plan holds.
    std::vector<std::shared_ptr<DeviceBuffer>> held;
    for (const auto& [ptr, bytes] : used)
        if (auto b = mm.claim(ptr, bytes)) held.push_back(std::move(b));
    ttc_memory_stats after;
    ttc_get_memory_stats(&after);
    kernels_ = (size_t)(after.kernels_launched - before.kernels_launched);
    graph_ = exec;
    graph_bufs_ = std::move(held);
}

void CompiledTape::execute() {
    for (const auto& op : tape_->operations()) {
        op->is_evaluated = false;
        op->result.reset();  // the previous run's result buffers go back to the pool
    }
    results_.clear();
    executor_.clear_results();
    // start every chunk's upload on the copy stream; chunk c's kernels wait for chunk c only
    for (const auto& t : prefetch_) {
        DeviceView v;
        const size_t n = t.total_elements();
        v.buf = MemoryManager::instance().allocate(n * sizeof(float));
        set_contiguous_strides(v, t.shape_vector());
        int ticket = -1;
        check(ttc_h2d_prefetch(v.buf->ptr(), t.host_data(), n * sizeof(float), &ticket));
        prefetched()[{(const void*)t.host_data(), n}] = {v, ticket};
    }
    struct Clear {
        ~Clear() { prefetched().clear(); }
    } clear_prefetched;
    executor_.execute_tape(*tape_);
    for (const auto& t : outputs_) {
        auto r = executor_.get_result(t.producer_node(), t.output_index());
        if (!r) throw std::runtime_error("CompiledTape: output was not produced");
        results_.push_back(r);
    }
    executor_.clear_results();
}

std::shared_ptr<Tensor> CompiledTape::result(size_t i) const { return results_.at(i); }

namespace {
int g_comm_timeout_ms = 60000;
}

std::vector<uint8_t> comm_unique_id() {
    std::vector<uint8_t> id(TTC_UNIQUE_ID_BYTES);
    check(ttc_comm_unique_id(id.data()));
    return id;
}

void comm_init(int nranks, int rank, const std::vector<uint8_t>& id, int timeout_ms) {
    if (id.size() != TTC_UNIQUE_ID_BYTES) throw std::runtime_error("comm_init: unique id must be 128 bytes");
    backend_init();
    g_comm_timeout_ms = timeout_ms;
    check(ttc_comm_init(nranks, rank, id.data(), timeout_ms));
}

void comm_destroy() { ttc_comm_destroy(); }

int comm_timeout_ms() { return g_comm_timeout_ms; }

void evaluate(std::vector<Tensor*> tensors) {
    std::vector<Tensor> lazy;
    for (Tensor* t : tensors)
        if (t->is_lazy()) lazy.push_back(*t);
    auto& mgr = static_cast<TapeEvaluationManager&>(get_evaluation_manager());
    mgr.evaluate_many(lazy);
    for (Tensor* t : tensors) t->eval();  // cache hits: one device-to-host copy each
}

}  // namespace tt_lazy
