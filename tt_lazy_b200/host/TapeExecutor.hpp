// TapeExecutor.hpp -- runs a tape through registered operation handlers
// (interface of the reference's src/tape/TapeExecutor.hpp:14-46), plus the
// device memory manager and the evaluation manager of the B200 backend.
#pragma once
#include <functional>
#include <map>
#include <memory>
#include <unordered_map>
#include <string>
#include <vector>

#include "Tape.hpp"

class TapeExecutor;
using OperationHandler = std::function<void(TapeOperation&, TapeExecutor&)>;

class TapeExecutor {
   public:
    TapeExecutor() = default;

    // Runs the operations in order. Results no later operation reads and
    // that are not tape outputs are released right after their last reader
    // runs, so their device buffers are reused by the operations that follow.
    void execute_tape(Tape& tape);
    void execute_operation(TapeOperation& op);

    void register_operation(OpTypeId op_type, OperationHandler handler);
    bool is_registered(OpTypeId op_type) const;
    size_t get_num_registered_operations() const;

    std::shared_ptr<Tensor> get_result(NodeId node_id) const;
    std::shared_ptr<Tensor> get_result(NodeId node_id, uint16_t output_index) const;
    void set_result(NodeId node_id, std::shared_ptr<Tensor> result);
    void set_result(NodeId node_id, uint16_t output_index, std::shared_ptr<Tensor> result);

    void clear_results();
    size_t memory_usage() const;
    size_t operations_executed() const { return ops_executed_; }

   private:
    std::map<std::pair<NodeId, uint16_t>, std::shared_ptr<Tensor>> results_;
    std::vector<OperationHandler> operation_handlers_;
    size_t ops_executed_ = 0;
};

// Installs the B200 handlers for every op type (reference:
// src/tape/OperationHandlers.cpp:224-232, which installs the CPU handlers).
void register_all_operations(TapeExecutor& executor);

namespace tt_lazy {

// Tracing: while profiling is on (set_profiling, or TT_LAZY_PROFILE=1), every
// tape operation runs inside an NVTX range named after it and between two
// CUDA-event marks; last_profile() holds the device time of each operation
// of the most recent tape execution (evaluate or Plan.run), in tape order.
struct OpProfile {
    std::string op;
    double ms = 0.0;
};
void set_profiling(bool on);
bool profiling();
std::vector<OpProfile> last_profile();
// "FusedGemm[matmul -> relu]", "FusedChain[...]" or the graph op's name.
std::string op_label(const TapeOperation& op);

// Selects the GPU (TT_LAZY_DEVICE, else LOCAL_RANK, else 0) and initialises
// the CUDA backend once. Throws std::runtime_error when no B200 is present.
void backend_init();
bool backend_ready();

// GEMM path of matmul / fused MLP operations: TTC_GEMM_AUTO (tcgen05 TF32
// where the shape suits it), TTC_GEMM_FFMA (fp32, the 1e-5 path) or
// TTC_GEMM_TF32. Defaults to the TT_LAZY_GEMM environment variable
// ("ffma" / "tf32"), else AUTO.
void set_gemm_path(int path);
int get_gemm_path();

// A device buffer from the MemoryManager; returns to its pool on release.
class DeviceBuffer {
   public:
    DeviceBuffer(float* p, size_t bytes) : ptr_(p), bytes_(bytes) {}
    ~DeviceBuffer();
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    float* ptr() const { return ptr_; }
    size_t bytes() const { return bytes_; }

   private:
    float* ptr_;
    size_t bytes_;
};

// Device HBM owner: size-bucketed free lists over stream-ordered device
// allocations, so a buffer released by the tape (after its last reader) is
// handed to the next operation that needs that size, and the same
// evaluation repeated reuses the same memory. Replaces the reference's
// unused host MemoryPool (src/core/MemoryManager.cpp:46-133).
class MemoryManager {
   public:
    static MemoryManager& instance();
    std::shared_ptr<DeviceBuffer> allocate(size_t bytes);
    void release(float* ptr, size_t bytes);
    void trim();  // returns cached blocks to the device pool
    struct Stats {
        size_t bytes_live = 0, bytes_peak = 0, bytes_cached = 0;
        size_t allocations = 0, reuses = 0;
    };
    Stats stats() const { return stats_; }
    void reset_peak() { stats_.bytes_peak = stats_.bytes_live; }
    // Host buffers of >= 1 MiB are pinned (page-locked) once the backend is up.
    static std::shared_ptr<float> host_buffer(size_t n);
    // Recording (CUDA-graph capture): every allocation between begin_record
    // and end_record is listed; claim() then takes a listed buffer that is
    // back in the pool out of it for good (the graph writes it on every
    // replay), handing ownership to the caller.
    void begin_record() {
        recording_ = true;
        recorded_.clear();
    }
    std::vector<std::pair<float*, size_t>> end_record() {
        recording_ = false;
        return std::move(recorded_);
    }
    std::shared_ptr<DeviceBuffer> claim(float* ptr, size_t bytes);

    // Guard bands (debug; set_canaries(true) or TT_LAZY_CANARY=1): each
    // buffer gets 256 extra bytes at its end filled with a known pattern;
    // check_canaries() reads every live band back (and release() each freed
    // one) and reports the buffers whose band was written, i.e. an overrun.
    void set_canaries(bool on) { canaries_ = on ? 1 : 0; }
    bool canaries();
    std::vector<std::string> check_canaries(const std::string& where);
    // Byte offset of `ptr`'s guard band (-1 when it has none).
    long long canary_offset(const float* ptr) const;

   private:
    std::unordered_map<size_t, std::vector<float*>> free_;
    Stats stats_;
    bool recording_ = false;
    std::vector<std::pair<float*, size_t>> recorded_;
    int canaries_ = -1;                          // -1: from TT_LAZY_CANARY on first use
    std::unordered_map<float*, size_t> guarded_;  // live buffers with a band -> bytes
    std::vector<std::string> violations_;        // found at release, reported by check_canaries
    bool band_intact(float* ptr, size_t bytes);
};

// Device copies of constant tensors (host pointer + size -> device buffer),
// kept across evaluations until clear_cache(): weights are uploaded once.
// Materialized non-constant inputs are uploaded on every evaluation.
DeviceView upload(const Tensor& t);
void clear_constant_cache();

// Dense row-major device copy of a strided view (rank <= 4) of `shape`; the
// view itself when it is already dense.
DeviceView dense_view(const DeviceView& v, const std::vector<uint32_t>& shape);

class EvaluationManager {
   public:
    virtual ~EvaluationManager() = default;
    EvaluationManager(const EvaluationManager&) = delete;
    EvaluationManager& operator=(const EvaluationManager&) = delete;
    virtual std::shared_ptr<Tensor> evaluate(const Tensor& tensor) = 0;
    virtual void clear_cache() = 0;
    struct EvaluationStats {
        size_t cache_hits = 0;
        size_t cache_misses = 0;
        size_t operations_executed = 0;
        size_t memory_allocated = 0;
        size_t fused_operations = 0;  // tape ops that absorbed >1 graph node
        size_t kernels_launched = 0;  // CUDA kernels of the last evaluation
        size_t device_peak_bytes = 0;
    };
    virtual EvaluationStats get_stats() const = 0;

   protected:
    EvaluationManager() = default;
};

EvaluationManager& get_evaluation_manager();

class TapeEvaluationManager : public EvaluationManager {
   public:
    TapeEvaluationManager();
    std::shared_ptr<Tensor> evaluate(const Tensor& tensor) override;
    // Evaluates several lazy tensors with one tape (shared sub-graphs run
    // once) and returns their device-resident results.
    std::vector<std::shared_ptr<Tensor>> evaluate_many(const std::vector<Tensor>& tensors);
    void clear_cache() override;
    EvaluationStats get_stats() const override { return stats_; }
    TapeGenerator& generator() { return generator_; }

   private:
    TapeGenerator generator_;
    TapeExecutor executor_;
    // keyed by (Context epoch, node id, output index): stale entries never
    // match after Context::clear()
    std::map<std::tuple<uint64_t, NodeId, uint16_t>, std::shared_ptr<Tensor>> cache_;
    EvaluationStats stats_;
};

// Materialises several tensors with one tape (the results are copied to
// host memory, as data_ptr() would).
void evaluate(std::vector<Tensor*> tensors);

// A tape generated once and executed many times: the serving / benchmark
// loop of a fixed graph. Constant inputs stay resident on the device,
// streamed inputs are re-uploaded on every run(), results stay on the
// device until fetched.
// pipeline_chunks > 1: the graph is rebuilt over that many row chunks of its
// streamed batch input (build_row_pipeline) and each chunk's upload overlaps
// the kernels of the chunks before it.
class CompiledTape {
   public:
    explicit CompiledTape(const std::vector<Tensor>& outputs, int pipeline_chunks = 1);
    ~CompiledTape();
    CompiledTape(const CompiledTape&) = delete;
    CompiledTape& operator=(const CompiledTape&) = delete;
    void run();
    // Runs once, then records one run into a CUDA graph; from then on run()
    // replays the graph with a single launch (same inputs, same device
    // buffers; streamed inputs are still copied from their host memory on
    // every replay). Plans with an all-reduce are not captured (it waits on
    // the host).
    void capture();
    bool captured() const { return graph_ != nullptr; }
    std::shared_ptr<Tensor> result(size_t i) const;
    size_t size() const { return tape_->size(); }
    size_t kernels_last_run() const { return kernels_; }
    const Tape& tape() const { return *tape_; }

   private:
    std::vector<Tensor> outputs_;
    std::unique_ptr<Tape> tape_;
    TapeExecutor executor_;
    std::vector<std::shared_ptr<Tensor>> results_;
    std::vector<Tensor> prefetch_;  // streamed chunk inputs uploaded on the copy stream
    size_t kernels_ = 0;
    void execute();
    void* graph_ = nullptr;                                  // ttc graph exec of the captured run
    std::vector<std::shared_ptr<DeviceBuffer>> graph_bufs_;  // every buffer the graph touches
};

// Row-chunked form of `outputs` over their one streamed rank-2 batch input
// (Pipeline.cpp); throws std::runtime_error when the graph is not row-local
// up to a batch-dim reduce_sum (optionally followed by all_reduce_sum).
std::vector<Tensor> build_row_pipeline(const std::vector<Tensor>& outputs, int chunks);

// Data parallelism across processes (one per GPU): an NCCL communicator and
// the all-reduce op of the front end (operations.hpp: all_reduce_sum).
std::vector<uint8_t> comm_unique_id();
void comm_init(int nranks, int rank, const std::vector<uint8_t>& id, int timeout_ms);
void comm_destroy();
int comm_timeout_ms();

}  // namespace tt_lazy
