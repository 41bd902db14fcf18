// operations.hpp -- frontend operations: each builds a graph node and
// returns lazy output tensors, computing nothing (interface of the
// reference's src/frontend/operations.hpp:9-43, plus the ops the reference
// documents but lacks: sigmoid (README.md:276-350), transpose and
// reduce_mean (ReduceArgs::Type::MEAN, operations.hpp:13-14)).
#pragma once
#include <string>
#include <vector>

#include "Node.hpp"
#include "Tensor.hpp"
#include "common.hpp"

DEFINE_OP_ARGS(Split, int64_t split_size = 0; int32_t dim = 0;);

DEFINE_OP_ARGS(MatMul, bool transpose_a = false; bool transpose_b = false; float alpha = 1.0f; float beta = 0.0f;);

DEFINE_OP_ARGS(Reduce, SmallVector<int32_t, 4> dims; bool keepdim = false;
               enum class Type
               : uint8_t{SUM, MEAN, MAX, MIN} type = Type::SUM;);

DEFINE_OP_ARGS(ReLU, bool inplace = false;);

DEFINE_OP_ARGS(Sigmoid, bool inplace = false;);

DEFINE_OP_ARGS(Add, );

DEFINE_OP_ARGS(Multiply, );

DEFINE_OP_ARGS(Transpose, );

// act(input . weights + bias): has_relu as in the reference; `activation`
// extends it (0 none, 1 relu, 2 sigmoid) for the fusion pass.
DEFINE_OP_ARGS(FusedMLP, bool has_relu = true; std::string fusion_info = ""; int activation = -1;);

// Sum of this tensor over every rank of the data-parallel communicator
// (tt_lazy::comm_init). No reference counterpart: the reference is
// single-process.
DEFINE_OP_ARGS(AllReduce, int32_t reduce_op = 0;);

std::vector<Tensor> make_output_tensors(NodeId node_id, size_t num_outputs,
                                        const std::vector<std::vector<uint32_t>>& shapes);

std::vector<Tensor> split(const Tensor& input, int64_t split_size, int32_t dim = 0);
Tensor matmul(const Tensor& a, const Tensor& b, bool transpose_a = false, bool transpose_b = false);
Tensor reduce_sum(const Tensor& input, const std::vector<int32_t>& dims = {}, bool keepdim = false);
Tensor reduce_mean(const Tensor& input, const std::vector<int32_t>& dims = {}, bool keepdim = false);
Tensor relu(const Tensor& input);
Tensor sigmoid(const Tensor& input);
Tensor add(const Tensor& a, const Tensor& b);
Tensor multiply(const Tensor& a, const Tensor& b);
Tensor transpose(const Tensor& input);
Tensor fused_mlp(const Tensor& input, const Tensor& weights, const Tensor& bias, bool has_relu = true);
Tensor all_reduce_sum(const Tensor& input);

// Output shape of a reduction over `dims` (empty = every dim): reduced dims
// are dropped, or kept as 1 with keepdim; a full reduction is shape [1].
std::vector<uint32_t> reduced_shape(const std::vector<uint32_t>& in, const std::vector<int32_t>& dims, bool keepdim);
