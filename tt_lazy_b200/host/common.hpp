// common.hpp -- ids, small containers and the op-argument machinery of the
// tt_lazy front end (interface of the reference's src/core/common.hpp and
// src/core/OpArgs.hpp, re-implemented).
#pragma once
#include <cassert>
#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <string>
#include <string_view>
#include <type_traits>
#include <vector>

class Tensor;
class Node;
class Context;

using OpTypeId = uint32_t;  // common.hpp:27 of the reference
using NodeId = uint32_t;
constexpr NodeId INVALID_NODE_ID = 0;

// The reference uses boost::container::small_vector<T, N>; the inline
// capacity is an allocation optimisation only, so a std::vector carries the
// same interface here without the Boost dependency.
template <typename T, size_t N = 4>
class SmallVector : public std::vector<T> {
   public:
    using std::vector<T>::vector;
    SmallVector() = default;
    template <size_t M>
    SmallVector(const SmallVector<T, M>& o) : std::vector<T>(o.begin(), o.end()) {}
};

namespace detail {
// Process-wide counter handing out one id per Args type on first use
// (common.hpp:33-44 of the reference: ids depend on first-use order).
inline OpTypeId next_op_id() {
    static OpTypeId counter = 0;
    return ++counter;
}
template <typename T>
OpTypeId get_op_id() {
    static const OpTypeId id = next_op_id();
    return id;
}
}  // namespace detail

class OpArgsBase {
   public:
    virtual std::string_view op_name() const = 0;

   protected:
    OpArgsBase() = default;
    ~OpArgsBase() = default;
};

template <typename Derived>
class OpArgsImpl : public OpArgsBase {
   public:
    OpArgsImpl() = default;
    virtual ~OpArgsImpl() = default;
    static OpTypeId type_id() { return detail::get_op_id<Derived>(); }
};

// DEFINE_OP_ARGS(Name, members...) declares `struct NameArgs` with a NAME,
// op_name() and a stable type_id() (common.hpp:47-55 of the reference).
#define DEFINE_OP_ARGS(OpName, ...)                         \
    struct OpName##Args : public OpArgsImpl<OpName##Args> { \
        static constexpr const char* NAME = #OpName;        \
        std::string_view op_name() const override {         \
            return NAME;                                    \
        }                                                   \
        virtual ~OpName##Args() = default;                  \
        __VA_ARGS__                                         \
    }
