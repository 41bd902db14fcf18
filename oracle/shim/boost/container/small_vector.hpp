// Minimal stand-in for boost::container::small_vector, used only to compile
// the reference sources into the CPU oracle (oracle/_ref). It keeps the
// interface the reference uses (construction, push_back, iteration, size,
// max_size) on top of std::vector; the inline-capacity optimisation of the
// real class has no effect on results.
#pragma once
#include <cstddef>
#include <vector>

namespace boost {
namespace container {
template <class T, std::size_t N>
class small_vector : public std::vector<T> {
   public:
    using std::vector<T>::vector;
    small_vector() = default;
};
}  // namespace container
}  // namespace boost
