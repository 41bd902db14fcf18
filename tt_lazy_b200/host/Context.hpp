// Context.hpp -- the global graph store (declared with Node in Node.hpp).
#pragma once
#include "Node.hpp"
