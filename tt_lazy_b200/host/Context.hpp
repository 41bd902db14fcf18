// Context.hpp -- the reference's include name for the global graph store
// (src/core/Context.hpp there), so code written against the reference's
// headers compiles against this front end unchanged; Context is declared with
// Node in Node.hpp.
#pragma once
#include "Node.hpp"
