// EvaluationManager.hpp -- the reference's include name for EvaluationManager (src/core/EvaluationManager.hpp there), so
// code written against the reference's headers compiles against this front end
// unchanged; the declarations live in TapeExecutor.hpp / Tape.hpp.
#pragma once
#include "TapeExecutor.hpp"
