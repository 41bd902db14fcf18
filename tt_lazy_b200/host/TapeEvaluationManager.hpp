// TapeEvaluationManager.hpp -- forwarding header: the declarations live in TapeExecutor.hpp / Tape.hpp.
#pragma once
#include "TapeExecutor.hpp"
