// Test shim: the reference include path mapped onto this build's restatement of the same inline helpers.
#pragma once
#include "strata_kv/types.hpp"
