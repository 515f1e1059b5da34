// Test shim: the reference include path mapped onto this build's header of the same name.
#pragma once
#include "strata_kv/kv_stream.hpp"
