// Test infrastructure: lets the reference's own planner unit test
// (cpp/test-moe-planner.cpp, which includes "llama-moe-planner.h") compile
// against this project's planner, moe_prefetch_b200/csrc/moe_planner.h.
#pragma once
#include "moe_planner.h"
