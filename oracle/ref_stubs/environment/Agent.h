// Stand-in for the reference's agent header: WorldGenerator.h only needs the
// AgentState position (reference: src/world/WorldGenerator.h:8,79 and
// src/world/WorldGenerator.cpp:10-34).
//
// Test infrastructure only; never linked into the product library.
#pragma once

#include <blocklab/utility/Math.h>

namespace blocklab {
struct AgentState {
    Vec3 position {};
};
} // namespace blocklab
