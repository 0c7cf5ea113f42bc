// V-JEPA 2-AC engine state of a context (the predictor's device weights and rollout workspaces).
#pragma once

namespace jb {

struct ACEngine {
    virtual ~ACEngine() = default;
};

}  // namespace jb
