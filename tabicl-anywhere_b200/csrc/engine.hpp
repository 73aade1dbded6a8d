// What the card tier (tier.cpp) uses of the engine beyond the C ABI: loading one fitted problem from a bundle on a
// thread of the tier's own, and its size before it is loaded.
#pragma once
#include <string>

#include "../../include/tabicl_b200.h"
#include "tirs.hpp"

namespace tcu {

struct Error {
    int code;
    std::string msg;
};

// A member's problem count and label digits (m{i}/meta[6], meta[5]).
struct MemberInfo {
    int nodes = 1, digits = 1;
};
MemberInfo member_info(const Bundle &b, const std::string &prefix);

// Problem `node` of member `prefix` of bundle b, its column cache too when with_col and the bundle holds it. The
// stored records stream to the device through the context's pinned staging buffers on a stream of their own; the
// context's lock is held only while the model is created, so predictions on the context go on meanwhile. Callable
// from any thread. Throws Error or BundleError.
tcu_model *load_node(tcu_weights *w, const Bundle &b, const std::string &prefix, int node, bool with_col);

// The bytes tcu_model_bytes reports for that problem once it is loaded (Gpu::model_bytes, src/gpu.rs:2064-2068).
size_t node_bytes(const tcu_weights *w, const Bundle &b, const std::string &prefix, int node, bool with_col);

// Whether the model holds the column stage's cache (the `rows` hook can answer).
bool has_col(const tcu_model *m);

// Set the current thread's device to the weights' and return the context.
tcu_ctx *ctx_of(const tcu_weights *w);
// The weights' context (no device call).
tcu_ctx *ctx_of_weights(const tcu_weights *w);

}  // namespace tcu
