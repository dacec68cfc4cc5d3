// metal_ops_compat.cpp -- mvllm::metal_ops::{init, shutdown, available,
// backend_name, moe_block} (src/gpu/metal_ops.hpp:15-18, :104-108) on top of
// the C ABI, for reference call sites such as glm53.cpp:150 and
// kimi_k3.cpp:157 that link against this library instead of metal_ops.cpp.
#include "../../include/mvllm_metal_ops.hpp"
#include "../../include/mvllm_moe.h"

#include <cstdlib>

namespace mvllm {
namespace metal_ops {

bool init() {
    const char *s = std::getenv("MVLLM_CUDA_DEVICE");
    return mvllm_moe_init(s ? std::atoi(s) : 0) == MVLLM_OK;
}

void shutdown() { mvllm_moe_shutdown(); }

bool available() { return mvllm_moe_available() != 0; }

const char *backend_name() { return mvllm_moe_backend_name(); }

bool moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
               const void *const *u, const void *const *d, const float *const *gs,
               const float *const *us, const float *const *ds, const float *xg, const int *xoff,
               const int *nr, const int *rows, const float *rw, float *out, int S, Act act,
               float act_a, float act_b) {
    return mvllm_moe_block(nb, D, Iinter, fmt, qgs, g, u, d, gs, us, ds, xg, xoff, nr, rows, rw,
                           out, S, static_cast<int>(act), act_a, act_b) == MVLLM_OK;
}

} // namespace metal_ops
} // namespace mvllm
