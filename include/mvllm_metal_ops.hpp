// mvllm_metal_ops.hpp -- the reference's C++ moe_block entry, served by the
// sm_100a library.
//
// Same namespace, enum and signature as src/gpu/metal_ops.hpp:15-18 (init,
// shutdown, available, backend_name), :44 (Act) and :104-108 (moe_block), so
// a reference translation unit that calls metal_ops::moe_block compiles and
// links against libmvllm_moe.so unchanged.  Semantics follow the reference:
// returns false on invalid arguments (the caller then uses its host kernel,
// metal_ops.hpp:10); it also returns false when the CUDA path fails, with the
// reason in mvllm_moe_last_error().  The device is MVLLM_CUDA_DEVICE (default
// 0).  Only the moe_block subset of metal_ops is provided here.
#pragma once

namespace mvllm {
namespace metal_ops {

bool init();
void shutdown();
bool available();
const char *backend_name(); // "cuda-sm100a"

enum class Act : int { Silu = 0, ClampSwiGLU = 1, Situ = 2 };

bool moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
               const void *const *u, const void *const *d, const float *const *gs,
               const float *const *us, const float *const *ds, const float *xg, const int *xoff,
               const int *nr, const int *rows, const float *rw, float *out, int S,
               Act act = Act::Silu, float act_a = 0.f, float act_b = 0.f);

} // namespace metal_ops
} // namespace mvllm
