// A reference-style C++ caller of metal_ops::moe_block, built against
// include/mvllm_metal_ops.hpp and linked with libmvllm_moe.so (no torch, no
// Python): the drop-in path a reference translation unit takes.  Built and run
// by tests/test_abi.py on the CPU, where it checks the reference's
// argument-rejection behaviour and the backend identity; with a GPU it also
// runs one identity-expert call and checks the result.  Prints CPP-CALLER-OK.
#include <cmath>
#include <cstdio>
#include <cstring>

#include "mvllm_metal_ops.hpp"

using mvllm::metal_ops::Act;

int main() {
    namespace mo = mvllm::metal_ops;
    if (std::strcmp(mo::backend_name(), "cuda-sm100a") != 0) {
        std::printf("unexpected backend %s\n", mo::backend_name());
        return 1;
    }
    // metal_ops.cpp:452-457: nb < 1 or a null out is "false", before any device work.
    float out[4] = {0, 0, 0, 0};
    const float x[4] = {1, 2, 3, 4};
    const int xoff = 0, nr = 1, rows = 0;
    const float rw = 1.f;
    if (mo::moe_block(0, 4, 4, 0, 0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, x,
                      &xoff, &nr, &rows, &rw, out, 1)) {
        std::printf("nb = 0 accepted\n");
        return 1;
    }
    if (!mo::init()) { // no GPU: the caller falls back to its host kernel
        std::printf("CPP-CALLER-OK (no device)\n");
        return 0;
    }
    // One f32 expert with identity gate/up/down on 4 features: SiLU(x) * x.
    float eye[16] = {};
    for (int i = 0; i < 4; ++i)
        eye[i * 4 + i] = 1.f;
    const void *w[1] = {eye};
    const bool ok = mo::moe_block(1, 4, 4, 0, 0, w, w, w, nullptr, nullptr, nullptr, x, &xoff,
                                  &nr, &rows, &rw, out, 1, Act::Silu);
    mo::shutdown();
    for (int i = 0; ok && i < 4; ++i) {
        const float want = x[i] / (1.f + std::exp(-x[i])) * x[i];
        if (std::fabs(out[i] - want) > 1e-3f * std::fabs(want) + 1e-5f) {
            std::printf("out[%d] = %g, want %g\n", i, out[i], want);
            return 1;
        }
    }
    if (!ok) {
        std::printf("moe_block failed on the device\n");
        return 1;
    }
    std::printf("CPP-CALLER-OK\n");
    return 0;
}
