// dense_ffn.cuh -- the activation step of a dense gated FFN evaluated in the
// reference's arithmetic, for DeepSeek-V4's shared expert and dense MLP
// (dsv4_cuda::one_expert / expert_fp8, dsv4_cuda.cpp:169-189, 826-832;
// dsv4.cpp:2849-2860, 2999-3008).  The three projections around it run on
// matmul_generic_kernel; this file holds h = act(g, u) elementwise.
//
// The activations are quant.hpp:22-50 operation by operation (no contraction,
// IEEE division), with e^x and tanh correctly rounded through double
// precision, so that an output differs from the host's only where the host's
// expf or tanhf misrounds.
#pragma once

#include "route_kernels.cuh"

namespace mvb {

__device__ __forceinline__ float tanhf_cr(float x) {
    return static_cast<float>(tanh(static_cast<double>(x)));
}

// quant::clamped_swiglu / quant::situ_glu / silu(g) * u, in the reference's order.
__device__ __forceinline__ float act_exact(float g, float u, int act, float a, float b) {
    if (act == MVLLM_ACT_CLAMP_SWIGLU) {
        if (a > 0.f && g > a)
            g = a;
        const float s = __fmul_rn(g, sigmoid_route(g));
        if (a > 0.f) {
            if (u > a)
                u = a;
            if (u < -a)
                u = -a;
        }
        return __fmul_rn(s, u);
    }
    if (act == MVLLM_ACT_SITU) {
        // b1 * tanh(g / b1) * sigmoid(g) * b2 * tanh(u / b2), left to right
        float r = __fmul_rn(a, tanhf_cr(__fdiv_rn(g, a)));
        r = __fmul_rn(r, sigmoid_route(g));
        r = __fmul_rn(r, b);
        return __fmul_rn(r, tanhf_cr(__fdiv_rn(u, b)));
    }
    return __fmul_rn(__fmul_rn(g, sigmoid_route(g)), u);
}

// g[i] = act(g[i], u[i]) for n elements.
__global__ void dense_act_kernel(float *__restrict__ g, const float *__restrict__ u, size_t n,
                                 int act, float a, float b) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        g[i] = act_exact(g[i], u[i], act, a, b);
}

// y[i] = y[i] + d[i] (the reference's `y[i] += sh[i]`, dsv4_cuda.cpp:845-846).
__global__ void add_rows_kernel(float *__restrict__ y, const float *__restrict__ d, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(y[i], d[i]);
}

} // namespace mvb
