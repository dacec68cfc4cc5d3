// route_kernels.cuh -- expert routing on the device: router scores and the
// deterministic top-k that feeds the permutation.
//
// Reference (GLM and Kimi K3 route the same way):
//   scores[e] = sigmoid(x . router[e])        quant::matmul_f32 (quant.cpp:156-168),
//                                             quant::sigmoid (quant.hpp:22-29)
//   choice[e] = scores[e] + bias[e]           glm53.cpp:1921-1931, kimi_k3.cpp:1986-1998
//   idx, w    = moe_topk(choice, E, K, mix = scores)            ops.cpp:860-890
// moe_topk keeps the K largest choices (equal values: the lower expert id
// first), takes w[i] = mix[idx[i]] (or the choice) clamped at 0, and divides
// by their sum accumulated in selection order (1/K each when the sum is 0).
// DeepSeek-V4 (dsv4_cuda.cpp:1541-1587) scores with sqrt(softplus(logit))
// (dsv4_cuda.cpp:26-34) instead of the sigmoid, selects the same way (top 6)
// and multiplies each normalised weight by routed_scale.
#pragma once

#include "aux_kernels.cuh"

namespace mvb {

// Correctly rounded single-precision e^x through double precision: the double
// result is within one double ulp, so rounding it to float is exact except
// within 2^-29 of a float rounding boundary.  It matches a correctly rounded
// host expf (glibc's is within 0.502 ulp) far more often than the
// single-precision device expf (within 2 ulp).
__device__ __forceinline__ float expf_cr(float x) {
    return static_cast<float>(exp(static_cast<double>(x)));
}

// log(1 + x) correctly rounded the same way (through double precision).
__device__ __forceinline__ float log1pf_cr(float x) {
    return static_cast<float>(log1p(static_cast<double>(x)));
}

// quant::sigmoid with the exponential above.
__device__ __forceinline__ float sigmoid_route(float x) {
    if (x >= 0.f)
        return __fdiv_rn(1.f, __fadd_rn(1.f, expf_cr(-x)));
    const float z = expf_cr(x);
    return __fdiv_rn(z, __fadd_rn(1.f, z));
}

// sqrt(max(softplus(z), 0)) with softplus's three branches (z > 20: z;
// z < -20: e^z; else log1p(e^z)), dsv4_cuda.cpp:26-34; the square root is
// IEEE (correctly rounded), as the host's sqrtf.
__device__ __forceinline__ float sqrt_softplus_route(float z) {
    float sp;
    if (z > 20.f)
        sp = z;
    else if (z < -20.f)
        sp = expf_cr(z);
    else
        sp = log1pf_cr(expf_cr(z));
    return __fsqrt_rn(sp < 0.f ? 0.f : sp); // std::max(sp, 0.f)
}

// Router score functions (MVLLM_SCORE_*).
__device__ __forceinline__ float route_score(float logit, int score_fn) {
    return score_fn == MVLLM_SCORE_SQRT_SOFTPLUS ? sqrt_softplus_route(logit)
                                                 : sigmoid_route(logit);
}

// The router dot products in the reference's order (sequential f32 over H,
// each product and sum rounded on its own): seq_dot_tile with one chain per
// thread, CTAs of 32 tokens x 4 experts (E = 256, T = 32: 64 CTAs), then the
// score function and the bias.
template <typename TX, bool ASYNC>
__global__ void __launch_bounds__(kSeqThreads)
    route_scores_kernel(const TX *__restrict__ x, const float *__restrict__ w,
                        const float *__restrict__ bias, int T, int H, int E, int score_fn,
                        float *__restrict__ scores, float *__restrict__ choice) {
    extern __shared__ __align__(16) uint8_t seq_smem[];
    const int t0 = blockIdx.y * kSeqS, e0 = blockIdx.x * 4;
    float acc[1];
    if constexpr (ASYNC)
        seq_dot_async<4, 1, MVLLM_FMT_F32>(x, w, nullptr, T, H, E, t0, e0, acc, seq_smem);
    else
        seq_dot_tile<1>(x, w, nullptr, MVLLM_FMT_F32, T, H, E, t0, e0, acc);
    using L = SeqAsync<4, 1, MVLLM_FMT_F32, TX>;
    const int t = t0 + (ASYNC ? L::s_of(threadIdx.x) : threadIdx.x >> 2);
    const int e = e0 + (ASYNC ? L::g_of(threadIdx.x) : threadIdx.x & 3);
    if (t < T && e < E) {
        const float s = route_score(acc[0], score_fn);
        scores[static_cast<size_t>(t) * E + e] = s;
        choice[static_cast<size_t>(t) * E + e] = bias ? __fadd_rn(s, bias[e]) : s;
    }
}

template <typename TX>
inline cudaError_t route_scores_launch(cudaStream_t st, const TX *x, const float *router,
                                       const float *bias, int T, int H, int E, int score_fn,
                                       float *scores, float *choice) {
    const dim3 grid((E + 3) / 4, (T + kSeqS - 1) / kSeqS);
    if (seq_async_ok(x, router, MVLLM_FMT_F32, H)) {
        using L = SeqAsync<4, 1, MVLLM_FMT_F32, TX>;
        static_assert(L::THREADS == kSeqThreads, "thread mapping");
        const cudaError_t e = cudaFuncSetAttribute(
            route_scores_kernel<TX, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
            int(L::SMEM));
        if (e != cudaSuccess)
            return e;
        route_scores_kernel<TX, true><<<grid, kSeqThreads, L::SMEM, st>>>(
            x, router, bias, T, H, E, score_fn, scores, choice);
    } else {
        route_scores_kernel<TX, false><<<grid, kSeqThreads, 0, st>>>(x, router, bias, T, H, E,
                                                                    score_fn, scores, choice);
    }
    return cudaGetLastError();
}

constexpr int kTopkMaxPerLane = 32; // E <= 1024
constexpr int kTopkMaxK = 32;       // one lane per selected expert

// One warp per token: K rounds of a warp-wide arg-max over the choices not yet
// taken, ordered by (value descending, id ascending) -- the order of the
// reference's partial_sort comparator -- then the weights as moe_topk forms
// them, times `scale` (1 for moe_topk itself; DeepSeek-V4's routed_scale,
// dsv4_cuda.cpp:1579-1585).  Slots K > E get id -1 and weight 0, as the
// callers preset them.
__global__ void topk_kernel(const float *__restrict__ choice, const float *__restrict__ mix, int T,
                            int E, int K, float scale, int *__restrict__ idx,
                            float *__restrict__ wt) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int per = (E + 31) >> 5;
    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        const float *ch = choice + static_cast<size_t>(t) * E;
        float v[kTopkMaxPerLane];
#pragma unroll
        for (int j = 0; j < kTopkMaxPerLane; ++j)
            v[j] = (j < per && lane + 32 * j < E) ? ch[lane + 32 * j] : 0.f;
        uint32_t taken = 0;
        for (int j = 0; j < per; ++j)
            if (lane + 32 * j >= E)
                taken |= 1u << j;
        const int k = min(K, E);
        int sel = -1; // lane r keeps the id chosen in round r
        for (int r = 0; r < k; ++r) {
            float bv = 0.f;
            int be = -1;
#pragma unroll
            for (int j = 0; j < kTopkMaxPerLane; ++j) {
                if (j >= per || ((taken >> j) & 1u))
                    continue;
                const int e = lane + 32 * j;
                if (be < 0 || v[j] > bv || (v[j] == bv && e < be)) {
                    bv = v[j];
                    be = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oe = __shfl_xor_sync(0xffffffffu, be, o);
                if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be))) {
                    bv = ov;
                    be = oe;
                }
            }
            if (be >= 0 && (be & 31) == lane)
                taken |= 1u << (be >> 5);
            if (lane == r)
                sel = be;
        }
        // Lane r holds round r's id; its weight, clamped at 0.
        float w_r = 0.f;
        if (lane < k) {
            const float m = mix ? mix[static_cast<size_t>(t) * E + sel] : ch[sel];
            w_r = m < 0.f ? 0.f : m;
        }
        // Sum in selection order (the reference's order), the same on every lane.
        float sum = 0.f;
        for (int r = 0; r < k; ++r)
            sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, w_r, r));
        if (lane < K) {
            int *io = idx + static_cast<size_t>(t) * K;
            float *wo = wt + static_cast<size_t>(t) * K;
            if (lane < k) {
                io[lane] = sel;
                const float q =
                    sum > 0.f ? __fdiv_rn(w_r, sum) : __fdiv_rn(1.f, static_cast<float>(k));
                wo[lane] = __fmul_rn(q, scale); // exact for scale 1
            } else {
                io[lane] = -1;
                wo[lane] = 0.f;
            }
        }
    }
}

} // namespace mvb
