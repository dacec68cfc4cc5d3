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

// ---- tolerance mode ---------------------------------------------------------
// Router scores with f32 fused multiply-adds in a different order than the
// reference: the dot products over H are split across a cluster of
// kRfSplit CTAs (one H slice each).  A CTA covers EXP experts x 32 tokens:
// warp w takes experts 2w and 2w+1, its lanes consecutive 8-column pieces of
// the slice, each lane keeping 2 x 32 partial sums that a butterfly of
// shuffles adds up.  Every rank stores its sums into the
// rank-0 CTA's shared memory (distributed shared memory), which adds the
// slices in rank order and applies the score function and the bias.
// Scores differ from the reference's by f32 reassociation (about 1e-6
// relative); the top-k that follows is the exact selection on those scores.
constexpr int kRfSplit = 8;

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Store to the same shared-memory variable of CTA `rank` of the cluster.
__device__ __forceinline__ void st_dsmem_f32(float *p, int rank, float v) {
    uint32_t a = smem_u32(p), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

__device__ __forceinline__ void load_x8(const float *p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

__device__ __forceinline__ void load_x8(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 q = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

// Shared memory of route_scores_fast_kernel: the CTA's slice of the 32 token
// rows and of its experts' router rows, then the partial sums.
template <typename TX, int EXP> __host__ __device__ inline size_t rf_smem_bytes(int H) {
    const int per = (H / 8 + kRfSplit - 1) / kRfSplit;
    return size_t(32) * per * 8 * sizeof(TX) + size_t(EXP) * per * 8 * 4 +
           size_t(kRfSplit) * EXP * 32 * 4;
}

// Grid: x = kRfSplit * ceil(E / EXP) (clusters of kRfSplit along x), y =
// ceil(T / 32); 16 * EXP threads (a warp per two experts); rf_smem_bytes of
// dynamic shared memory.  H a multiple of 8, rows 16-byte aligned.  The
// slices of the token rows and the router rows are staged in shared memory
// first (coalesced, every load independent), so the dot products wait on
// shared memory, not on a chain of global loads; tokens go in groups of 4 so
// that eight independent FMA chains are in flight per lane.
template <typename TX, int EXP>
__global__ void __launch_bounds__(16 * EXP, 1)
    route_scores_fast_kernel(const TX *__restrict__ x, const float *__restrict__ w,
                             const float *__restrict__ bias, int T, int H, int E, int score_fn,
                             float *__restrict__ scores, float *__restrict__ choice) {
    extern __shared__ __align__(16) uint8_t rf_smem[];
    const int rank = blockIdx.x % kRfSplit; // the CTA's rank in its cluster
    const int e0 = (blockIdx.x / kRfSplit) * EXP;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.y * 32, nt = min(32, T - t0);
    const int n8 = H / 8, per = (n8 + kRfSplit - 1) / kRfSplit;
    const int c0 = rank * per, c1 = min(n8, (rank + 1) * per); // 8-column pieces of the slice
    const int np = max(0, c1 - c0);
    TX *xs = reinterpret_cast<TX *>(rf_smem); // [32][per * 8]
    float *wsm = reinterpret_cast<float *>(rf_smem + size_t(32) * per * 8 * sizeof(TX));
    // [kRfSplit][EXP][32]: every rank's partial sums, gathered in rank 0's copy
    float *red = wsm + size_t(EXP) * per * 8;
    // Both slices arrive by bulk copies (a row piece each, all in flight at
    // once); the router rows' are issued before waiting for the kernels
    // before this one, which they do not depend on.
    __shared__ __align__(8) uint64_t bar;
    const uint32_t xrow_b = uint32_t(np) * 8u * uint32_t(sizeof(TX)), wrow_b = uint32_t(np) * 32u;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, uint32_t(EXP) * wrow_b + uint32_t(nt) * xrow_b);
        if (np > 0)
            for (int el = 0; el < EXP; ++el)
                bulk_g2s(wsm + static_cast<size_t>(el) * per * 8,
                         w + static_cast<size_t>(min(e0 + el, E - 1)) * H + 8 * c0, wrow_b, &bar,
                         policy_evict_first());
    }
    pdl_wait(); // x comes from the kernels before this one
    if (threadIdx.x == 0 && np > 0)
        for (int t = 0; t < nt; ++t)
            bulk_g2s(xs + static_cast<size_t>(t) * per * 8,
                     x + static_cast<size_t>(t0 + t) * H + 8 * c0, xrow_b, &bar,
                     policy_evict_last());
    for (int i = threadIdx.x; i < (32 - nt) * np; i += blockDim.x) { // padding tokens: zeros
        const int t = nt + i / np, c = i % np;
        float *z = reinterpret_cast<float *>(xs + static_cast<size_t>(t) * per * 8 + 8 * c);
        *reinterpret_cast<uint4 *>(z) = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (sizeof(TX) == 4)
            *reinterpret_cast<uint4 *>(z + 4) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads(); // the barrier's initialisation and the padding rows
    mbar_wait(&bar, 0, nullptr);
    const float *wa = wsm + static_cast<size_t>(2 * warp) * per * 8;
    const float *wb = wa + static_cast<size_t>(per) * 8;
    float sa[32], sb[32];
#pragma unroll
    for (int t = 0; t < 32; ++t)
        sa[t] = sb[t] = 0.f;
    for (int c = lane; c < np; c += 32) {
        float va[8], vb[8];
        load_x8(wa + 8 * c, va);
        load_x8(wb + 8 * c, vb);
#pragma unroll
        for (int tg = 0; tg < 32; tg += 4) {
            float xv[4][8];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                load_x8(xs + static_cast<size_t>(tg + u) * per * 8 + 8 * c, xv[u]);
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    sa[tg + u] = fmaf(xv[u][j], va[j], sa[tg + u]);
                    sb[tg + u] = fmaf(xv[u][j], vb[j], sb[tg + u]);
                }
        }
    }
    // Butterfly: after it lane l holds token l's sums over the warp's lanes.
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int t = 0; t < off; ++t) {
            // keep the half of the entries that matches this lane's bit
            const float ka = upper ? sa[t + off] : sa[t], ga = upper ? sa[t] : sa[t + off];
            const float kb = upper ? sb[t + off] : sb[t], gb = upper ? sb[t] : sb[t + off];
            sa[t] = ka + __shfl_xor_sync(0xffffffffu, ga, off);
            sb[t] = kb + __shfl_xor_sync(0xffffffffu, gb, off);
        }
    }
    // Push this rank's sums into rank 0's shared memory (remote stores do
    // not wait), then one cluster barrier.
    st_dsmem_f32(red + (static_cast<size_t>(rank) * EXP + 2 * warp) * 32 + lane, 0, sa[0]);
    st_dsmem_f32(red + (static_cast<size_t>(rank) * EXP + 2 * warp + 1) * 32 + lane, 0, sb[0]);
    cluster_sync_all();
    if (rank == 0) {
        for (int i = threadIdx.x; i < EXP * 32; i += blockDim.x) {
            const int el = i >> 5, tl = i & 31;
            float sum = 0.f;
#pragma unroll
            for (int r = 0; r < kRfSplit; ++r)
                sum += red[(static_cast<size_t>(r) * EXP + el) * 32 + tl];
            const int e = e0 + el, tt = t0 + tl;
            if (e < E && tt < T) {
                const float sc = route_score(sum, score_fn);
                scores[static_cast<size_t>(tt) * E + e] = sc;
                choice[static_cast<size_t>(tt) * E + e] = bias ? sc + bias[e] : sc;
            }
        }
    }
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
    pdl_wait(); // the scores come from the kernel before this one
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
