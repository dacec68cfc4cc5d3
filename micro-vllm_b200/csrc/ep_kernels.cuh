// ep_kernels.cuh -- expert-parallel dispatch and combine for the MoE layer
// sharded over ranks (one GPU each).
//
// Placement: by default expert e lives on rank e % nranks as that rank's
// local expert e / nranks (strided: with Zipf-skewed routing it balances the
// ranks far better than contiguous blocks).  A placement table may instead
// give, per expert, its rank or -1 -- a replicated expert that every rank
// holds and serves for its own tokens (hot experts stop concentrating load on
// one rank) -- and its local id on the rank that serves it.  A step on rank r:
//   plan     which of r's tokens each rank needs (a token goes to rank d once,
//            however many of its experts d owns) and where each lands in the
//            destination-major send buffer;
//   pack     token rows + per-slot local expert ids (-1 where another rank
//            owns the slot) + routing weights into the send buffer;
//   (all-to-all: NCCL, counts then rows)
//   compute  the received rows through the rank's local experts
//            (mvllm_moe_layer_dev: slots marked -1 are skipped);
//   (all-to-all back: each token's partial sums per rank)
//   combine  out[c] += the partials of token c in ascending rank order.
// The reference runs every expert on one host (metal_ops.cpp:466-509 over the
// rows that moe_layer_n gathers, glm53.cpp:1936-1994); the partition, the
// exchanges and the combine order are this layer's own.  Every sum has a
// fixed order, so runs are bit-reproducible; the association differs from the
// single-GPU order, within the parity tolerance.
#pragma once

#include "aux_kernels.cuh"

namespace mvb {

// The rank that serves expert e for a token of rank `self`, and its local id
// there (dest == nullptr: strided placement).
__device__ __forceinline__ int ep_dest(int e, int nranks, const int *dest, int self) {
    if (!dest)
        return e % nranks;
    const int d = __ldg(dest + e);
    return d < 0 ? self : d;
}
__device__ __forceinline__ int ep_local_id(int e, int nranks, const int *lid) {
    return lid ? __ldg(lid + e) : e / nranks;
}

// Expert parallelism without a token exchange (DeepSeek-V4's EP2,
// route_moe_ep2 with map_ep_expert's parity split, dsv4_cuda.cpp:1356-1369,
// 1841-1906): every rank holds all tokens and keeps only the slots it serves,
// as local ids; the other slots become -1 and the layer skips them.  The
// ranks' partial sums are then added by an all-reduce.  Every expert has
// exactly one serving rank here (dest[e] in [0, nranks); a replicated expert
// would be counted once per rank, so -1 entries serve no rank).
__global__ void ep_local_ids_kernel(const int *__restrict__ idx, int n, int E, int nranks,
                                    const int *__restrict__ dest, const int *__restrict__ lid,
                                    int self, int *__restrict__ out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int e = idx[i];
        int v = -1;
        if (e >= 0 && e < E && (dest ? __ldg(dest + e) : e % nranks) == self)
            v = ep_local_id(e, nranks, lid);
        out[i] = v;
    }
}

// One CTA: per destination rank a block scan over the tokens gives the
// position of each sent token among those of that rank; a second pass adds the
// destination offsets.  pos[c * nranks + d] = send-buffer row or -1.
// cap > 0: destination d's rows start at d * cap (fixed-size send segments,
// so the exchange needs no counts on the host); else right after d - 1's.
__global__ void ep_plan_kernel(const int *__restrict__ idx, int T, int K, int E, int nranks,
                               const int *__restrict__ dest, int self, int *__restrict__ pos,
                               int *__restrict__ send_cnt, int cap) {
    __shared__ int warp_sums[32];
    __shared__ int carry[32];
    __shared__ int off[33];
    if (threadIdx.x < 32)
        carry[threadIdx.x] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < T; c0 += blockDim.x) {
        const int c = c0 + threadIdx.x;
        uint32_t mask = 0;
        if (c < T)
            for (int k = 0; k < K; ++k) {
                const int e = idx[static_cast<size_t>(c) * K + k];
                if (e >= 0 && e < E)
                    mask |= 1u << ep_dest(e, nranks, dest, self);
            }
        for (int d = 0; d < nranks; ++d) {
            const int f = (mask >> d) & 1;
            int tot;
            const int ex = block_exclusive_scan(f, warp_sums, &tot);
            if (c < T)
                pos[static_cast<size_t>(c) * nranks + d] = f ? carry[d] + ex : -1;
            __syncthreads();
            if (threadIdx.x == 0)
                carry[d] += tot;
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) {
        off[0] = 0;
        for (int d = 0; d < nranks; ++d) {
            send_cnt[d] = carry[d];
            off[d + 1] = cap > 0 ? (d + 1) * cap : off[d] + carry[d];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * nranks; i += blockDim.x) {
        const int p = pos[i];
        if (p >= 0)
            pos[i] = p + off[i % nranks];
    }
}

// One CTA per token: its row (16-byte vectors) to every destination that
// needs it, with the slots' local ids (or -1) and weights.
template <typename TX>
__global__ void ep_pack_kernel(const TX *__restrict__ x, const int *__restrict__ idx,
                               const float *__restrict__ wt, int T, int K, int D, int E,
                               int nranks, const int *__restrict__ dest,
                               const int *__restrict__ lid, int self, const int *__restrict__ pos,
                               TX *__restrict__ send_x, int *__restrict__ send_idx,
                               float *__restrict__ send_wt) {
    constexpr int VEC = 16 / sizeof(TX);
    for (int c = blockIdx.x; c < T; c += gridDim.x) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(c) * D);
        for (int d = 0; d < nranks; ++d) {
            const int p = pos[static_cast<size_t>(c) * nranks + d];
            if (p < 0)
                continue;
            uint4 *dst = reinterpret_cast<uint4 *>(send_x + static_cast<size_t>(p) * D);
            for (int v = threadIdx.x; v < D / VEC; v += blockDim.x)
                dst[v] = src[v];
            for (int k = threadIdx.x; k < K; k += blockDim.x) {
                const int e = idx[static_cast<size_t>(c) * K + k];
                const bool mine = e >= 0 && e < E && ep_dest(e, nranks, dest, self) == d;
                send_idx[static_cast<size_t>(p) * K + k] = mine ? ep_local_id(e, nranks, lid) : -1;
                send_wt[static_cast<size_t>(p) * K + k] = wt[static_cast<size_t>(c) * K + k];
            }
        }
    }
}

// ---- exchange over peer memory ------------------------------------------
// Every rank owns one exchange window (cudaMalloc'd, mapped by the others
// through CUDA IPC) of nranks * seg rows, seg = the tokens a rank owns per
// step (fixed segments: rank s's rows for rank d are rows s*seg .. s*seg +
// seg - 1 of d's window).  Regions, each 256-byte aligned:
//   x    [nranks*seg, D]   the received token rows (the caller's x dtype)
//   ids  [nranks*seg, K]   int32 local expert ids (-1: no slot here)
//   wt   [nranks*seg, K]   f32 routing weights
//   back [nranks*seg, 2D+16] partial rows returned to this rank (row d*seg + j:
//                         rank d's partial sum for this rank's j-th token sent to d)
struct WindowLayout {
    size_t x, ids, wt, back, total;
};
inline WindowLayout ep_window_layout(int nranks, int seg, int K, int D, size_t xsize) {
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t rows = size_t(nranks) * seg;
    WindowLayout w;
    w.x = 0;
    w.ids = up(rows * D * xsize);
    w.wt = w.ids + up(rows * K * 4);
    w.back = w.wt + up(rows * K * 4);
    w.total = w.back + up(rows * (2 * size_t(D) + 16));
    return w;
}

// Dispatch by stores into the destinations' windows (the pack and both
// dispatch exchanges in one kernel): token c of rank `self`, planned into
// row d*seg + j for rank d (pos from ep_plan_kernel with cap = seg), goes to
// row self*seg + j of d's window -- its x row, the slots' local ids (-1 where
// another rank serves the slot) and weights.  Rows j >= send_cnt[d] of that
// segment get ids -1, so d's experts skip them.  Own rows (d == self) go to
// this rank's own window.  Every thread ends with a system-scope fence: the
// rows are visible to the destinations once the kernel has completed.
template <typename TX>
__global__ void ep_dispatch_peer_kernel(const TX *__restrict__ x, const int *__restrict__ idx,
                                        const float *__restrict__ wt, int T, int K, int D, int E,
                                        int nranks, const int *__restrict__ dest,
                                        const int *__restrict__ lid, int self, int seg,
                                        const int *__restrict__ pos,
                                        const int *__restrict__ send_cnt,
                                        uint8_t *const *__restrict__ win, WindowLayout lay) {
    constexpr int VEC = 16 / sizeof(TX);
    for (int c = blockIdx.x; c < T; c += gridDim.x) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(c) * D);
        for (int d = 0; d < nranks; ++d) {
            const int p = pos[static_cast<size_t>(c) * nranks + d];
            if (p < 0)
                continue;
            const size_t q = static_cast<size_t>(self) * seg + (p - d * seg);
            uint8_t *w = win[d];
            uint4 *dst = reinterpret_cast<uint4 *>(w + lay.x + q * D * sizeof(TX));
            for (int v = threadIdx.x; v < D / VEC; v += blockDim.x)
                dst[v] = src[v];
            int *di = reinterpret_cast<int *>(w + lay.ids) + q * K;
            float *dw = reinterpret_cast<float *>(w + lay.wt) + q * K;
            for (int k = threadIdx.x; k < K; k += blockDim.x) {
                const int e = idx[static_cast<size_t>(c) * K + k];
                const bool mine = e >= 0 && e < E && ep_dest(e, nranks, dest, self) == d;
                di[k] = mine ? ep_local_id(e, nranks, lid) : -1;
                dw[k] = wt[static_cast<size_t>(c) * K + k];
            }
        }
    }
    // The unused rows of this rank's segment on every destination.
    const size_t n = static_cast<size_t>(nranks) * seg * K;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(i / (static_cast<size_t>(seg) * K));
        const int j = static_cast<int>((i / K) % seg);
        if (j >= send_cnt[d])
            reinterpret_cast<int *>(win[d] + lay.ids)[(static_cast<size_t>(self) * seg + j) * K +
                                                      i % K] = -1;
    }
    __threadfence_system();
}

// out[c] += sum over ranks d ascending of back[pos[c, d]] (f32, float4).
__global__ void ep_combine_kernel(const float *__restrict__ back, const int *__restrict__ pos,
                                  int T, int nranks, int D, float *__restrict__ out) {
    const int n4 = D / 4;
    for (int c = blockIdx.y; c < T; c += gridDim.y) {
        for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += gridDim.x * blockDim.x) {
            float4 acc = reinterpret_cast<const float4 *>(out + static_cast<size_t>(c) * D)[v];
            for (int d = 0; d < nranks; ++d) {
                const int p = pos[static_cast<size_t>(c) * nranks + d];
                if (p < 0)
                    continue;
                const float4 b = reinterpret_cast<const float4 *>(back + static_cast<size_t>(p) * D)[v];
                acc.x = __fadd_rn(acc.x, b.x);
                acc.y = __fadd_rn(acc.y, b.y);
                acc.z = __fadd_rn(acc.z, b.z);
                acc.w = __fadd_rn(acc.w, b.w);
            }
            reinterpret_cast<float4 *>(out + static_cast<size_t>(c) * D)[v] = acc;
        }
    }
}

// out[c] += sum over ranks d ascending of the partial row back16[pos[c, d]]:
// f16 values times the row's power-of-two scale (exact in f32), then f32 adds.
__global__ void ep_combine16_kernel(const uint8_t *__restrict__ back16, const int *__restrict__ pos,
                                    int T, int nranks, int D, float *__restrict__ out) {
    const int n4 = D / 4;
    const size_t pitch = 2 * static_cast<size_t>(D) + 16;
    for (int c = blockIdx.y; c < T; c += gridDim.y) {
        for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += gridDim.x * blockDim.x) {
            float4 acc = reinterpret_cast<const float4 *>(out + static_cast<size_t>(c) * D)[v];
            for (int d = 0; d < nranks; ++d) {
                const int p = pos[static_cast<size_t>(c) * nranks + d];
                if (p < 0)
                    continue;
                const uint8_t *row = back16 + static_cast<size_t>(p) * pitch;
                const float sc = *reinterpret_cast<const float *>(row + 2 * static_cast<size_t>(D));
                const uint2 u = *reinterpret_cast<const uint2 *>(row + 8 * static_cast<size_t>(v));
                const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
                const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
                acc.x = __fadd_rn(acc.x, __fmul_rn(lo.x, sc));
                acc.y = __fadd_rn(acc.y, __fmul_rn(lo.y, sc));
                acc.z = __fadd_rn(acc.z, __fmul_rn(hi.x, sc));
                acc.w = __fadd_rn(acc.w, __fmul_rn(hi.y, sc));
            }
            reinterpret_cast<float4 *>(out + static_cast<size_t>(c) * D)[v] = acc;
        }
    }
}

} // namespace mvb
