// aux_kernels.cuh -- everything around the expert GEMMs: planning, operand
// staging, token permutation, ordered combine, the generic (any shape, any
// format) expert kernels and the device-side weight packers.
#pragma once

#include "common.cuh"

namespace mvb {

// ---------------------------------------------------------------------------
// Block-wide exclusive scan of one int per thread (blockDim.x multiple of 32,
// <= 1024).  Returns the exclusive prefix; *total gets the block sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_sums, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o)
            x += y;
    }
    if (lane == 31)
        warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o)
                s += y;
        }
        if (lane < nwarps)
            warp_sums[lane] = s; // inclusive
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    *total = warp_sums[nwarps - 1];
    __syncthreads();
    return before;
}

// NV exclusive block scans at once (one set of barriers for all of them):
// v[k] -> the sum of v[k] over the lower threads, tot[k] the block's total.
// warp_sums holds NV x 32 ints.
template <int NV>
__device__ __forceinline__ void block_exclusive_scan_n(int (&v)[NV], int *warp_sums,
                                                       int (&tot)[NV]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int x[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        x[k] = v[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x[k], o);
            if (lane >= o)
                x[k] += y;
        }
        if (lane == 31)
            warp_sums[k * 32 + warp] = x[k];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            int s = lane < nwarps ? warp_sums[k * 32 + lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o)
                    s += y;
            }
            if (lane < nwarps)
                warp_sums[k * 32 + lane] = s; // inclusive
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int before = (warp > 0 ? warp_sums[k * 32 + warp - 1] : 0) + x[k] - v[k];
        tot[k] = warp_sums[k * 32 + nwarps - 1];
        v[k] = before;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Plan (one CTA): the reference's per-expert bookkeeping of cpu_moe_block
// (src/gpu/metal_ops.cpp:285-300): base advances by nr for every expert with
// nr > 0; an expert runs only when its weight (and, for fmt 4/7, scale)
// pointers are all non-null.  Emits base[], cnt[] (rows that run, else 0)
// and the item prefix arrays of both phases (blocks x token chunks).
struct PlanArgs {
    int nb, fmt;
    const int *nr;
    const void *const *g, *const *u, *const *d, *const *gs, *const *us, *const *ds;
    int chunk1, blocks1; // phase 1 token chunk and row blocks per expert
    int chunk2, blocks2;
    int *base, *cnt, *off1, *off2, *total_rows;
    const int *xoff; // operand rows must satisfy 0 <= xoff[e], xoff[e]+nr[e] <= x_rows
    int x_rows;
    int align_mask; // fast path: every weight and scale pointer has these address bits clear
                    // (15: 16-byte aligned; 31 for the mxf8f6f4 path's expanding TMA)
    int *err;
    // Tensor-core path: experts with at least tc_min rows get no decode items;
    // their 256-row token tiles (and a rest wider than tc_small rows) become
    // tc_blocks{1,2} CTA-pair items per tile (offsets toff1/toff2), a rest of
    // at most tc_small rows tc_sblocks{1,2} single-CTA items (soff1/soff2).
    // tc_min <= 0 disables the path.
    int tc_min, tc_small, tc_blocks1, tc_blocks2, tc_sblocks1, tc_sblocks2;
    int tc_shift; // pair token tiles of 2^tc_shift rows
    int *clear_word; // zeroed once the plan is written (the tensor-map "rewritten" flag)
    int *toff1, *toff2, *soff1, *soff2;
    // Redo lists: the tensor-core experts' rows as decode items (offsets
    // roff1/roff2), run when a tensor-core kernel raises *range_word (zeroed
    // here) for scale codes its operands cannot represent.
    int *roff1, *roff2, *range_word;
    // A rest of more than tc_small and at most tc_wide rows: tc_sblocks{1,2}
    // wide single-CTA items (offsets woff1/woff2); tc_wide <= tc_small: none.
    int tc_wide;
    int *woff1, *woff2;
};

// An expert's six weight / scale pointers, loaded ahead of their use.
struct ExpertPtrs {
    uintptr_t p[6];
};
__device__ __forceinline__ ExpertPtrs expert_ptrs(const PlanArgs &a, int e) {
    ExpertPtrs r;
    r.p[0] = reinterpret_cast<uintptr_t>(a.g[e]);
    r.p[1] = reinterpret_cast<uintptr_t>(a.u[e]);
    r.p[2] = reinterpret_cast<uintptr_t>(a.d[e]);
    const bool more = a.fmt != MVLLM_FMT_F32 || a.align_mask;
    r.p[3] = more ? reinterpret_cast<uintptr_t>(a.gs[e]) : 0;
    r.p[4] = more ? reinterpret_cast<uintptr_t>(a.us[e]) : 0;
    r.p[5] = more ? reinterpret_cast<uintptr_t>(a.ds[e]) : 0;
    return r;
}
// Bit 0: every array the format needs is present; bit 1: one of them breaks
// the fast path's alignment (a.align_mask).
__device__ __forceinline__ int expert_ptr_bits(const PlanArgs &a, const ExpertPtrs &r) {
    bool present = r.p[0] && r.p[1] && r.p[2];
    if (a.fmt != MVLLM_FMT_F32)
        present = present && r.p[3] && r.p[4] && r.p[5];
    if (!present)
        return 0;
    const uintptr_t any = r.p[0] | r.p[1] | r.p[2] | r.p[3] | r.p[4] | r.p[5];
    return (a.align_mask && (any & static_cast<uintptr_t>(a.align_mask))) ? 3 : 1;
}

// tab_pre >= 0: expert_ptr_bits of expert threadIdx.x, computed by the caller
// from pointers it loaded earlier (only when a.nb <= blockDim.x).
__device__ __forceinline__ void plan_body(const PlanArgs &a, int tab_pre = -1) {
    __shared__ int warp_sums[11 * 32];
    __shared__ int carry[11];
    if (threadIdx.x < 11)
        carry[threadIdx.x] = 0;
    __syncthreads();
    for (int e0 = 0; e0 < a.nb; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        int n = 0, c = 0, i1 = 0, i2 = 0, j1 = 0, j2 = 0, k1 = 0, k2 = 0, r1 = 0, r2 = 0;
        int m1 = 0, m2 = 0;
        if (e < a.nb) {
            n = max(a.nr[e], 0);
            bool ok = n > 0;
            if (ok) {
                const int tb = tab_pre >= 0 ? tab_pre : expert_ptr_bits(a, expert_ptrs(a, e));
                ok = (tb & 1) != 0;
                if (ok && (tb & 2)) {
                    set_error(a.err, MVLLM_ERR_DEVICE); // would break the bulk copies: skip
                    ok = false;
                }
            }
            if (ok && (a.xoff[e] < 0 || a.xoff[e] + n > a.x_rows)) {
                set_error(a.err, MVLLM_ERR_DEVICE); // out-of-range operand rows: skip
                ok = false;
            }
            c = ok ? n : 0;
            if (a.tc_min > 0 && c >= a.tc_min) {
                int npair, nsolo, nwide;
                tc_tiles3(c, a.tc_small, a.tc_wide, a.tc_shift, npair, nsolo, nwide);
                j1 = a.tc_blocks1 * npair;
                j2 = a.tc_blocks2 * npair;
                k1 = a.tc_sblocks1 * nsolo;
                k2 = a.tc_sblocks2 * nsolo;
                m1 = a.tc_sblocks1 * nwide;
                m2 = a.tc_sblocks2 * nwide;
                r1 = a.blocks1 * ((c + a.chunk1 - 1) / a.chunk1);
                r2 = a.blocks2 * ((c + a.chunk2 - 1) / a.chunk2);
            } else {
                i1 = c ? a.blocks1 * ((c + a.chunk1 - 1) / a.chunk1) : 0;
                i2 = c ? a.blocks2 * ((c + a.chunk2 - 1) / a.chunk2) : 0;
            }
        }
        // One scan of all eleven lists: rows, decode items, pair / single /
        // redo / wide items of both phases.
        int v[11] = {n, i1, i2, j1, j2, k1, k2, r1, r2, m1, m2}, tot[11];
        block_exclusive_scan_n<11>(v, warp_sums, tot);
        if (e < a.nb) {
            a.base[e] = carry[0] + v[0];
            a.cnt[e] = c;
            a.off1[e] = carry[1] + v[1];
            a.off2[e] = carry[2] + v[2];
            a.toff1[e] = carry[3] + v[3];
            a.toff2[e] = carry[4] + v[4];
            a.soff1[e] = carry[5] + v[5];
            a.soff2[e] = carry[6] + v[6];
            if (a.roff1) {
                a.roff1[e] = carry[7] + v[7];
                a.roff2[e] = carry[8] + v[8];
            }
            if (a.woff1) {
                a.woff1[e] = carry[9] + v[9];
                a.woff2[e] = carry[10] + v[10];
            }
        }
        __syncthreads();
        if (threadIdx.x < 11)
            carry[threadIdx.x] += tot[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (a.clear_word)
            *a.clear_word = 0;
        if (a.range_word)
            *a.range_word = 0;
        if (a.roff1) {
            a.roff1[a.nb] = carry[7];
            a.roff2[a.nb] = carry[8];
        }
        if (a.woff1) {
            a.woff1[a.nb] = carry[9];
            a.woff2[a.nb] = carry[10];
        }
        a.off1[a.nb] = carry[1];
        a.off2[a.nb] = carry[2];
        a.toff1[a.nb] = carry[3];
        a.toff2[a.nb] = carry[4];
        a.soff1[a.nb] = carry[5];
        a.soff2[a.nb] = carry[6];
        *a.total_rows = carry[0];
    }
}

__global__ void plan_kernel(const PlanArgs a) {
    pdl_wait();
    plan_body(a);
}

// ---------------------------------------------------------------------------
// Per-expert tensor maps for the decode kernels: each is a host-encoded
// template (shape, strides, box, swizzle) with the global address swapped in
// on the device (tensormap.replace), so the device-pointer entries need no
// host copy of the expert tables.  Maps of null pointers keep the template
// address; the plan never schedules those experts.  A map is rewritten only
// when its bytes change, and any rewrite raises *dirty, which tells the
// decode kernels to acquire maps through the tensormap proxy before use; with
// static weights the maps never change and no fence is needed.
constexpr int kTmapsPerExpert = 6; // gate, up, down packed rows; gate, up, down scales
template <int N> struct TmapSet {
    CUtensorMap m[N];
};
template <int N> struct TableSet {
    const void *const *t[N];
};
using TmapTemplates = TmapSet<kTmapsPerExpert>;

// Map `idx` = (expert e, map k): table t[k]'s entry e swapped into template k;
// `mine` is the thread's 128-byte shared-memory slot.
template <int N>
__device__ __forceinline__ void build_map_one(const TmapSet<N> &tpl, const TableSet<N> &tabs,
                                              int nb, uint8_t *__restrict__ out, int *dirty,
                                              int idx, uint4 *mine) {
    if (idx >= nb * N)
        return;
    const int e = idx / N, k = idx % N;
    const void *src = tabs.t[k] ? tabs.t[k][e] : nullptr;
    // A null array belongs to an expert this launch skips: its map is never
    // read, so it keeps whatever an earlier call left there (a call that runs
    // its experts in several batches, each with the others null, then finds
    // every map unchanged and needs no proxy fences).
    if (!src)
        return;
    uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(idx) * 128);
    // The wanted map in shared memory: template with the address swapped in.
    const uint4 *from = reinterpret_cast<const uint4 *>(&tpl.m[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        mine[i] = from[i];
    asm volatile("tensormap.replace.tile.global_address.shared::cta.b1024.b64 [%0], %1;" ::"r"(
                     smem_u32(mine)),
                 "l"(src)
                 : "memory");
    bool same = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 a = mine[i], b = dst[i];
        same &= (a.x == b.x) & (a.y == b.y) & (a.z == b.z) & (a.w == b.w);
    }
    if (!same) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            dst[i] = mine[i];
        tmap_release();
        atomicExch(dirty, 1);
    }
}

// One thread per (expert, map): map k of expert e gets table t[k]'s entry e.
template <int N>
__global__ void build_tmaps_kernel(const __grid_constant__ TmapSet<N> tpl, const TableSet<N> tabs,
                                   int nb, uint8_t *__restrict__ out, int *dirty) {
    pdl_wait();
    __shared__ __align__(128) uint8_t staged[128 * 128];
    build_map_one<N>(tpl, tabs, nb, out, dirty, blockIdx.x * blockDim.x + threadIdx.x,
                     reinterpret_cast<uint4 *>(staged + threadIdx.x * 128));
}

// ---------------------------------------------------------------------------
// Operand staging: rows of x (f32 or bf16, row length D) into f16 rows in the
// column order of the format (stage_pos), or into plain f32 rows.  With
// `index`, output row r reads input row index[r] (the permutation gather).
template <typename TIn, typename TOut>
__global__ void stage_rows_kernel(const TIn *__restrict__ x, const int *__restrict__ index,
                                  const int *__restrict__ nrows_dev, int nrows_host, int D,
                                  int fmt, TOut *__restrict__ out) {
    const int nrows = nrows_dev ? *nrows_dev : nrows_host;
    for (int r = blockIdx.x; r < nrows; r += gridDim.x) {
        const int src = index ? index[r] : r;
        const TIn *xr = x + static_cast<size_t>(src) * D;
        TOut *orow = out + static_cast<size_t>(r) * D;
        for (int k = threadIdx.x; k < D; k += blockDim.x) {
            float v;
            if constexpr (sizeof(TIn) == 4)
                v = xr[k];
            else
                v = __bfloat162float(xr[k]);
            if constexpr (sizeof(TOut) == 4)
                orow[k] = v;
            else
                orow[stage_pos(k, fmt)] = __float2half_rn(v);
        }
    }
}

// Eight consecutive values of row xr (the aligned 8-column chunk c) as the 16
// bytes of f16 the staged row holds there, in stage_pos order.  `big` is set
// when a finite value lies beyond the f16 range (it would otherwise become inf).
template <typename TIn>
__device__ __forceinline__ uint4 stage_chunk8(const TIn *__restrict__ xr, int c, int fmt,
                                              bool &big) {
    float v[8];
    if constexpr (sizeof(TIn) == 4) {
        const float4 *p = reinterpret_cast<const float4 *>(xr) + 2 * c;
        const float4 a = __ldg(p), b = __ldg(p + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
        v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(xr) + c);
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = __uint_as_float(w[j] << 16);
            v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
        big |= beyond_f16(v[j]);
    __half2 h[4];
    if (fmt == MVLLM_FMT_INT4_G64) { // k0,k4,k1,k5,k2,k6,k3,k7
#pragma unroll
        for (int j = 0; j < 4; ++j)
            h[j] = __floats2half2_rn(v[j], v[j + 4]);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    }
    return *reinterpret_cast<const uint4 *>(h);
}

// Vectorised form for the fast path (D % 8 == 0): a CTA per row at a time,
// a thread per aligned 8-column chunk, 16-byte stores of f16 in stage_pos
// order (several chunks per thread in flight).  A finite value beyond the
// f16 range records MVLLM_ERR_ACT_RANGE.  `index`, when given, holds at least
// nblocks entries: the block's first one is loaded together with the row
// count.
template <typename TIn>
__device__ __forceinline__ void stage_rows_body(const TIn *__restrict__ x,
                                                const int *__restrict__ index,
                                                const int *__restrict__ nrows_dev, int nrows_host,
                                                int D, int fmt, __half *__restrict__ out,
                                                int *err, int block, int nblocks) {
    const int src0 = index ? __ldg(index + block) : block;
    const int nrows = nrows_dev ? *nrows_dev : nrows_host;
    const int chunks = D >> 3;
    for (int r = block; r < nrows; r += nblocks) {
        const int src = r == block ? src0 : index ? __ldg(index + r) : r;
        const TIn *xr = x + static_cast<size_t>(src) * D;
        uint4 *orow = reinterpret_cast<uint4 *>(out + static_cast<size_t>(r) * D);
#pragma unroll 4
        for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
            bool big = false;
            const uint4 v = stage_chunk8(xr, c, fmt, big);
            if (big)
                set_error(err, MVLLM_ERR_ACT_RANGE);
            orow[c] = v;
        }
    }
}

template <typename TIn>
__global__ void stage_rows_f16x8_kernel(const TIn *__restrict__ x, const int *__restrict__ index,
                                        const int *__restrict__ nrows_dev, int nrows_host, int D,
                                        int fmt, __half *__restrict__ out, int *err) {
    pdl_wait();
    stage_rows_body(x, index, nrows_dev, nrows_host, D, fmt, out, err, blockIdx.x, gridDim.x);
}

// The gather-stage of the token rows (blocks [0, stage_blocks)) and the
// decode kernels' per-expert tensor maps (the blocks after them, a thread per
// map) in one launch: both only need the permutation and the plan.
template <typename TIn>
__global__ void __launch_bounds__(256)
    stage_maps_kernel(const TIn *__restrict__ x, const int *__restrict__ index,
                      const int *__restrict__ nrows_dev, int D, int fmt, __half *__restrict__ out,
                      int *err, int stage_blocks, const __grid_constant__ TmapTemplates tpl,
                      const TableSet<kTmapsPerExpert> tabs, int nb, uint8_t *__restrict__ maps,
                      int *dirty) {
    pdl_wait();
    if (static_cast<int>(blockIdx.x) < stage_blocks) {
        stage_rows_body(x, index, nrows_dev, 0, D, fmt, out, err, blockIdx.x, stage_blocks);
        return;
    }
    __shared__ __align__(128) uint8_t staged[256 * 128];
    build_map_one<kTmapsPerExpert>(
        tpl, tabs, nb, maps, dirty, (blockIdx.x - stage_blocks) * blockDim.x + threadIdx.x,
        reinterpret_cast<uint4 *>(staged + threadIdx.x * 128));
}

// ---------------------------------------------------------------------------
// Token permutation (caller gather order, src/model/glm53.cpp:1958-1971).
// Step 1, thread per token: for each distinct valid id among the token's K
// entries (first occurrence), wsum = sum_t wt[c,t]*[idx[c,t]==e] in t order
// from 0.f; a non-zero wsum sets membership bit (e, c).
__global__ void permute_member_kernel(const int *__restrict__ idx, const float *__restrict__ wt,
                                      int T, int K, int E, int n_shared, int words,
                                      uint32_t *__restrict__ bitmap, float *__restrict__ wsum_out,
                                      int *__restrict__ tok_pos) {
    const int KK = K + n_shared;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < T; c += gridDim.x * blockDim.x) {
        const int *ic = idx + static_cast<size_t>(c) * K;
        const float *wc = wt + static_cast<size_t>(c) * K;
        for (int t = 0; t < K; ++t) {
            const int e = ic[t];
            tok_pos[static_cast<size_t>(c) * KK + t] = -1;
            if (e < 0 || e >= E)
                continue;
            bool dup = false;
            for (int t2 = 0; t2 < t; ++t2)
                dup |= (ic[t2] == e);
            if (dup)
                continue;
            float wsum = 0.f;
            for (int t2 = 0; t2 < K; ++t2)
                if (ic[t2] == e)
                    wsum = __fadd_rn(wsum, wc[t2]);
            if (wsum == 0.f)
                continue;
            wsum_out[static_cast<size_t>(c) * KK + t] = wsum;
            tok_pos[static_cast<size_t>(c) * KK + t] = -2; // placed in step 2
            atomicOr(&bitmap[static_cast<size_t>(e) * words + (c >> 5)], 1u << (c & 31));
        }
        if (n_shared) {
            wsum_out[static_cast<size_t>(c) * KK + K] = 1.f;
            tok_pos[static_cast<size_t>(c) * KK + K] = -2;
            atomicOr(&bitmap[static_cast<size_t>(E) * words + (c >> 5)], 1u << (c & 31));
        }
    }
}

// Step 2, one CTA per expert: the popcount of every bitmap word and their
// exclusive prefix (the rank, inside the expert's segment, of the word's first
// member), and the member count.
__global__ void permute_count_kernel(int words, const uint32_t *__restrict__ bitmap,
                                     int *__restrict__ wpre, int *__restrict__ nr) {
    __shared__ int warp_sums[32];
    const int e = blockIdx.x;
    const uint32_t *row = bitmap + static_cast<size_t>(e) * words;
    int *pre = wpre + static_cast<size_t>(e) * words;
    int carry = 0;
    for (int j0 = 0; j0 < words; j0 += blockDim.x) {
        const int j = j0 + threadIdx.x;
        const int v = j < words ? __popc(row[j]) : 0;
        int tot;
        const int ex = block_exclusive_scan(v, warp_sums, &tot);
        if (j < words)
            pre[j] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0)
        nr[e] = carry;
}

// Step 3 (one CTA): segment starts in ascending expert id.
__global__ void permute_offsets_kernel(int EE, const int *__restrict__ nr, int *__restrict__ xoff,
                                       int *__restrict__ n_rows) {
    __shared__ int warp_sums[32];
    int carry = 0;
    for (int e0 = 0; e0 < EE; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const int v = e < EE ? nr[e] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, warp_sums, &tot);
        if (e < EE)
            xoff[e] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0)
        *n_rows = carry;
}

// Step 4, thread per (token, slot): each member slot marked by step 1 (the
// first slot of the token holding that expert) takes the position of its
// bit in the expert's bitmap row -- ascending token order inside the segment.
__global__ void permute_place_kernel(const int *__restrict__ idx, int T, int K, int E,
                                     int n_shared, int words, const uint32_t *__restrict__ bitmap,
                                     const int *__restrict__ wpre, const int *__restrict__ xoff,
                                     const float *__restrict__ wsum_in, int *__restrict__ rows,
                                     float *__restrict__ rw, int *__restrict__ tok_pos) {
    const int KK = K + n_shared;
    const size_t n = static_cast<size_t>(T) * KK;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        if (tok_pos[i] != -2)
            continue;
        const int c = static_cast<int>(i / KK), s = static_cast<int>(i - static_cast<size_t>(c) * KK);
        const int e = s < K ? idx[static_cast<size_t>(c) * K + s] : E;
        const size_t wi = static_cast<size_t>(e) * words + (c >> 5);
        const int pos = xoff[e] + wpre[wi] + __popc(bitmap[wi] & ((1u << (c & 31)) - 1u));
        rows[pos] = c;
        rw[pos] = wsum_in[i];
        tok_pos[i] = pos;
    }
}

// Steps 1-4 in one CTA for small batches (decode: T <= kPermSmallT, so a
// bitmap row is at most 8 words): the same arithmetic in one launch instead
// of four plus the bitmap clear.  Global memory written by the CTA's own
// threads is visible to all of them after each __syncthreads.
constexpr int kPermSmallT = 256;
__device__ __forceinline__ void permute_small_body(
    const int *__restrict__ idx, const float *__restrict__ wt, int T, int K, int E, int n_shared,
    int words, uint32_t *__restrict__ bitmap, int *__restrict__ wpre, float *__restrict__ wsum,
    int *__restrict__ nr, int *__restrict__ xoff, int *__restrict__ n_rows,
    int *__restrict__ rows, float *__restrict__ rw, int *__restrict__ tok_pos) {
    __shared__ int warp_sums[32];
    const int EE = E + n_shared, KK = K + n_shared;
    for (int i = threadIdx.x; i < EE * words; i += blockDim.x)
        bitmap[i] = 0u;
    __syncthreads();
    // step 1: membership and per-token weight sums (permute_member_kernel)
    for (int c = threadIdx.x; c < T; c += blockDim.x) {
        const int *ic = idx + static_cast<size_t>(c) * K;
        const float *wc = wt + static_cast<size_t>(c) * K;
        for (int t = 0; t < K; ++t) {
            const int e = ic[t];
            tok_pos[static_cast<size_t>(c) * KK + t] = -1;
            if (e < 0 || e >= E)
                continue;
            bool dup = false;
            for (int t2 = 0; t2 < t; ++t2)
                dup |= (ic[t2] == e);
            if (dup)
                continue;
            float s = 0.f;
            for (int t2 = 0; t2 < K; ++t2)
                if (ic[t2] == e)
                    s = __fadd_rn(s, wc[t2]);
            if (s == 0.f)
                continue;
            wsum[static_cast<size_t>(c) * KK + t] = s;
            tok_pos[static_cast<size_t>(c) * KK + t] = -2;
            atomicOr(&bitmap[static_cast<size_t>(e) * words + (c >> 5)], 1u << (c & 31));
        }
        if (n_shared) {
            wsum[static_cast<size_t>(c) * KK + K] = 1.f;
            tok_pos[static_cast<size_t>(c) * KK + K] = -2;
            atomicOr(&bitmap[static_cast<size_t>(E) * words + (c >> 5)], 1u << (c & 31));
        }
    }
    __syncthreads();
    // step 2: word prefixes and member counts, a thread per expert
    for (int e = threadIdx.x; e < EE; e += blockDim.x) {
        int carry = 0;
        for (int j = 0; j < words; ++j) {
            wpre[static_cast<size_t>(e) * words + j] = carry;
            carry += __popc(bitmap[static_cast<size_t>(e) * words + j]);
        }
        nr[e] = carry;
    }
    __syncthreads();
    // step 3: segment starts in ascending expert id (permute_offsets_kernel)
    int carry = 0;
    for (int e0 = 0; e0 < EE; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const int v = e < EE ? nr[e] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, warp_sums, &tot);
        if (e < EE)
            xoff[e] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0)
        *n_rows = carry;
    __syncthreads();
    // step 4: positions (permute_place_kernel)
    const int n = T * KK;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        if (tok_pos[i] != -2)
            continue;
        const int c = i / KK, sl = i - c * KK;
        const int e = sl < K ? idx[static_cast<size_t>(c) * K + sl] : E;
        const size_t wi = static_cast<size_t>(e) * words + (c >> 5);
        const int pos = xoff[e] + wpre[wi] + __popc(bitmap[wi] & ((1u << (c & 31)) - 1u));
        rows[pos] = c;
        rw[pos] = wsum[i];
        tok_pos[i] = pos;
    }
}

__global__ void __launch_bounds__(1024)
    permute_small_kernel(const int *__restrict__ idx, const float *__restrict__ wt, int T, int K,
                         int E, int n_shared, int words, uint32_t *__restrict__ bitmap,
                         int *__restrict__ wpre, float *__restrict__ wsum, int *__restrict__ nr,
                         int *__restrict__ xoff, int *__restrict__ n_rows,
                         int *__restrict__ rows, float *__restrict__ rw,
                         int *__restrict__ tok_pos) {
    pdl_wait();
    permute_small_body(idx, wt, T, K, E, n_shared, words, bitmap, wpre, wsum, nr, xoff, n_rows,
                       rows, rw, tok_pos);
}

// The same four steps for the layer's decode-sized calls (K <= KMAX), with
// every array the CTA reads back in shared memory: the membership bitmap and
// word prefixes (bm, wp, [E + n_shared][words]), the counts and segment
// starts (nr_s, xoff_s, [E + n_shared]) and per slot the weight sum and state
// (ws, tk, [T][K + n_shared]; tk = the slot's expert while it waits to be
// placed, -1 for none).  A token's ids and weights are loaded once into
// registers.  Outputs (nr, xoff, n_rows, rows, rw, tok_pos) are those of
// permute_small_body, bit for bit: the same membership, the same ascending
// order of the weight sums.
template <int KMAX>
__device__ __forceinline__ void permute_small_smem_body(
    const int *__restrict__ idx, const float *__restrict__ wt, int T, int K, int E, int n_shared,
    int words, uint32_t *bm, int *wp, float *ws, int *tk, int *nr_s, int *xoff_s,
    int *__restrict__ nr, int *__restrict__ xoff, int *__restrict__ n_rows,
    int *__restrict__ rows, float *__restrict__ rw, int *__restrict__ tok_pos) {
    __shared__ int warp_sums[32];
    const int EE = E + n_shared, KK = K + n_shared;
    for (int i = threadIdx.x; i < EE * words; i += blockDim.x)
        bm[i] = 0u;
    __syncthreads();
    // step 1: membership and per-token weight sums
    for (int c = threadIdx.x; c < T; c += blockDim.x) {
        const int *ic = idx + static_cast<size_t>(c) * K;
        const float *wc = wt + static_cast<size_t>(c) * K;
        int ids[KMAX];
        float w[KMAX];
#pragma unroll
        for (int t = 0; t < KMAX; ++t) {
            ids[t] = t < K ? ic[t] : -1;
            w[t] = t < K ? wc[t] : 0.f;
        }
#pragma unroll
        for (int t = 0; t < KMAX; ++t) {
            if (t >= K)
                continue; // (not break: the loop stays fully unrolled, ids / w in registers)
            const int e = ids[t];
            int st = -1;
            if (e >= 0 && e < E) {
                bool dup = false;
#pragma unroll
                for (int t2 = 0; t2 < t; ++t2)
                    dup |= (ids[t2] == e);
                if (!dup) {
                    float sum = 0.f;
#pragma unroll
                    for (int t2 = 0; t2 < KMAX; ++t2)
                        if (t2 < K && ids[t2] == e)
                            sum = __fadd_rn(sum, w[t2]);
                    if (sum != 0.f) {
                        ws[c * KK + t] = sum;
                        st = e;
                        atomicOr(&bm[e * words + (c >> 5)], 1u << (c & 31));
                    }
                }
            }
            tk[c * KK + t] = st;
        }
        if (n_shared) {
            ws[c * KK + K] = 1.f;
            tk[c * KK + K] = E;
            atomicOr(&bm[E * words + (c >> 5)], 1u << (c & 31));
        }
    }
    __syncthreads();
    // step 2: word prefixes and member counts, a thread per expert
    for (int e = threadIdx.x; e < EE; e += blockDim.x) {
        int carry = 0;
        for (int j = 0; j < words; ++j) {
            wp[e * words + j] = carry;
            carry += __popc(bm[e * words + j]);
        }
        nr_s[e] = carry;
        nr[e] = carry;
    }
    __syncthreads();
    // step 3: segment starts in ascending expert id
    int carry = 0;
    for (int e0 = 0; e0 < EE; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const int v = e < EE ? nr_s[e] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, warp_sums, &tot);
        if (e < EE) {
            xoff_s[e] = carry + ex;
            xoff[e] = carry + ex;
        }
        carry += tot;
    }
    if (threadIdx.x == 0)
        *n_rows = carry;
    __syncthreads();
    // step 4: positions; every slot's tok_pos written (-1 where none)
    const int n = T * KK;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = tk[i];
        if (e < 0) {
            tok_pos[i] = -1;
            continue;
        }
        const int c = i / KK;
        const int wi = e * words + (c >> 5);
        const int pos = xoff_s[e] + wp[wi] + __popc(bm[wi] & ((1u << (c & 31)) - 1u));
        rows[pos] = c;
        rw[pos] = ws[i];
        tok_pos[i] = pos;
    }
}

// Shared-memory bytes permute_small_smem_body needs (its arrays, 4 bytes
// each), for the launch's dynamic shared memory.
__host__ __device__ constexpr size_t perm_smem_bytes(int T, int KK, int EE, int words) {
    return (size_t(2) * EE * words + size_t(2) * EE + size_t(2) * T * KK) * 4;
}
constexpr int kPermSmemMaxK = 16;
constexpr size_t kPermSmemMaxBytes = 40 * 1024;

// Decode-sized layer calls (T <= kPermSmallT): the call's error word cleared,
// the permutation, and the expert plan over its counts, in one CTA -- three
// launches and a memset folded into one.  The plan reads nr / xoff that the
// permutation wrote: global memory the CTA's own threads wrote is visible to
// all of them after __syncthreads.
struct PermSmallArgs {
    const int *idx;
    const float *wt;
    int T, K, E, n_shared, words;
    uint32_t *bitmap;
    int *wpre;
    float *wsum;
    int *nr, *xoff, *n_rows, *rows;
    float *rw;
    int *tok_pos;
};

//
// smem != 0 (K <= kPermSmemMaxK, perm_smem_bytes in the launch's dynamic
// shared memory): the permutation keeps what it reads back in shared memory
// and the plan reads the counts and segment starts from there; the experts'
// pointer tables are loaded at the start (one expert per thread when they
// fit) and checked only in the plan, so their latency overlaps the
// permutation.
__global__ void __launch_bounds__(1024) layer_prep_small_kernel(const PermSmallArgs q,
                                                                const PlanArgs a, int smem) {
    extern __shared__ __align__(16) int psm[];
    pdl_wait();
    const bool pre = smem && a.nb <= static_cast<int>(blockDim.x);
    ExpertPtrs ptrs{};
    if (pre && static_cast<int>(threadIdx.x) < a.nb)
        ptrs = expert_ptrs(a, threadIdx.x);
    if (threadIdx.x == 0)
        *a.err = 0;
    if (!smem) {
        permute_small_body(q.idx, q.wt, q.T, q.K, q.E, q.n_shared, q.words, q.bitmap, q.wpre,
                           q.wsum, q.nr, q.xoff, q.n_rows, q.rows, q.rw, q.tok_pos);
        __syncthreads();
        plan_body(a);
        return;
    }
    const int EE = q.E + q.n_shared, KK = q.K + q.n_shared;
    uint32_t *bm = reinterpret_cast<uint32_t *>(psm);
    int *wp = psm + EE * q.words;
    int *nr_s = wp + EE * q.words;
    int *xoff_s = nr_s + EE;
    int *tk = xoff_s + EE;
    float *ws = reinterpret_cast<float *>(tk + q.T * KK);
    permute_small_smem_body<kPermSmemMaxK>(q.idx, q.wt, q.T, q.K, q.E, q.n_shared, q.words, bm,
                                           wp, ws, tk, nr_s, xoff_s, q.nr, q.xoff, q.n_rows,
                                           q.rows, q.rw, q.tok_pos);
    __syncthreads();
    PlanArgs as = a;
    as.nr = nr_s;
    as.xoff = xoff_s;
    plan_body(as, pre ? (static_cast<int>(threadIdx.x) < a.nb ? expert_ptr_bits(a, ptrs) : 0)
                      : -1);
}

// ---------------------------------------------------------------------------
// Rows of the experts' outputs y: f16 on the fast path (the decode and
// tensor-core kernels write them), f32 on the generic path.
__device__ __forceinline__ float4 load_y4(const float *y, size_t i) {
    return __ldcs(reinterpret_cast<const float4 *>(y + i));
}
__device__ __forceinline__ float4 load_y4(const __half *y, size_t i) {
    const uint2 u = __ldcs(reinterpret_cast<const uint2 *>(y + i));
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float load_y1(const float *y, size_t i) { return y[i]; }
__device__ __forceinline__ float load_y1(const __half *y, size_t i) { return __half2float(y[i]); }

// CW consecutive values of a y row (f16 or f32), streamed (read once): the
// raw words, converted to floats where they are added (fewer registers held
// while the loads are in flight).
template <typename TY, int CW> struct YWords;
template <> struct YWords<__half, 8> {
    uint4 u;
    __device__ __forceinline__ void load(const __half *y, size_t i) {
        u = __ldcs(reinterpret_cast<const uint4 *>(y + i));
    }
    __device__ __forceinline__ float get(int q) const {
        const uint32_t w = q < 2 ? u.x : q < 4 ? u.y : q < 6 ? u.z : u.w;
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
        return (q & 1) ? f.y : f.x;
    }
};
template <> struct YWords<__half, 4> {
    uint2 u;
    __device__ __forceinline__ void load(const __half *y, size_t i) {
        u = __ldcs(reinterpret_cast<const uint2 *>(y + i));
    }
    __device__ __forceinline__ float get(int q) const {
        const uint32_t w = q < 2 ? u.x : u.y;
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
        return (q & 1) ? f.y : f.x;
    }
};
template <int CW> struct YWords<float, CW> {
    float4 f[CW / 4];
    __device__ __forceinline__ void load(const float *y, size_t i) {
#pragma unroll
        for (int q = 0; q < CW / 4; ++q)
            f[q] = __ldcs(reinterpret_cast<const float4 *>(y + i) + q);
    }
    __device__ __forceinline__ float get(int q) const {
        const float4 &a = f[q >> 2];
        return (q & 3) == 0 ? a.x : (q & 3) == 1 ? a.y : (q & 3) == 2 ? a.z : a.w;
    }
};

// The token's slot rows spos[0..n) (ascending) in order: acc += w * y, one
// multiply and one add per term.  Up to eight rows' loads are in flight
// before their ordered adds.
template <int CW, typename TY>
__device__ __forceinline__ void ordered_sum(float (&acc)[CW], const TY *__restrict__ y,
                                            const float *__restrict__ rw, const int *spos, int n,
                                            size_t col, int D) {
    constexpr int kB = 8;
    for (int j0 = 0; j0 < n; j0 += kB) {
        YWords<TY, CW> v[kB];
        float w[kB];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            if (j0 + b < n) {
                const int r = spos[j0 + b];
                w[b] = __ldg(rw + r);
                v[b].load(y, static_cast<size_t>(r) * D + col);
            }
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
            if (j0 + b < n) {
#pragma unroll
                for (int q = 0; q < CW; ++q)
                    acc[q] = __fadd_rn(acc[q], __fmul_rn(w[b], v[b].get(q)));
            }
        }
    }
}

// The block's token c: its slot positions (tok_pos row, -1 = no slot) sorted
// ascending into spos[0..n) in shared memory by the first warp (each lane
// places its value by the count of smaller ones; positions are distinct).
// Returns n to every thread.  KK <= 32.
// token_slots_from takes the first warp's tok_pos values loaded by the
// caller (lane < KK: tok_pos[c * KK + lane], else -1), so the load can be
// issued ahead of other loads.
__device__ __forceinline__ int token_slots_from(int p, int KK, int *spos, int *sn) {
    __syncthreads();  // the previous token's readers are done with spos
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const uint32_t valid = __ballot_sync(0xffffffffu, p >= 0);
        int rank = 0;
        for (int u = 0; u < KK; ++u) {
            const int q = __shfl_sync(0xffffffffu, p, u);
            rank += (q >= 0 && q < p) ? 1 : 0;
        }
        if (p >= 0)
            spos[rank] = p;
        if (lane == 0)
            *sn = __popc(valid);
    }
    __syncthreads();
    return *sn;
}
__device__ __forceinline__ int token_slot_load(const int *__restrict__ tok_pos, int c, int KK) {
    return threadIdx.x < static_cast<unsigned>(KK) ? tok_pos[static_cast<size_t>(c) * KK + threadIdx.x]
                                                   : -1;
}
__device__ __forceinline__ int token_slots_shared(const int *__restrict__ tok_pos, int c, int KK,
                                                  int *spos, int *sn) {
    return token_slots_from(token_slot_load(tok_pos, c, KK), KK, spos, sn);
}

// Token-major gather-stage for large calls (fast path, D % 8 == 0, KK <= 32):
// a CTA per token at a time reads the token's row once, converts each
// 8-column chunk once (stage_chunk8) and stores it at every expert-major
// position the permutation gave the token's slots (tok_pos >= 0).  The bytes
// written are those of stage_rows_body over rows[]; x is read once per token
// instead of once per slot, so its reads do not depend on x staying in L2
// while the K-fold larger staged rows stream through it.  A token without a
// slot is neither read nor range-checked, as in the row form.
template <typename TIn>
__global__ void __launch_bounds__(256)
    stage_tokens_f16x8_kernel(const TIn *__restrict__ x, const int *__restrict__ tok_pos, int T,
                              int KK, int D, int fmt, __half *__restrict__ out, int *err) {
    pdl_wait();
    __shared__ int spos[32], sn;
    const int chunks = D >> 3;
    for (int c = blockIdx.x; c < T; c += gridDim.x) {
        const int n = token_slots_shared(tok_pos, c, KK, spos, &sn);
        if (n == 0)
            continue; // uniform over the block
        const TIn *xr = x + static_cast<size_t>(c) * D;
        for (int k = threadIdx.x; k < chunks; k += blockDim.x) {
            bool big = false;
            const uint4 v = stage_chunk8(xr, k, fmt, big);
            if (big)
                set_error(err, MVLLM_ERR_ACT_RANGE);
            for (int j = 0; j < n; ++j)
                reinterpret_cast<uint4 *>(out + static_cast<size_t>(spos[j]) * D)[k] = v;
        }
    }
}

// Ordered combine, layer form: out[c] += wsum*y over the token's segment
// positions in ascending order (= ascending expert id), one multiply and one
// add per term as in glm53.cpp:1978-1984 (no fused multiply-add).  CW
// columns per thread (8 when D is a multiple of 8: 16-byte f16 loads).
template <typename TY, int CW>
__global__ void __launch_bounds__(256, sizeof(TY) == 2 ? 3 : 2)
    combine_tokens_kernel(float *__restrict__ out, const TY *__restrict__ y,
                                      const float *__restrict__ rw,
                                      const int *__restrict__ tok_pos, int T, int KK, int D,
                                      const int *err) {
    pdl_wait();
    // A device-side error in this call (recorded in *err): `out` is left as
    // the caller passed it; mvllm_moe_layer_error reports the code.  The
    // error word, the token's slot positions and the thread's first `out`
    // columns are loaded together, one round trip before the y rows.
    const bool failed = err && load_volatile(err) != 0;
    __shared__ int spos[32], sn;
    const int col0 = (blockIdx.x * blockDim.x + threadIdx.x) * CW;
    for (int c = blockIdx.y; c < T; c += gridDim.y) {
        const int p = token_slot_load(tok_pos, c, KK);
        float first[CW];
        if (col0 < D) {
            const float *o = out + static_cast<size_t>(c) * D + col0;
#pragma unroll
            for (int q = 0; q < CW; q += 4) {
                const float4 a = *reinterpret_cast<const float4 *>(o + q);
                first[q] = a.x, first[q + 1] = a.y, first[q + 2] = a.z, first[q + 3] = a.w;
            }
        }
        if (failed)
            return; // uniform over the grid, before any barrier of this token
        const int n = token_slots_from(p, KK, spos, &sn);
        for (int col = col0; col < D; col += gridDim.x * blockDim.x * CW) {
            float *o = out + static_cast<size_t>(c) * D + col;
            float acc[CW];
            if (col == col0) {
#pragma unroll
                for (int q = 0; q < CW; ++q)
                    acc[q] = first[q];
            } else {
#pragma unroll
                for (int q = 0; q < CW; q += 4) {
                    const float4 a = *reinterpret_cast<const float4 *>(o + q);
                    acc[q] = a.x, acc[q + 1] = a.y, acc[q + 2] = a.z, acc[q + 3] = a.w;
                }
            }
            ordered_sum<CW>(acc, y, rw, spos, n, col, D);
#pragma unroll
            for (int q = 0; q < CW; q += 4)
                *reinterpret_cast<float4 *>(o + q) =
                    make_float4(acc[q], acc[q + 1], acc[q + 2], acc[q + 3]);
        }
    }
}

// Where the partial rows of an expert-parallel rank go when the return is
// fused into their producer: row c of the call (the rank received it from
// rank c / seg as that rank's row c % seg) is stored over NVLink into row
// self * seg + c % seg of the back region of rank (c / seg)'s exchange window.
// win == nullptr: rows stay local, row c of out16.
struct PeerRows {
    uint8_t *const *win;  // device array [nranks] of window bases (own at self)
    size_t back_off;      // byte offset of the back region in every window
    int seg, self;
};

// Partial-sum rows for the expert-parallel return: the sums of
// combine_tokens_kernel taken from zero, stored as f16 of v / 2^s with one
// power-of-two scale per row (the row's largest |v| / 2^s lands in
// [2^14, 2^15), so no value overflows), 2^s as an f32 in the row's 16-byte
// tail.  Row pitch 2*D + 16 bytes; relative error at most 2^-11 per element
// (f16 rounding), half the bytes of f32 rows.  One CTA per token at a time,
// the f32 row staged in shared memory (D floats) for the row maximum.
// With peer.win the rows are stored into the owners' windows (PeerRows);
// rows without a slot on this rank are then not written (their owner reads
// none), and every thread ends with a system-scope fence so that the rows are
// visible to the owners once the kernel has completed.
template <typename TY>
__global__ void combine_tokens_f16_kernel(uint8_t *__restrict__ out16, const TY *__restrict__ y,
                                          const float *__restrict__ rw,
                                          const int *__restrict__ tok_pos, int T, int KK, int D,
                                          const int *err, const PeerRows peer) {
    extern __shared__ float4 srow[];
    // A device-side error in this call (recorded in *err): zero rows (h = 0,
    // scale 0), so the owners add nothing from this rank; the serving rank's
    // mvllm_moe_layer_error reports the code.
    const bool failed = err && load_volatile(err) != 0;
    __shared__ float wmax[32];
    const int n8 = D / 8;
    const size_t pitch = 2 * static_cast<size_t>(D) + 16;
    __shared__ int spos[32], sn;
    for (int c = blockIdx.x; c < T; c += gridDim.x) {
        const int n = token_slots_shared(tok_pos, c, KK, spos, &sn);
        if (peer.win && n == 0)
            continue;  // uniform over the block: every thread read the same slots
        float m = 0.f;
        for (int v = threadIdx.x; v < n8; v += blockDim.x) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            ordered_sum<8>(acc, y, rw, spos, n, 8 * static_cast<size_t>(v), D);
            srow[2 * v] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            srow[2 * v + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
            for (int q = 0; q < 8; ++q)
                m = fmaxf(m, fabsf(acc[q]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31) == 0)
            wmax[threadIdx.x >> 5] = m;
        __syncthreads();
        float M = 0.f;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w)
            M = fmaxf(M, wmax[w]);
        // 2^s: s = floor(log2 M) - 14 for a finite non-zero maximum, else 0
        // (zeros stay zeros; inf / NaN pass through the f16 conversion).
        const int s = (M > 0.f && M <= 3.4e38f) ? ilogbf(M) - 14 : 0;
        const float inv = ldexpf(1.f, -s);
        uint8_t *row = out16 + static_cast<size_t>(c) * pitch;
        if (peer.win) {
            const int o = c / peer.seg, j = c - o * peer.seg;
            row = peer.win[o] + peer.back_off +
                  (static_cast<size_t>(peer.self) * peer.seg + j) * pitch;
        }
        for (int v = threadIdx.x; v < n8; v += blockDim.x) {
            const float4 a = srow[2 * v], b = srow[2 * v + 1];
            __half2 h[4] = {__floats2half2_rn(a.x * inv, a.y * inv),
                            __floats2half2_rn(a.z * inv, a.w * inv),
                            __floats2half2_rn(b.x * inv, b.y * inv),
                            __floats2half2_rn(b.z * inv, b.w * inv)};
            if (failed)
                h[0] = h[1] = h[2] = h[3] = __floats2half2_rn(0.f, 0.f);
            *reinterpret_cast<uint4 *>(row + 16 * static_cast<size_t>(v)) =
                *reinterpret_cast<const uint4 *>(h);
        }
        if (threadIdx.x == 0)
            *reinterpret_cast<float4 *>(row + 2 * static_cast<size_t>(D)) =
                make_float4(failed ? 0.f : ldexpf(1.f, s), 0.f, 0.f, 0.f);
        __syncthreads();
    }
    if (peer.win)
        __threadfence_system();
}

// Ordered combine, moe_block form: CSR of destination rows (row ids ascending
// within each destination), scatter order of metal_ops.cpp:328-339.
template <typename TY>
__global__ void combine_csr_kernel(float *__restrict__ out, const TY *__restrict__ y,
                                   const float *__restrict__ rw, const int *__restrict__ off,
                                   const int *__restrict__ ids, int S, int D) {
    for (int s = blockIdx.y; s < S; s += gridDim.y) {
    const int j0 = off[s], j1 = off[s + 1];
    if (j0 == j1)
        continue;
    for (int col = blockIdx.x * blockDim.x + threadIdx.x; col < D; col += gridDim.x * blockDim.x) {
        float acc = out[static_cast<size_t>(s) * D + col];
        for (int j = j0; j < j1; ++j) {
            const int r = ids[j];
            acc = __fadd_rn(acc, __fmul_rn(rw[r], load_y1(y, static_cast<size_t>(r) * D + col)));
        }
        out[static_cast<size_t>(s) * D + col] = acc;
    }
    }
}

// Device CSR builder for the device-pointer moe_block (one CTA): rows of
// experts that ran (found through base/cnt) with 0 <= dest < S are bucketed
// by destination; buckets are then sorted so row ids ascend.
__global__ void build_csr_kernel(const int *__restrict__ rows, const int *__restrict__ base,
                                 const int *__restrict__ cnt, int nb,
                                 const int *__restrict__ total_rows, int S,
                                 int *__restrict__ hist, int *__restrict__ off,
                                 int *__restrict__ ids) {
    __shared__ int warp_sums[32];
    __shared__ int carry;
    const int R = *total_rows;
    for (int s = threadIdx.x; s < S; s += blockDim.x)
        hist[s] = 0;
    __syncthreads();
    auto valid_dest = [&](int r) -> int {
        // owner expert: largest e with base[e] <= r (it has rows, see plan)
        int lo = 0, hi = nb;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (base[mid] <= r)
                lo = mid;
            else
                hi = mid;
        }
        if (cnt[lo] == 0)
            return -1;
        const int dest = rows[r];
        return (dest >= 0 && dest < S) ? dest : -1;
    };
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int dest = valid_dest(r);
        if (dest >= 0)
            atomicAdd(&hist[dest], 1);
    }
    if (threadIdx.x == 0)
        carry = 0;
    __syncthreads();
    for (int s0 = 0; s0 < S; s0 += blockDim.x) {
        const int s = s0 + threadIdx.x;
        const int v = s < S ? hist[s] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, warp_sums, &tot);
        if (s < S) {
            off[s] = carry + ex;
            hist[s] = carry + ex; // becomes the fill cursor
        }
        __syncthreads();
        if (threadIdx.x == 0)
            carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0)
        off[S] = carry;
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int dest = valid_dest(r);
        if (dest >= 0)
            ids[atomicAdd(&hist[dest], 1)] = r;
    }
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const int j0 = off[s], j1 = off[s + 1];
        for (int j = j0 + 1; j < j1; ++j) {
            const int v = ids[j];
            int k = j;
            while (k > j0 && ids[k - 1] > v) {
                ids[k] = ids[k - 1];
                --k;
            }
            ids[k] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// Generic expert kernels: any D / Iinter, any of fmt 0/4/7, f32 arithmetic.
// Dequantised element (o, k) of a weight matrix with row length K
// (src/quant/quant.cpp:203-228 and :298-321).
// DeepSeek-V4's e4m3fn and e8m0 decoders (native_act.cpp:65-69, 90-100):
// e4m3fn code 0x7f/0xff is NaN, exponent 0 is man * 2^-9, else
// (1 + man/8) * 2^(exp-7); e8m0 255 is NaN and 0 is 2^-127 (unlike the
// MXFP4 scale decoder above, which maps them to inf and 0).  Both exact.
__device__ __forceinline__ float e4m3fn_to_f32(uint32_t v) {
    const uint32_t ex = (v >> 3) & 15u, man = v & 7u;
    if (ex == 15u && man == 7u)
        return __int_as_float(0x7fc00000);
    const float mag = ex == 0u ? __fmul_rn(static_cast<float>(man), 0.001953125f)
                               : __uint_as_float(((ex + 120u) << 23) | (man << 20));
    return (v & 0x80u) ? -mag : mag;
}
__device__ __forceinline__ float e8m0_to_f32(uint32_t e) {
    if (e == 255u)
        return __int_as_float(0x7fc00000);
    return e == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(e << 23);
}

__device__ __forceinline__ float deq_elem(const void *w, const void *s, int fmt, int o, int k,
                                          int K) {
    if (fmt == MVLLM_FMT_F32)
        return static_cast<const float *>(w)[static_cast<size_t>(o) * K + k];
    if (fmt == MVLLM_FMT_FP8_B128) {
        // dsv4_cuda.cpp:127-135: q * scale of the (o / 128, k / 128) tile
        const uint8_t q = static_cast<const uint8_t *>(w)[static_cast<size_t>(o) * K + k];
        const uint8_t e =
            static_cast<const uint8_t *>(s)[static_cast<size_t>(o >> 7) * ((K + 127) / 128) +
                                            (k >> 7)];
        return __fmul_rn(e4m3fn_to_f32(q), e8m0_to_f32(e));
    }
    const uint8_t b = static_cast<const uint8_t *>(w)[static_cast<size_t>(o) * ((K + 1) / 2) +
                                                      (k >> 1)];
    const uint32_t nib = (k & 1) ? (b >> 4) : (b & 15u);
    if (fmt == MVLLM_FMT_INT4_G64) {
        const float sc = static_cast<const float *>(s)[static_cast<size_t>(o) * ((K + 63) / 64) +
                                                       (k >> 6)];
        return static_cast<float>(static_cast<int>(nib) - 8) * sc;
    }
    const uint8_t e = static_cast<const uint8_t *>(s)[static_cast<size_t>(o) * ((K + 31) / 32) +
                                                      (k >> 5)];
    const float mag = (nib & 7u) == 0   ? 0.f
                      : (nib & 7u) == 1 ? 0.5f
                      : (nib & 7u) == 2 ? 1.f
                      : (nib & 7u) == 3 ? 1.5f
                      : (nib & 7u) == 4 ? 2.f
                      : (nib & 7u) == 5 ? 3.f
                      : (nib & 7u) == 6 ? 4.f
                                        : 6.f;
    return ((nib & 8u) ? -mag : mag) * ue8m0_to_f32(e);
}

struct GenericArgs {
    const void *const *w0, *const *w1, *const *s0, *const *s1;
    const int *xrow, *orow, *cnt, *item_off;
    int nb, fmt;
    const float *x; // f32 rows of length K
    int K, O;       // phase 1: K = D, O = Iinter; phase 2: K = Iinter, O = D
    float *out;     // phase 1: h f32 [R, Iinter]; phase 2: y f32 [R, D]
    int act;
    float act_a, act_b;
};

// Item = (expert, 8 output rows); warp w computes row o = 8*blk + w for all
// the expert's tokens, 4 tokens at a time, lanes striding over k.
template <int PHASE> __global__ void __launch_bounds__(256) generic_ffn_kernel(const GenericArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = a.item_off[a.nb];
    for (int i = blockIdx.x; i < total; i += gridDim.x) {
        const int e = find_owner(a.item_off, a.nb, i);
        const int o = (i - a.item_off[e]) * 8 + warp;
        if (o >= a.O)
            continue;
        const int ce = a.cnt[e];
        const float *xe = a.x + static_cast<size_t>(a.xrow[e]) * a.K;
        const size_t ob = static_cast<size_t>(a.orow[e]);
        for (int r0 = 0; r0 < ce; r0 += 4) {
            const int nrr = min(4, ce - r0);
            float g4[4] = {0.f, 0.f, 0.f, 0.f}, u4[4] = {0.f, 0.f, 0.f, 0.f};
            for (int k = lane; k < a.K; k += 32) {
                const float wg = deq_elem(a.w0[e], a.s0 ? a.s0[e] : nullptr, a.fmt, o, k, a.K);
                float wu = 0.f;
                if (PHASE == 1)
                    wu = deq_elem(a.w1[e], a.s1 ? a.s1[e] : nullptr, a.fmt, o, k, a.K);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < nrr) {
                        const float xv = xe[static_cast<size_t>(r0 + j) * a.K + k];
                        g4[j] = fmaf(xv, wg, g4[j]);
                        if (PHASE == 1)
                            u4[j] = fmaf(xv, wu, u4[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int s = 16; s > 0; s >>= 1) {
                    g4[j] += __shfl_xor_sync(0xffffffffu, g4[j], s);
                    if (PHASE == 1)
                        u4[j] += __shfl_xor_sync(0xffffffffu, u4[j], s);
                }
            }
            if (lane == 0) {
                for (int j = 0; j < nrr; ++j) {
                    const float v =
                        (PHASE == 1) ? apply_act(g4[j], u4[j], a.act, a.act_a, a.act_b) : g4[j];
                    a.out[(ob + r0 + j) * a.O + o] = v;
                }
            }
        }
    }
}

// Sequential-order dot products for small row counts, the reference's
// arithmetic per output (quant.cpp:143-156, 203-228, 255-268, 298-321;
// DeepSeek-V4's FP8 tiles, dsv4_cuda.cpp:618-623): acc += x[i] * w[i] in
// ascending i, each product and sum rounded on its own (no contraction),
// w = q * scale as the reference decodes it.  So results are bit-identical
// to the reference's host loops.
//
// A CTA covers 32 rows of x and 4*OT rows of W with 128 threads; thread
// (s, og) = (tid / 4, tid % 4) owns rows og*OT .. og*OT+OT-1 of the tile for
// x row s, so every thread runs OT independent chains.  Each K tile of 64
// is staged in shared memory (x transposed to [k][s], W decoded to f32
// [o][k], both padded against bank conflicts) from coalesced loads, and the
// next tile's global loads are issued into registers before the current
// tile is consumed, so their latency hides behind the chains.  The chains'
// length (I) bounds a launch from below, so the grid spreads over W rows:
// small row counts (decode batches, the router) still fill the SMs.
constexpr int kSeqS = 32;        // x rows per CTA
constexpr int kSeqKt = 64;       // K tile
constexpr int kSeqThreads = 128; // (32 x rows) x (4 W-row groups)

__device__ __forceinline__ float x_to_f32(float v) { return v; }
__device__ __forceinline__ float x_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// One W element as f32 (int8 rows: the raw code; the row scale comes last).
__device__ __forceinline__ float seq_w(const void *w, const void *sc, int fmt, int o, int k,
                                       int I) {
    if (fmt == MVLLM_FMT_INT8_ROW)
        return static_cast<float>(static_cast<const int8_t *>(w)[static_cast<size_t>(o) * I + k]);
    return deq_elem(w, sc, fmt, o, k, I);
}

template <int OT, typename TX>
__device__ __forceinline__ void seq_dot_tile(const TX *__restrict__ x, const void *w,
                                             const void *sc, int fmt, int S, int I, int O,
                                             int s0, int oc, float (&acc)[OT]) {
    constexpr int RO = 4 * OT;                          // W rows per CTA
    constexpr int XPER = kSeqS * kSeqKt / kSeqThreads;  // x values staged per thread
    constexpr int WPER = RO * kSeqKt / kSeqThreads;     // W values staged per thread
    static_assert(WPER >= 1 && (RO * kSeqKt) % kSeqThreads == 0, "tile shape");
    __shared__ float xs[kSeqKt][kSeqS + 1];
    __shared__ float wsm[RO][kSeqKt + 1];
    const int tid = threadIdx.x;
    const int s_loc = tid >> 2, og = tid & 3;
    const int ns = min(kSeqS, S - s0), no = min(RO, O - oc);
    float xr[XPER], wr[WPER];
    auto fetch = [&](int k0) {
        const int kn = min(kSeqKt, I - k0);
#pragma unroll
        for (int i = 0; i < XPER; ++i) {
            const int j = i * kSeqThreads + tid;
            const int s = j / kSeqKt, k = j % kSeqKt;
            xr[i] = (s < ns && k < kn) ? x_to_f32(x[static_cast<size_t>(s0 + s) * I + k0 + k])
                                       : 0.f;
        }
#pragma unroll
        for (int i = 0; i < WPER; ++i) {
            const int j = i * kSeqThreads + tid;
            const int r = j / kSeqKt, k = j % kSeqKt;
            wr[i] = (r < no && k < kn) ? seq_w(w, sc, fmt, oc + r, k0 + k, I) : 0.f;
        }
    };
#pragma unroll
    for (int r = 0; r < OT; ++r)
        acc[r] = 0.f;
    fetch(0);
    for (int k0 = 0; k0 < I; k0 += kSeqKt) {
        const int kn = min(kSeqKt, I - k0);
        __syncthreads(); // the previous tile is consumed
#pragma unroll
        for (int i = 0; i < XPER; ++i) {
            const int j = i * kSeqThreads + tid;
            xs[j % kSeqKt][j / kSeqKt] = xr[i];
        }
#pragma unroll
        for (int i = 0; i < WPER; ++i) {
            const int j = i * kSeqThreads + tid;
            wsm[j / kSeqKt][j % kSeqKt] = wr[i];
        }
        __syncthreads();
        if (k0 + kSeqKt < I)
            fetch(k0 + kSeqKt); // in flight while this tile's chains run
#pragma unroll 4
        for (int kk = 0; kk < kn; ++kk) {
            const float xv = xs[kk][s_loc];
#pragma unroll
            for (int r = 0; r < OT; ++r)
                acc[r] = __fadd_rn(acc[r], __fmul_rn(xv, wsm[og * OT + r][kk]));
        }
    }
}

// The same chains with the operands streamed through a cp.async ring
// (kAsStages chunks of kAsKc in flight per CTA): the per-tile fetch above
// leaves a few KB per CTA in flight, which bounds a weight stream far below
// HBM bandwidth (Little's law); here three chunks of x and of the raw W rows
// are always on their way.  Each landed W chunk is decoded once into f32 in
// shared memory (the decoders of deq_elem), then every thread runs its
// chains over it in ascending k, so results are identical to seq_dot_tile.
// Needs 16-byte aligned x and W and rows that are whole 16-byte pieces
// (seq_async_ok); other shapes take seq_dot_tile.
constexpr int kAsKc = 128;   // K chunk
constexpr int kAsStages = 4; // chunks in the ring

__host__ __device__ constexpr int seq_w_bits(int fmt) {
    return fmt == MVLLM_FMT_F32 ? 32
           : (fmt == MVLLM_FMT_INT8_ROW || fmt == MVLLM_FMT_FP8_B128) ? 8
                                                                      : 4;
}
template <typename TX>
inline bool seq_async_ok(const TX *x, const void *w, int fmt, int I) {
    const long xb = long(I) * static_cast<long>(sizeof(TX));
    const long wbits = long(I) * seq_w_bits(fmt);
    return (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(w) & 15) == 0 && xb % 16 == 0 && wbits % 128 == 0;
}

// RO W rows per CTA, OT of them per thread: 32 * RO / OT threads, thread
// (s, g) = (lane, warp): a warp runs one group of OT rows for all 32 x rows,
// so every W value it reads is one broadcast and the x values of a lane's
// row come four at a time.  Shared memory: the x ring
// [stage][32][Kc + 16 bytes], the raw W ring [stage][RO][row chunk + 16
// bytes] (the pads keep 16-byte alignment and spread rows over the banks)
// and the decoded chunk [Kc][RO] f32.
template <int RO, int OT, int FMT, typename TX> struct SeqAsync {
    static constexpr int G = RO / OT;
    static constexpr int THREADS = kSeqS * G;
    static constexpr int XRB = kAsKc * static_cast<int>(sizeof(TX)) + 16;
    static constexpr int WCB = kAsKc * seq_w_bits(FMT) / 8; // W bytes per row chunk
    static constexpr int WRB = WCB + 16;
    static constexpr int XPC = kAsKc * static_cast<int>(sizeof(TX)) / 16;
    static constexpr int WPC = WCB / 16;
    static constexpr size_t SMEM = size_t(kAsStages) * (kSeqS * XRB + RO * WRB) +
                                   size_t(RO) * kAsKc * sizeof(float);
    __device__ static int s_of(int tid) { return tid & 31; }
    __device__ static int g_of(int tid) { return tid >> 5; }
};

// Four consecutive x values (16-byte aligned for f32, 8-byte for bf16).
__device__ __forceinline__ float4 ld4_x(const float *p) {
    return *reinterpret_cast<const float4 *>(p);
}
__device__ __forceinline__ float4 ld4_x(const __nv_bfloat16 *p) {
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Element kl of a raw W row chunk starting at global column k0 (k0 a
// multiple of kAsKc, so nibble parity is kept), decoded as deq_elem does.
template <int FMT>
__device__ __forceinline__ float seq_deq_raw(const uint8_t *row, int kl, const void *sc, int o,
                                             int k, int I) {
    if constexpr (FMT == MVLLM_FMT_F32) {
        return reinterpret_cast<const float *>(row)[kl];
    } else if constexpr (FMT == MVLLM_FMT_INT8_ROW) {
        return static_cast<float>(static_cast<int8_t>(row[kl]));
    } else if constexpr (FMT == MVLLM_FMT_FP8_B128) {
        const uint8_t e =
            static_cast<const uint8_t *>(sc)[static_cast<size_t>(o >> 7) * ((I + 127) / 128) +
                                             (k >> 7)];
        return __fmul_rn(e4m3fn_to_f32(row[kl]), e8m0_to_f32(e));
    } else {
        const uint8_t b = row[kl >> 1];
        const uint32_t nib = (kl & 1) ? (b >> 4) : (b & 15u);
        if constexpr (FMT == MVLLM_FMT_INT4_G64) {
            const float scv =
                static_cast<const float *>(sc)[static_cast<size_t>(o) * ((I + 63) / 64) + (k >> 6)];
            return static_cast<float>(static_cast<int>(nib) - 8) * scv;
        } else {
            const uint8_t e =
                static_cast<const uint8_t *>(sc)[static_cast<size_t>(o) * ((I + 31) / 32) +
                                                 (k >> 5)];
            const float mag = (nib & 7u) == 0   ? 0.f
                              : (nib & 7u) == 1 ? 0.5f
                              : (nib & 7u) == 2 ? 1.f
                              : (nib & 7u) == 3 ? 1.5f
                              : (nib & 7u) == 4 ? 2.f
                              : (nib & 7u) == 5 ? 3.f
                              : (nib & 7u) == 6 ? 4.f
                                                : 6.f;
            return ((nib & 8u) ? -mag : mag) * ue8m0_to_f32(e);
        }
    }
}

template <int RO, int OT, int FMT, typename TX>
__device__ __forceinline__ void seq_dot_async(const TX *__restrict__ x, const void *w,
                                              const void *sc, int S, int I, int O, int s0,
                                              int oc, float (&acc)[OT], uint8_t *smem) {
    using L = SeqAsync<RO, OT, FMT, TX>;
    uint8_t *xst = smem;                                             // [stage][32][XRB]
    uint8_t *wst = xst + size_t(kAsStages) * kSeqS * L::XRB;         // [stage][RO][WRB]
    float *wsm = reinterpret_cast<float *>(wst + size_t(kAsStages) * RO * L::WRB); // [Kc][RO]
    const int tid = threadIdx.x;
    const int s_loc = L::s_of(tid), og = L::g_of(tid);
    const int ns = min(kSeqS, S - s0), no = min(RO, O - oc);
    const size_t xrow = size_t(I) * sizeof(TX), wrow = size_t(I) * seq_w_bits(FMT) / 8;
    const int nchunks = (I + kAsKc - 1) / kAsKc;
    const uint8_t *xb = reinterpret_cast<const uint8_t *>(x);
    const uint8_t *wbp = static_cast<const uint8_t *>(w);
    auto issue = [&](int c) {
        const int st = c % kAsStages;
        const size_t xk0 = size_t(c) * kAsKc * sizeof(TX), wk0 = size_t(c) * L::WCB;
        for (int p = tid; p < kSeqS * L::XPC; p += L::THREADS) {
            const int srow = p / L::XPC, pc = p % L::XPC;
            const size_t off = xk0 + size_t(pc) * 16;
            const bool ok = srow < ns && off < xrow;
            cp_async16_zfill(xst + (size_t(st) * kSeqS + srow) * L::XRB + pc * 16,
                             ok ? xb + size_t(s0 + srow) * xrow + off : xb, ok ? 16 : 0);
        }
        for (int p = tid; p < RO * L::WPC; p += L::THREADS) {
            const int r = p / L::WPC, pc = p % L::WPC;
            const size_t off = wk0 + size_t(pc) * 16;
            const bool ok = r < no && off < wrow;
            cp_async16_zfill(wst + (size_t(st) * RO + r) * L::WRB + pc * 16,
                             ok ? wbp + size_t(oc + r) * wrow + off : wbp, ok ? 16 : 0);
        }
    };
#pragma unroll
    for (int r = 0; r < OT; ++r)
        acc[r] = 0.f;
#pragma unroll
    for (int c = 0; c < kAsStages - 1; ++c) {
        if (c < nchunks)
            issue(c);
        cp_async_commit();
    }
    for (int c = 0; c < nchunks; ++c) {
        const int st = c % kAsStages;
        const int k0 = c * kAsKc, kn = min(kAsKc, I - k0);
        cp_async_wait<kAsStages - 2>();
        __syncthreads(); // chunk c landed for every thread; chunk c-1 consumed
        // decoded to [k][row]: consecutive threads take consecutive rows
        for (int j = tid; j < RO * kAsKc; j += L::THREADS) {
            const int r = j % RO, kl = j / RO;
            float v = 0.f;
            if (r < no && kl < kn)
                v = seq_deq_raw<FMT>(wst + (size_t(st) * RO + r) * L::WRB, kl, sc, oc + r,
                                     k0 + kl, I);
            wsm[kl * RO + r] = v;
        }
        if (c + kAsStages - 1 < nchunks)
            issue(c + kAsStages - 1);
        cp_async_commit();
        __syncthreads(); // decoded chunk visible
        // kn is a multiple of 4 (whole 16-byte x pieces): x four k at a time,
        // the thread's OT weights of one k in one vector load.
        const TX *xs = reinterpret_cast<const TX *>(xst + (size_t(st) * kSeqS + s_loc) * L::XRB);
        const float *wrow_s = wsm + og * OT;
#pragma unroll 2
        for (int kk = 0; kk < kn; kk += 4) {
            const float4 x4 = ld4_x(xs + kk);
            const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float *wq = wrow_s + (kk + q) * RO;
                float wv[OT];
                if constexpr (OT == 4) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(wq);
                    wv[0] = w4.x;
                    wv[1 % OT] = w4.y;
                    wv[2 % OT] = w4.z;
                    wv[3 % OT] = w4.w;
                } else if constexpr (OT == 2) {
                    const float2 w2 = *reinterpret_cast<const float2 *>(wq);
                    wv[0] = w2.x;
                    wv[1 % OT] = w2.y;
                } else {
#pragma unroll
                    for (int r = 0; r < OT; ++r)
                        wv[r] = wq[r];
                }
#pragma unroll
                for (int r = 0; r < OT; ++r)
                    acc[r] = __fadd_rn(acc[r], __fmul_rn(xv[q], wv[r]));
            }
        }
    }
    cp_async_wait<0>();
}

// Generic dequantised GEMM y[S,O] = x[S,I] . W[O,I]^T (f32), fmt 0 / 4 / 7 /
// 8 / 9, bit-identical to the reference's matmuls; int8 rows (fmt 8) take the
// row scale at the end (quant.cpp:255-268).  16 W rows per CTA: on the
// cp.async ring 2 per thread (256 threads, so eight warps per SM hide the
// chains' latency), otherwise seq_dot_tile's 4 per thread.
constexpr int kMmRO = 16;
constexpr int kMmOT = 2;
// Up to two products over the same x in one launch (blockIdx.z picks one):
// a gated FFN's gate and up projections share the x stream and fill twice
// the CTAs.
struct MmOut {
    float *y[2];
    const void *w[2];
    const void *sc[2];
};
template <int FMT>
__global__ void __launch_bounds__(SeqAsync<kMmRO, kMmOT, FMT, float>::THREADS)
    matmul_async_kernel(const MmOut p, const float *x, int S, int I, int O) {
    using L = SeqAsync<kMmRO, kMmOT, FMT, float>;
    extern __shared__ __align__(16) uint8_t seq_smem[];
    const int z = blockIdx.z;
    const int s0 = blockIdx.y * kSeqS, oc = blockIdx.x * kMmRO;
    float acc[kMmOT];
    seq_dot_async<kMmRO, kMmOT, FMT>(x, p.w[z], p.sc[z], S, I, O, s0, oc, acc, seq_smem);
    const int s = s0 + L::s_of(threadIdx.x);
    if (s < S) {
#pragma unroll
        for (int r = 0; r < kMmOT; ++r) {
            const int o = oc + L::g_of(threadIdx.x) * kMmOT + r;
            if (o < O)
                p.y[z][static_cast<size_t>(s) * O + o] =
                    FMT == MVLLM_FMT_INT8_ROW
                        ? __fmul_rn(acc[r], static_cast<const float *>(p.sc[z])[o])
                        : acc[r];
        }
    }
}
__global__ void __launch_bounds__(kSeqThreads) matmul_generic_kernel(int fmt, const MmOut p,
                                                                     const float *x, int S,
                                                                     int I, int O) {
    const int z = blockIdx.z;
    const int s0 = blockIdx.y * kSeqS, oc = blockIdx.x * kMmRO;
    float acc[4];
    seq_dot_tile<4>(x, p.w[z], p.sc[z], fmt, S, I, O, s0, oc, acc);
    const int s = s0 + (threadIdx.x >> 2);
    if (s < S) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int o = oc + (threadIdx.x & 3) * 4 + r;
            if (o < O)
                p.y[z][static_cast<size_t>(s) * O + o] =
                    fmt == MVLLM_FMT_INT8_ROW
                        ? __fmul_rn(acc[r], static_cast<const float *>(p.sc[z])[o])
                        : acc[r];
        }
    }
}
inline dim3 matmul_grid(int S, int O, int n = 1) {
    return dim3((O + kMmRO - 1) / kMmRO, (S + kSeqS - 1) / kSeqS, n);
}

template <int FMT>
inline cudaError_t matmul_async_launch(cudaStream_t st, const MmOut &p, int n, const float *x,
                                       int S, int I, int O) {
    using L = SeqAsync<kMmRO, kMmOT, FMT, float>;
    const cudaError_t e = cudaFuncSetAttribute(
        matmul_async_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L::SMEM));
    if (e != cudaSuccess)
        return e;
    matmul_async_kernel<FMT><<<matmul_grid(S, O, n), L::THREADS, L::SMEM, st>>>(p, x, S, I, O);
    return cudaGetLastError();
}

// y_j = x . W_j^T for the n (1 or 2) products of p, all of format fmt and
// shape [O, I]: on the cp.async ring where x and every W allow it.
inline cudaError_t matmul_generic_launch(cudaStream_t st, int fmt, const MmOut &p, int n,
                                         const float *x, int S, int I, int O) {
    bool async = true;
    for (int j = 0; j < n; ++j)
        async = async && seq_async_ok(x, p.w[j], fmt, I);
    if (async) {
        switch (fmt) {
        case MVLLM_FMT_F32:
            return matmul_async_launch<MVLLM_FMT_F32>(st, p, n, x, S, I, O);
        case MVLLM_FMT_INT4_G64:
            return matmul_async_launch<MVLLM_FMT_INT4_G64>(st, p, n, x, S, I, O);
        case MVLLM_FMT_MXFP4:
            return matmul_async_launch<MVLLM_FMT_MXFP4>(st, p, n, x, S, I, O);
        case MVLLM_FMT_INT8_ROW:
            return matmul_async_launch<MVLLM_FMT_INT8_ROW>(st, p, n, x, S, I, O);
        case MVLLM_FMT_FP8_B128:
            return matmul_async_launch<MVLLM_FMT_FP8_B128>(st, p, n, x, S, I, O);
        default:
            break;
        }
    }
    matmul_generic_kernel<<<matmul_grid(S, O, n), kSeqThreads, 0, st>>>(fmt, p, x, S, I, O);
    return cudaGetLastError();
}
inline cudaError_t matmul_generic_launch(cudaStream_t st, int fmt, float *y, const float *x,
                                         const void *w, const void *sc, int S, int I, int O) {
    const MmOut p{{y, nullptr}, {w, nullptr}, {sc, nullptr}};
    return matmul_generic_launch(st, fmt, p, 1, x, S, I, O);
}

// rmsnorm per row, exactly as quant.cpp:384-398: the sum of squares in
// ascending order on one thread (each product and sum rounded on its own),
// inv = 1 / sqrt(ss / n + eps) with IEEE division and square root, then
// y = x * inv * w.  One CTA per row; the row is staged in shared memory
// (n floats of dynamic shared memory) so the serial sum reads it at shared
// latency, its squares computed by all threads first.
__global__ void rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                    float *__restrict__ y, int T, int n, float eps) {
    extern __shared__ float sq[];
    __shared__ float inv_s;
    for (int r = blockIdx.x; r < T; r += gridDim.x) {
        const float *xr = x + static_cast<size_t>(r) * n;
        for (int i = threadIdx.x; i < n; i += blockDim.x)
            sq[i] = __fmul_rn(xr[i], xr[i]);
        __syncthreads();
        if (threadIdx.x == 0) {
            float ss = 0.f;
#pragma unroll 8
            for (int i = 0; i < n; ++i)
                ss = __fadd_rn(ss, sq[i]);
            inv_s = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps)));
        }
        __syncthreads();
        const float inv = inv_s;
        float *yr = y + static_cast<size_t>(r) * n;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = __fmul_rn(xr[i], inv);
            yr[i] = w ? __fmul_rn(v, w[i]) : v;
        }
        __syncthreads();
    }
}

// h += u * routed_scale, then h += shared (kimi_k3.cpp:2090-2105,
// glm53.cpp:1997-2026): separate roundings, in that order.
__global__ void epilogue_residual_kernel(float *__restrict__ h, const float *__restrict__ u,
                                         const float *__restrict__ shared, float routed_scale,
                                         size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float v = __fadd_rn(h[i], __fmul_rn(u[i], routed_scale));
        if (shared)
            v = __fadd_rn(v, shared[i]);
        h[i] = v;
    }
}

// ---------------------------------------------------------------------------
// Device weight packers, one thread per (row, group); same arithmetic as the
// reference (IEEE division, roundf = std::round, ties to the lower e2m1 code).
__global__ void quantize_int4_g64_kernel(const float *__restrict__ w, int O, int I,
                                         uint8_t *__restrict__ packed, float *__restrict__ scales) {
    const int ng = (I + 63) / 64, stride = (I + 1) / 2;
    const size_t total = static_cast<size_t>(O) * ng;
    for (size_t id = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; id < total;
         id += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int o = static_cast<int>(id / ng), gidx = static_cast<int>(id % ng);
        const int i0 = gidx * 64, i1 = min(i0 + 64, I);
        const float *row = w + static_cast<size_t>(o) * I;
        float amax = 0.f;
        for (int i = i0; i < i1; ++i) {
            const float a = fabsf(row[i]);
            if (a > amax)
                amax = a;
        }
        float scale = __fdiv_rn(amax, 7.f);
        if (scale < 1e-8f)
            scale = 1e-8f;
        scales[static_cast<size_t>(o) * ng + gidx] = scale;
        const float inv = __fdiv_rn(1.f, scale);
        uint8_t *prow = packed + static_cast<size_t>(o) * stride;
        for (int i = i0; i < i1; i += 2) {
            int q0 = static_cast<int>(roundf(__fmul_rn(row[i], inv)));
            q0 = min(max(q0, -8), 7);
            int q1 = 0;
            uint32_t hi = 0;
            if (i + 1 < i1) {
                q1 = static_cast<int>(roundf(__fmul_rn(row[i + 1], inv)));
                q1 = min(max(q1, -8), 7);
                hi = static_cast<uint32_t>(q1 + 8);
            }
            prow[i >> 1] = static_cast<uint8_t>(static_cast<uint32_t>(q0 + 8) | (hi << 4));
        }
    }
}

__device__ __forceinline__ uint32_t ue8m0_cover_dev(float need) {
    // src/quant/quant.cpp:47-77
    if (!(need > 0.f))
        return 0;
    if (!isfinite(need))
        return 255;
    const uint32_t bits = __float_as_uint(need);
    const int exp_field = static_cast<int>((bits >> 23) & 0xffu);
    const uint32_t frac = bits & 0x7fffffu;
    int e;
    if (exp_field == 0)
        e = 1;
    else if (exp_field == 255)
        e = 255;
    else
        e = (frac == 0) ? exp_field : exp_field + 1;
    e = min(max(e, 0), 255);
    while (e < 255 && ue8m0_to_f32(static_cast<uint32_t>(e)) < need)
        ++e;
    while (e > 0 && ue8m0_to_f32(static_cast<uint32_t>(e - 1)) >= need)
        --e;
    return static_cast<uint32_t>(e);
}

__device__ __forceinline__ uint32_t closest_mx4_dev(float w, float scale) {
    // src/quant/quant.cpp:79-96
    const float lut[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    float target = 0.f;
    if (scale > 0.f && isfinite(scale))
        target = __fdiv_rn(w, scale);
    const float a = fabsf(target);
    int best = 0;
    float best_d = fabsf(lut[0] - a);
#pragma unroll
    for (int k = 1; k < 8; ++k) {
        const float d = fabsf(__fsub_rn(lut[k], a));
        if (d < best_d) {
            best_d = d;
            best = k;
        }
    }
    if (signbit(w))
        best |= 8;
    return static_cast<uint32_t>(best);
}

__global__ void pack_mxfp4_kernel(const float *__restrict__ w, int O, int I,
                                  uint8_t *__restrict__ packed, uint8_t *__restrict__ scales) {
    const int ng = (I + 31) / 32, stride = (I + 1) / 2;
    const size_t total = static_cast<size_t>(O) * ng;
    for (size_t id = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; id < total;
         id += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int o = static_cast<int>(id / ng), gidx = static_cast<int>(id % ng);
        const int i0 = gidx * 32, i1 = min(i0 + 32, I);
        const float *row = w + static_cast<size_t>(o) * I;
        float amax = 0.f;
        for (int i = i0; i < i1; ++i) {
            const float a = fabsf(row[i]);
            if (a > amax)
                amax = a;
        }
        const uint32_t e = ue8m0_cover_dev(__fdiv_rn(amax, 6.f));
        scales[static_cast<size_t>(o) * ng + gidx] = static_cast<uint8_t>(e);
        const float scale = ue8m0_to_f32(e);
        uint8_t *prow = packed + static_cast<size_t>(o) * stride;
        for (int i = i0; i < i1; i += 2) {
            const uint32_t lo = closest_mx4_dev(row[i], scale);
            const uint32_t hi = (i + 1 < i1) ? closest_mx4_dev(row[i + 1], scale) : 0u;
            prow[i >> 1] = static_cast<uint8_t>(lo | (hi << 4));
        }
    }
}

} // namespace mvb
