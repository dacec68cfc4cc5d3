// decode_ffn.cuh -- weight-streaming expert FFN for the small-M (decode) regime.
//
// Replaces the three quant::matmul_* calls of cpu_moe_block
// (src/gpu/metal_ops.cpp:308-327) for fmt 4 (int4-g64) and fmt 7 (MXFP4).
// Two persistent launches per moe_block:
//   phase 1: item = (expert, 32 gate rows + the matching 32 up rows, chunk of
//            <= 8*NT tokens) -> h = act(gate, up), f16, written straight into
//            the operand layout phase 2 reads;
//   phase 2: item = (expert, 64 down rows, chunk) -> y, f32.
// Within a CTA one producer warp streams each item's weight rows, K-slice by
// K-slice, into a ring of shared-memory stages with cp.async.bulk (TMA,
// 16-byte aligned, no multicast), together with the matching slice of the
// token operand rows.  Eight consumer warps dequantise the packed nibbles in
// registers (cvt.rn.f16x2.e2m1x2, or a magic-number int4 decode) and feed
// mma.m16n8k16 with f32 accumulation.  Each MMA covers 16 columns of ONE
// quantisation group, so the group scale is applied in f32 to the MMA result
// (acc += tmp * scale): no scale is ever folded into an f16 value.
//
// Per weight row a lane owns 4 bytes of each group: rows R0 = mb*16 + g and
// R1 = R0 + 8 (g = lane/4) and word t = lane%4 of the group, which is exactly
// the m16n8k16 A-fragment shape once the group's columns are assigned to
// k-slots in the order produced by the nibble decoder.  The token operand is
// stored in that same column order (stage_pos in common.cuh), so one 16-byte
// shared load gives a lane both B fragments of a 32-column MXFP4 group.
#pragma once

#include "common.cuh"

namespace mvb {

constexpr int kDecodeRows = 64;                     // weight rows per item
constexpr int kDecodeConsumerWarps = 8;             // 4 row blocks x 2 K halves
constexpr int kDecodeThreads = (kDecodeConsumerWarps + 1) * 32;

struct DecodeArgs {
    const void *const *w0; // phase 1: gate pointers; phase 2: down pointers  [nb]
    const void *const *w1; // phase 1: up pointers                            [nb]
    const void *const *s0; // matching scale pointers                        [nb]
    const void *const *s1;
    const int *xrow;     // first operand row of each expert                 [nb]
    const int *orow;     // first output row of each expert (reference base) [nb]
    const int *cnt;      // rows of each expert (0 when skipped)             [nb]
    const int *item_off; // exclusive prefix of items per expert             [nb+1]
    int nb;
    const __half *x;     // operand rows, K f16 each, stage_pos column order
    int K;               // reduction length (phase 1: D, phase 2: Iinter)
    int O;               // output row length (phase 1: Iinter, phase 2: D)
    void *out;           // phase 1: __half h [R, Iinter]; phase 2: float y [R, D]
    int act;
    float act_a, act_b;
    int nstages;
    int *err;
};

template <int KS, int NT> struct DecodeLayout {
    static constexpr int MT = 8 * NT;
    static constexpr int WROW = KS + 16;     // +16 B: conflict-free A-fragment loads
    static constexpr int XROW = 4 * KS + 64; // 2*KS f16 per row, +64 B for LDS.128
    static constexpr int RS = MT + 1;        // reduction row stride (floats)
    static constexpr int RED_BYTES = 2 * kDecodeRows * RS * 4;
    static constexpr int BAR_BYTES = 128;    // up to 8 full + 8 empty barriers
    static constexpr int STAGE_BYTES = ((kDecodeRows * WROW + MT * XROW) + 127) / 128 * 128;
    static constexpr int HEAD_BYTES = (BAR_BYTES + RED_BYTES + 127) / 128 * 128;
    static int smem_bytes(int nstages) { return HEAD_BYTES + nstages * STAGE_BYTES + 128; }
};

template <int FMT, int KS> struct StageScales {
    // MXFP4: KS/32 ue8m0 bytes per row; int4: KS/64 f32 per row.
    static constexpr int WORDS = (FMT == MVLLM_FMT_MXFP4) ? (KS / 32) / 4 : (KS / 64);
    uint32_t r0[WORDS], r1[WORDS];
};

template <int FMT, int KS>
__device__ __forceinline__ void load_stage_scales(StageScales<FMT, KS> &sc, const void *srow0,
                                                  const void *srow1, int kbase) {
    // kbase = first column (element index) of this warp's part of the stage.
    if constexpr (FMT == MVLLM_FMT_MXFP4) {
        const uint8_t *p0 = static_cast<const uint8_t *>(srow0) + kbase / 32;
        const uint8_t *p1 = static_cast<const uint8_t *>(srow1) + kbase / 32;
#pragma unroll
        for (int w = 0; w < StageScales<FMT, KS>::WORDS; w += 4) {
            if constexpr (StageScales<FMT, KS>::WORDS >= 4) {
                const uint4 a = ldg_stream128(p0 + 4 * w), b = ldg_stream128(p1 + 4 * w);
                sc.r0[w] = a.x, sc.r0[w + 1] = a.y, sc.r0[w + 2] = a.z, sc.r0[w + 3] = a.w;
                sc.r1[w] = b.x, sc.r1[w + 1] = b.y, sc.r1[w + 2] = b.z, sc.r1[w + 3] = b.w;
            }
        }
        if constexpr (StageScales<FMT, KS>::WORDS == 2) {
            const uint2 a = __ldg(reinterpret_cast<const uint2 *>(p0));
            const uint2 b = __ldg(reinterpret_cast<const uint2 *>(p1));
            sc.r0[0] = a.x, sc.r0[1] = a.y, sc.r1[0] = b.x, sc.r1[1] = b.y;
        }
    } else {
        const float *p0 = static_cast<const float *>(srow0) + kbase / 64;
        const float *p1 = static_cast<const float *>(srow1) + kbase / 64;
#pragma unroll
        for (int w = 0; w < StageScales<FMT, KS>::WORDS; w += 4) {
            const uint4 a = ldg_stream128(p0 + w), b = ldg_stream128(p1 + w);
            sc.r0[w] = a.x, sc.r0[w + 1] = a.y, sc.r0[w + 2] = a.z, sc.r0[w + 3] = a.w;
            sc.r1[w] = b.x, sc.r1[w + 1] = b.y, sc.r1[w + 2] = b.z, sc.r1[w + 3] = b.w;
        }
    }
}

template <int FMT, int KS, int NT>
__device__ __forceinline__ void decode_stage_compute(uint32_t wrow0, uint32_t xaddr,
                                                     const StageScales<FMT, KS> &sc,
                                                     float (&acc)[NT][4], int nt_active) {
    using L = DecodeLayout<KS, NT>;
    const uint32_t wrow1 = wrow0 + 8 * L::WROW;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (FMT == MVLLM_FMT_MXFP4) {
        constexpr int NG = KS / 32; // 16-byte groups in this warp's half of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint32_t w0 = lds32(wrow0 + j * 16), w1 = lds32(wrow1 + j * 16);
            uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
            e2m1x8_to_f16x8(w0, p0, p1, p2, p3);
            e2m1x8_to_f16x8(w1, q0, q1, q2, q3);
            const float s0 = ue8m0_to_f32((sc.r0[j >> 2] >> (8 * (j & 3))) & 0xffu);
            const float s1 = ue8m0_to_f32((sc.r1[j >> 2] >> (8 * (j & 3))) & 0xffu);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (nt < nt_active) {
                    const uint4 xb = lds128(xaddr + nt * 8 * L::XROW + j * 64);
                    float tmp[4];
                    mma_f16_16816(tmp, p0, q0, p1, q1, xb.x, xb.y, zero);
                    mma_f16_16816(tmp, p2, q2, p3, q3, xb.z, xb.w, tmp);
                    acc[nt][0] = fmaf(tmp[0], s0, acc[nt][0]);
                    acc[nt][1] = fmaf(tmp[1], s0, acc[nt][1]);
                    acc[nt][2] = fmaf(tmp[2], s1, acc[nt][2]);
                    acc[nt][3] = fmaf(tmp[3], s1, acc[nt][3]);
                }
            }
        }
    } else {
        constexpr int NG = KS / 64; // 32-byte groups in this warp's half of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint32_t w0a = lds32(wrow0 + j * 32), w0b = lds32(wrow0 + j * 32 + 16);
            const uint32_t w1a = lds32(wrow1 + j * 32), w1b = lds32(wrow1 + j * 32 + 16);
            uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
            uint32_t u0, u1, u2, u3, v0, v1, v2, v3;
            int4x8_to_f16x8(w0a, p0, p1, p2, p3);
            int4x8_to_f16x8(w1a, q0, q1, q2, q3);
            int4x8_to_f16x8(w0b, u0, u1, u2, u3);
            int4x8_to_f16x8(w1b, v0, v1, v2, v3);
            const float s0 = __uint_as_float(sc.r0[j]);
            const float s1 = __uint_as_float(sc.r1[j]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (nt < nt_active) {
                    const uint32_t xa = xaddr + nt * 8 * L::XROW + j * 128;
                    const uint4 xl = lds128(xa), xh = lds128(xa + 64);
                    float tmp[4];
                    mma_f16_16816(tmp, p0, q0, p1, q1, xl.x, xl.y, zero);
                    mma_f16_16816(tmp, p2, q2, p3, q3, xl.z, xl.w, tmp);
                    mma_f16_16816(tmp, u0, v0, u1, v1, xh.x, xh.y, tmp);
                    mma_f16_16816(tmp, u2, v2, u3, v3, xh.z, xh.w, tmp);
                    acc[nt][0] = fmaf(tmp[0], s0, acc[nt][0]);
                    acc[nt][1] = fmaf(tmp[1], s0, acc[nt][1]);
                    acc[nt][2] = fmaf(tmp[2], s1, acc[nt][2]);
                    acc[nt][3] = fmaf(tmp[3], s1, acc[nt][3]);
                }
            }
        }
    }
}

template <int FMT, int PHASE, int KS, int NT>
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_ffn_kernel(const DecodeArgs p) {
    using L = DecodeLayout<KS, NT>;
    constexpr int MT = L::MT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                                ~uintptr_t(127));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 8;
    float *red = reinterpret_cast<float *>(smem + L::BAR_BYTES);
    uint8_t *stages = smem + L::HEAD_BYTES;

    const int NS = p.nstages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDecodeConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int total = __ldg(p.item_off + p.nb);
    const int nks = (p.K / 2) / KS; // K-slices per item
    const size_t rowbytes = static_cast<size_t>(p.K) / 2;

    if (warp == kDecodeConsumerWarps) {
        // ------------------------------ producer ------------------------------
        const uint64_t pol_w = policy_evict_first(); // weights: read once per step
        const uint64_t pol_x = policy_evict_last();  // operand rows: re-read per item
        uint32_t it = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
            const int e = find_owner(p.item_off, p.nb, i);
            const int local = i - __ldg(p.item_off + e);
            const int ce = __ldg(p.cnt + e);
            const int chunks = (ce + MT - 1) / MT;
            const int rb = local / chunks, chunk = local - rb * chunks;
            const int n0 = chunk * MT, nv = min(MT, ce - n0);
            const uint8_t *wb0 = static_cast<const uint8_t *>(p.w0[e]);
            const uint8_t *wb1 = (PHASE == 1) ? static_cast<const uint8_t *>(p.w1[e]) : nullptr;
            const __half *xb = p.x + static_cast<size_t>(__ldg(p.xrow + e) + n0) * p.K;
            for (int ks = 0; ks < nks; ++ks, ++it) {
                const int slot = it % NS;
                const uint32_t par = (it / NS) & 1u;
                if (!mbar_wait(&empty[slot], par ^ 1u, p.err)) {
                    ok = false;
                    break;
                }
                if (lane == 0)
                    mbar_arrive_expect_tx(&full[slot], kDecodeRows * KS + nv * 4 * KS);
                __syncwarp();
                uint8_t *sw = stages + slot * L::STAGE_BYTES;
                uint8_t *sx = sw + kDecodeRows * L::WROW;
#pragma unroll
                for (int rr = 0; rr < kDecodeRows / 32; ++rr) {
                    const int r = lane + 32 * rr;
                    const uint8_t *src;
                    if (PHASE == 1)
                        src = (r < 32) ? wb0 + static_cast<size_t>(rb * 32 + r) * rowbytes
                                       : wb1 + static_cast<size_t>(rb * 32 + r - 32) * rowbytes;
                    else
                        src = wb0 + static_cast<size_t>(rb * 64 + r) * rowbytes;
                    bulk_g2s(sw + r * L::WROW, src + static_cast<size_t>(ks) * KS, KS,
                             &full[slot], pol_w);
                }
                if (lane < nv)
                    bulk_g2s(sx + lane * L::XROW,
                             xb + static_cast<size_t>(lane) * p.K + static_cast<size_t>(ks) * 2 * KS,
                             4 * KS, &full[slot], pol_x);
            }
        }
        // Drain: no copy may still be in flight when this warp leaves, also
        // on the error path (bounded wait that ignores the error word).
        const uint32_t first = it > static_cast<uint32_t>(NS) ? it - NS : 0u;
        for (uint32_t j = first; j < it; ++j)
            mbar_wait(&full[j % NS], (j / NS) & 1u, nullptr);
        return;
    }

    // ------------------------------- consumers --------------------------------
    const int mb = warp & 3, kp = warp >> 2;
    const int g = lane >> 2, t = lane & 3;
    const int R0 = mb * 16 + g, R1 = R0 + 8;
    const int tid = threadIdx.x; // 0..255
    uint32_t it = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < total; i += gridDim.x) {
        const int e = find_owner(p.item_off, p.nb, i);
        const int local = i - __ldg(p.item_off + e);
        const int ce = __ldg(p.cnt + e);
        const int chunks = (ce + MT - 1) / MT;
        const int rb = local / chunks, chunk = local - rb * chunks;
        const int n0 = chunk * MT, nv = min(MT, ce - n0);
        const int nt_active = (nv + 7) >> 3;

        // Scale rows of this lane's two weight rows.
        const void *srow0, *srow1;
        {
            const size_t sstride = (FMT == MVLLM_FMT_MXFP4) ? static_cast<size_t>(p.K) / 32
                                                            : static_cast<size_t>(p.K) / 64 * 4;
            auto srow = [&](int r) -> const void * {
                const uint8_t *base;
                int grow;
                if (PHASE == 1) {
                    base = static_cast<const uint8_t *>(r < 32 ? p.s0[e] : p.s1[e]);
                    grow = rb * 32 + (r & 31);
                } else {
                    base = static_cast<const uint8_t *>(p.s0[e]);
                    grow = rb * 64 + r;
                }
                return base + static_cast<size_t>(grow) * sstride;
            };
            srow0 = srow(R0);
            srow1 = srow(R1);
        }

        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

        StageScales<FMT, KS> sc_next;
        load_stage_scales<FMT, KS>(sc_next, srow0, srow1, kp * KS);
        for (int ks = 0; ks < nks; ++ks, ++it) {
            const StageScales<FMT, KS> sc = sc_next;
            if (ks + 1 < nks)
                load_stage_scales<FMT, KS>(sc_next, srow0, srow1, (ks + 1) * 2 * KS + kp * KS);
            const int slot = it % NS;
            const uint32_t par = (it / NS) & 1u;
            if (ok && !mbar_wait(&full[slot], par, p.err))
                ok = false;
            if (ok) {
                uint8_t *sw = stages + slot * L::STAGE_BYTES;
                const uint32_t wrow0 = smem_u32(sw) + R0 * L::WROW + kp * (KS / 2) + t * 4;
                const uint32_t xaddr = smem_u32(sw + kDecodeRows * L::WROW) + g * L::XROW +
                                       (kp * KS + t * 8) * 2;
                decode_stage_compute<FMT, KS, NT>(wrow0, xaddr, sc, acc, nt_active);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }

        // Epilogue: reduce the two K halves through shared memory.
        named_sync(1, 256);
        if (ok) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (nt < nt_active) {
                    float *r0 = red + (kp * kDecodeRows + R0) * L::RS + nt * 8 + 2 * t;
                    float *r1 = red + (kp * kDecodeRows + R1) * L::RS + nt * 8 + 2 * t;
                    r0[0] = acc[nt][0];
                    r0[1] = acc[nt][1];
                    r1[0] = acc[nt][2];
                    r1[1] = acc[nt][3];
                }
            }
        }
        named_sync(1, 256);
        if (ok) {
            const size_t orow0 = static_cast<size_t>(__ldg(p.orow + e) + n0);
            if (PHASE == 1) {
                __half *h = static_cast<__half *>(p.out);
                for (int idx = tid; idx < 32 * nv; idx += 256) {
                    const int f = idx & 31, n = idx >> 5;
                    const float gt = red[f * L::RS + n] + red[(kDecodeRows + f) * L::RS + n];
                    const float up =
                        red[(32 + f) * L::RS + n] + red[(kDecodeRows + 32 + f) * L::RS + n];
                    const float hv = apply_act(gt, up, p.act, p.act_a, p.act_b);
                    h[(orow0 + n) * p.O + stage_pos(rb * 32 + f, FMT)] = __float2half_rn(hv);
                }
            } else {
                float *y = static_cast<float *>(p.out);
                for (int idx = tid; idx < kDecodeRows * nv; idx += 256) {
                    const int r = idx & 63, n = idx >> 6;
                    y[(orow0 + n) * p.O + rb * 64 + r] =
                        red[r * L::RS + n] + red[(kDecodeRows + r) * L::RS + n];
                }
            }
        }
    }
}

} // namespace mvb
