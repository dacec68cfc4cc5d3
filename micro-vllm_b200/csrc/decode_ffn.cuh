// decode_ffn.cuh -- weight-streaming expert FFN for the small-M (decode) regime.
//
// Replaces the three quant::matmul_* calls of cpu_moe_block
// (src/gpu/metal_ops.cpp:308-327) for fmt 4 (int4-g64) and fmt 7 (MXFP4).
// Two persistent launches per moe_block:
//   phase 1: item = (expert, 32 gate rows + the matching 32 up rows, chunk of
//            <= 8*NT tokens) -> h = act(gate, up), f16, written straight into
//            the operand layout phase 2 reads;
//   phase 2: item = (expert, 64 down rows, chunk) -> y, f32.
//
// CTA = 1 producer warp + 16 consumer warps (4 row blocks x 4 K quarters of a
// stage, 4 warps per scheduler).  Each stage of the shared-memory ring holds
// one K-slice of an item: its 64 weight rows, the slice's scale bytes, an
// item header and the matching slice of the item's token rows.  The producer
// warp resolves items (prefix sums kept in shared memory, expert tensor maps
// fetched one item ahead) and fills stages:
//   * weight rows as 2-D tensor-TMA boxes of 32/64 rows x 128 bytes with the
//     128-byte swizzle (cp.async.bulk.tensor, never multicast): a handful of
//     8 KB copies per stage instead of one copy per row, which is what lets
//     the stream reach HBM speed (per-copy issue cost dominates small
//     copies);
//   * scale bytes as one dense tensor box per matrix;
//   * token rows with cp.async.bulk (2 KB each);
//   * the header with a plain shared store released by lane 0's arrival.
// All completions are mbarrier tx bytes.  Consumer warps issue no global loads
// at all: they wait on the
// stage, decode nibbles in registers (cvt.rn.f16x2.e2m1x2, or a magic-number
// int4 decode) and run mma.m16n8k16 (f16 x f16 -> f32).  Each MMA covers 16
// columns of ONE quantisation group, so the group scale is applied in f32 to
// the MMA result (acc += tmp * scale): no scale is ever folded into f16.
//
// Lane (g = lane/4, t = lane%4) owns weight rows R0 = 16*mb + g and R0 + 8 and
// word t of each group: exactly the m16n8k16 A-fragment once a group's
// columns are assigned to k-slots in the decoder's pair order.  The token
// operand is stored in that column order (stage_pos in common.cuh), so one
// 16-byte shared load gives a lane both B fragments of a 32-column group.
#pragma once

#include "common.cuh"

namespace mvb {

constexpr int kDecodeRows = 64;                          // weight rows per item
constexpr int kDecodeKParts = 4;                         // K quarters of a stage
constexpr int kDecodeConsumerWarps = 4 * kDecodeKParts;  // 4 row blocks x 4 K parts
constexpr int kDecodeConsumers = kDecodeConsumerWarps * 32;
constexpr int kDecodeThreads = kDecodeConsumers + 32;
constexpr int kDecodeSmemExperts = 512; // expert tables mirrored in shared memory

// Per-expert tensor maps (128 bytes each), built on the device from the
// expert pointer tables: packed gate, up, down rows, then their scales.
enum { kTmGateP = 0, kTmUpP, kTmDownP, kTmGateS, kTmUpS, kTmDownS, kTmCount };
constexpr int kTmBytes = 128;

struct DecodeArgs {
    const uint8_t *tmaps; // [nb][kTmCount] tensor maps
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

template <int FMT, int KS, int NT> struct DecodeLayout {
    static constexpr int MT = 8 * NT;
    static constexpr int SB = (FMT == MVLLM_FMT_MXFP4) ? KS / 16 : KS / 8; // scale bytes/row
    static constexpr int NBOX = KS / 128;    // 128-byte swizzled column boxes per stage
    static constexpr int BOX_BYTES = kDecodeRows * 128;
    static constexpr int XROW = 4 * KS + 64; // 2*KS f16 per row, +64 B for LDS.128
    static constexpr int RS = MT + 1;        // reduction row stride (floats)
    static constexpr int RED_BYTES = kDecodeKParts * kDecodeRows * RS * 4;
    static constexpr int BAR_BYTES = 128;    // up to 8 full + 8 empty barriers
    static constexpr int TAB_BYTES = 2 * (kDecodeSmemExperts + 1) * 4;
    static constexpr int OFF_W = 0;          // 1024-aligned: the 128-byte swizzle needs it
    static constexpr int OFF_SC = OFF_W + NBOX * BOX_BYTES;
    static constexpr int OFF_HDR = OFF_SC + kDecodeRows * SB;
    static constexpr int OFF_X = OFF_HDR + 16;
    static constexpr int STAGE_BYTES = (OFF_X + MT * XROW + 1023) / 1024 * 1024;
    static constexpr int HEAD_BYTES = (BAR_BYTES + TAB_BYTES + RED_BYTES + 1023) / 1024 * 1024;
    static int smem_bytes(int nstages) { return HEAD_BYTES + nstages * STAGE_BYTES + 1024; }
};

// Shared address of byte b (multiple of 4) of stage row R in the swizzled
// weight boxes: box b/128, 16-byte chunk ((b/16) % 8) XOR (R % 8).
__device__ __forceinline__ uint32_t swz_addr(uint32_t wbase, int R, int b) {
    return wbase + (b >> 7) * (kDecodeRows * 128) + R * 128 +
           ((((b >> 4) & 7) ^ (R & 7)) << 4) + (b & 15);
}

template <int FMT, int KS> struct StageScales {
    // A warp covers KS/2 columns of a stage: MXFP4 KS/64 ue8m0 bytes per row,
    // int4 KS/128 f32 per row.
    static constexpr int WORDS = (FMT == MVLLM_FMT_MXFP4) ? (KS / 256) : (KS / 128);
    uint32_t r0[WORDS], r1[WORDS];
};

template <int FMT, int KS>
__device__ __forceinline__ void lds_scales(StageScales<FMT, KS> &sc, uint32_t a0, uint32_t a1) {
    constexpr int W = StageScales<FMT, KS>::WORDS;
    if constexpr (W == 1) {
        sc.r0[0] = lds32(a0);
        sc.r1[0] = lds32(a1);
    } else if constexpr (W == 2) {
        const uint2 x = lds64(a0), y = lds64(a1);
        sc.r0[0] = x.x, sc.r0[1] = x.y, sc.r1[0] = y.x, sc.r1[1] = y.y;
    } else {
        const uint4 x = lds128(a0), y = lds128(a1);
        sc.r0[0] = x.x, sc.r0[1] = x.y, sc.r0[2] = x.z, sc.r0[3] = x.w;
        sc.r1[0] = y.x, sc.r1[1] = y.y, sc.r1[2] = y.z, sc.r1[3] = y.w;
    }
}

// wbase: shared address of the stage's weight boxes; R0: this lane's first
// row (R0 + 8 is the second, same swizzle phase); b0: byte offset of this
// warp's quarter plus 4*t.
template <int FMT, int KS, int NT>
__device__ __forceinline__ void decode_stage_compute(uint32_t wbase, int R0, int b0,
                                                     uint32_t xaddr,
                                                     const StageScales<FMT, KS> &sc,
                                                     float (&acc)[NT][4], int nt_active) {
    using L = DecodeLayout<FMT, KS, NT>;
    constexpr uint32_t kRow8 = 8 * 128; // rows R0 and R0 + 8 share the swizzle phase
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (FMT == MVLLM_FMT_MXFP4) {
        constexpr int NG = KS / 64; // 16-byte groups in this warp's quarter of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint32_t a0 = swz_addr(wbase, R0, b0 + j * 16);
            const uint32_t w0 = lds32(a0), w1 = lds32(a0 + kRow8);
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
        constexpr int NG = KS / 128; // 32-byte groups in this warp's quarter of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint32_t aa = swz_addr(wbase, R0, b0 + j * 32);
            const uint32_t ab = swz_addr(wbase, R0, b0 + j * 32 + 16);
            const uint32_t w0a = lds32(aa), w0b = lds32(ab);
            const uint32_t w1a = lds32(aa + kRow8), w1b = lds32(ab + kRow8);
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

// What the producer knows about one item.
struct DecodeItem {
    const uint8_t *tm; // the expert's kTmCount tensor maps
    const __half *x;   // first operand row of the item's token chunk
    int rb, nv, orow0;
};

template <int NT>
__device__ __forceinline__ DecodeItem resolve_item(const DecodeArgs &p, const int *s_off,
                                                   const int *s_cnt, bool tab_in_smem, int i) {
    constexpr int MT = 8 * NT;
    int e, local, ce;
    if (tab_in_smem) {
        int lo = 0, hi = p.nb; // largest e with off[e] <= i
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_off[mid] <= i)
                lo = mid;
            else
                hi = mid;
        }
        e = lo;
        local = i - s_off[e];
        ce = s_cnt[e];
    } else {
        e = find_owner(p.item_off, p.nb, i);
        local = i - __ldg(p.item_off + e);
        ce = __ldg(p.cnt + e);
    }
    const int chunks = (ce + MT - 1) / MT;
    const int rb = local / chunks, chunk = local - rb * chunks;
    const int n0 = chunk * MT;
    DecodeItem it;
    it.rb = rb;
    it.nv = min(MT, ce - n0);
    it.tm = p.tmaps + static_cast<size_t>(e) * kTmCount * kTmBytes;
    it.x = p.x + static_cast<size_t>(__ldg(p.xrow + e) + n0) * p.K;
    it.orow0 = __ldg(p.orow + e) + n0;
    return it;
}

template <int FMT, int PHASE, int KS, int NT>
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_ffn_kernel(const DecodeArgs p) {
    static_assert(KS == 256 || KS == 512, "stage K-slice");
    using L = DecodeLayout<FMT, KS, NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 8;
    int *s_off = reinterpret_cast<int *>(smem + L::BAR_BYTES);
    int *s_cnt = s_off + kDecodeSmemExperts + 1;
    float *red = reinterpret_cast<float *>(smem + L::BAR_BYTES + L::TAB_BYTES);
    uint8_t *stages = smem + L::HEAD_BYTES;

    const int NS = p.nstages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool tab_in_smem = p.nb <= kDecodeSmemExperts;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1); // producer's expect_tx arrival; the rest is tx bytes
            mbar_init(&empty[s], kDecodeConsumerWarps);
        }
        fence_barrier_init();
    }
    if (tab_in_smem)
        for (int e = threadIdx.x; e <= p.nb; e += blockDim.x) {
            s_off[e] = p.item_off[e];
            if (e < p.nb)
                s_cnt[e] = p.cnt[e];
        }
    __syncthreads();

    const int total = tab_in_smem ? s_off[p.nb] : __ldg(p.item_off + p.nb);
    const int nks = (p.K / 2) / KS; // K-slices per item
    // Scale-box x coordinate per K-slice, in scale elements (bytes / f32).
    constexpr int SX = (FMT == MVLLM_FMT_MXFP4) ? L::SB : L::SB / 4;

    if (warp == kDecodeConsumerWarps) {
        // ------------------------------ producer ------------------------------
        const uint64_t pol_w = policy_evict_first(); // weights: read once per step
        const uint64_t pol_x = policy_evict_last();  // operand rows: re-read per item
        uint32_t it = 0;
        bool ok = true;
        int i = blockIdx.x;
        DecodeItem nxt{};
        if (i < total)
            nxt = resolve_item<NT>(p, s_off, s_cnt, tab_in_smem, i);
        for (; i < total && ok; i += gridDim.x) {
            const DecodeItem cur = nxt;
            if (i + static_cast<int>(gridDim.x) < total) // loads in flight during this item
                nxt = resolve_item<NT>(p, s_off, s_cnt, tab_in_smem, i + gridDim.x);
            // Lanes 0..NBOX-1 load weight boxes (two half-height boxes in
            // phase 1: gate rows then up rows), lanes 8/9 the scale boxes.
            const uint8_t *tm_w0 = cur.tm + (PHASE == 1 ? kTmGateP : kTmDownP) * kTmBytes;
            const uint8_t *tm_w1 = cur.tm + kTmUpP * kTmBytes;
            const uint8_t *tm_s0 = cur.tm + (PHASE == 1 ? kTmGateS : kTmDownS) * kTmBytes;
            const uint8_t *tm_s1 = cur.tm + kTmUpS * kTmBytes;
            if (lane < L::NBOX) {
                tmap_acquire(tm_w0);
                if (PHASE == 1)
                    tmap_acquire(tm_w1);
            } else if (lane == 8) {
                tmap_acquire(tm_s0);
            } else if (lane == 9 && PHASE == 1) {
                tmap_acquire(tm_s1);
            }
            const int row0 = PHASE == 1 ? cur.rb * 32 : cur.rb * 64;
            for (int ks = 0; ks < nks; ++ks, ++it) {
                const int slot = it % NS;
                const uint32_t par = (it / NS) & 1u;
                if (!mbar_wait(&empty[slot], par ^ 1u, p.err)) {
                    ok = false;
                    break;
                }
                uint8_t *st = stages + slot * L::STAGE_BYTES;
                if (lane == 0) {
                    *reinterpret_cast<int4 *>(st + L::OFF_HDR) =
                        make_int4(cur.rb, cur.nv, cur.orow0, 0);
                    mbar_arrive_expect_tx(&full[slot], kDecodeRows * (KS + L::SB) +
                                                           cur.nv * 4 * KS);
                }
                __syncwarp();
                if (lane < L::NBOX) {
                    uint8_t *dst = st + L::OFF_W + lane * L::BOX_BYTES;
                    const int x = ks * KS + lane * 128;
                    if (PHASE == 1) {
                        tma_load_2d(dst, tm_w0, x, row0, &full[slot], pol_w);
                        tma_load_2d(dst + 32 * 128, tm_w1, x, row0, &full[slot], pol_w);
                    } else {
                        tma_load_2d(dst, tm_w0, x, row0, &full[slot], pol_w);
                    }
                } else if (lane == 8) {
                    tma_load_2d(st + L::OFF_SC, tm_s0, ks * SX, row0, &full[slot], pol_w);
                } else if (lane == 9 && PHASE == 1) {
                    tma_load_2d(st + L::OFF_SC + 32 * L::SB, tm_s1, ks * SX, row0, &full[slot],
                                pol_w);
                }
                if (lane >= 16 && lane - 16 < cur.nv) {
                    const int r = lane - 16;
                    bulk_g2s(st + L::OFF_X + r * L::XROW,
                             cur.x + static_cast<size_t>(r) * p.K +
                                 static_cast<size_t>(ks) * 2 * KS,
                             4 * KS, &full[slot], pol_x);
                }
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
    // Consumer warps touch no global memory until the epilogue stores.
    const int mb = warp & 3, kp = warp >> 2; // row block, K quarter
    const int g = lane >> 2, t = lane & 3;
    const int R0 = mb * 16 + g, R1 = R0 + 8;
    const int tid = threadIdx.x; // 0..kDecodeConsumers-1
    constexpr int KQ = KS / 2;   // columns of one K quarter of a stage
    uint32_t it = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < total; i += gridDim.x) {
        int rb = 0, nv = 0, orow0 = 0, nt_active = 0;
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        for (int ks = 0; ks < nks; ++ks, ++it) {
            const int slot = it % NS;
            const uint32_t par = (it / NS) & 1u;
            if (ok && !mbar_wait(&full[slot], par, p.err))
                ok = false;
            if (ok) {
                uint8_t *st = stages + slot * L::STAGE_BYTES;
                if (ks == 0) {
                    const int4 h = *reinterpret_cast<const int4 *>(st + L::OFF_HDR);
                    rb = h.x, nv = h.y, orow0 = h.z;
                    nt_active = (nv + 7) >> 3;
                }
                StageScales<FMT, KS> sc;
                const uint32_t sbase = smem_u32(st + L::OFF_SC) + kp * (L::SB / 4);
                lds_scales<FMT, KS>(sc, sbase + R0 * L::SB, sbase + R1 * L::SB);
                const uint32_t xaddr =
                    smem_u32(st + L::OFF_X) + g * L::XROW + (kp * KQ + t * 8) * 2;
                decode_stage_compute<FMT, KS, NT>(smem_u32(st + L::OFF_W), R0,
                                                  kp * (KS / 4) + t * 4, xaddr, sc, acc,
                                                  nt_active);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }

        // Epilogue: reduce the four K quarters through shared memory.
        named_sync(1, kDecodeConsumers);
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
        named_sync(1, kDecodeConsumers);
        if (ok) {
            if (PHASE == 1) {
                __half *h = static_cast<__half *>(p.out);
                for (int idx = tid; idx < 32 * nv; idx += kDecodeConsumers) {
                    const int f = idx & 31, n = idx >> 5;
                    float gt = 0.f, up = 0.f;
#pragma unroll
                    for (int q = 0; q < kDecodeKParts; ++q) {
                        gt += red[(q * kDecodeRows + f) * L::RS + n];
                        up += red[(q * kDecodeRows + 32 + f) * L::RS + n];
                    }
                    const float hv = apply_act(gt, up, p.act, p.act_a, p.act_b);
                    h[static_cast<size_t>(orow0 + n) * p.O + stage_pos(rb * 32 + f, FMT)] =
                        __float2half_rn(hv);
                }
            } else {
                float *y = static_cast<float *>(p.out);
                for (int idx = tid; idx < kDecodeRows * nv; idx += kDecodeConsumers) {
                    const int r = idx & 63, n = idx >> 6;
                    float v = 0.f;
#pragma unroll
                    for (int q = 0; q < kDecodeKParts; ++q)
                        v += red[(q * kDecodeRows + r) * L::RS + n];
                    y[static_cast<size_t>(orow0 + n) * p.O + rb * 64 + r] = v;
                }
            }
        }
    }
}

} // namespace mvb
