// decode_ffn.cuh -- weight-streaming expert FFN for the small-M (decode) regime.
//
// Replaces the three quant::matmul_* calls of cpu_moe_block
// (src/gpu/metal_ops.cpp:308-327) for fmt 4 (int4-g64) and fmt 7 (MXFP4).
// Two persistent launches per moe_block:
//   phase 1: item = (expert, 32 gate rows + the matching 32 up rows, chunk of
//            <= 8*NT tokens) -> h = act(gate, up), f16, written straight into
//            the operand layout phase 2 reads;
//   phase 2: item = (expert, 64 down rows, chunk) -> y, f16 (a value beyond
//            the f16 range records MVLLM_ERR_ACT_RANGE).
//
// CTA = 16 consumer warps (4 row blocks x 4 K quarters of a stage, 4 warps per
// scheduler) + 2 producer warps + 2 epilogue warps.  Each stage of the
// shared-memory ring holds one K-slice of an item: its 64 weight rows, the
// slice's scale bytes, an item header and the matching slice of the item's
// token rows.  The producer warps resolve items one ahead, acquire the next
// item's tensor maps while the current one streams, and fill stages -- one
// warp the weight rows, the other the header, scales and token rows -- with:
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
// At the end of an item the consumers drop their partial sums into one of two
// reduction buffers and go straight on to the next item; the epilogue warps
// reduce the four K quarters, apply the activation (phase 1) and store.  So
// the ring keeps streaming across item boundaries.
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
constexpr int kDecodeEpilogueWarps = 2;
constexpr int kDecodeEpilogue = kDecodeEpilogueWarps * 32;
constexpr int kDecodeProducerWarp = kDecodeConsumerWarps; // weight rows
constexpr int kDecodeSideWarp = kDecodeProducerWarp + 1;   // header, scales, token rows
constexpr int kDecodeThreads = kDecodeConsumers + 64 + kDecodeEpilogue;
// Reduction buffers between the consumers and the epilogue warps: consumers
// start the next item while the epilogue drains earlier ones.
constexpr int kDecodeRedBufs = 2;
static_assert(16 + 2 * kDecodeRedBufs <= 32, "barrier block holds 32 barriers");

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
    const int *tmaps_dirty; // non-zero: maps were rewritten, acquire before use
    int wbox3d;             // weight maps are 3-D: one box per matrix per stage
    int *err;
    const int *enable;      // redo launch: runs only when *enable is non-zero (null: always)
};

template <int FMT, int KS, int NT> struct DecodeLayout {
    static constexpr int MT = 8 * NT;
    static constexpr int SB = (FMT == MVLLM_FMT_MXFP4) ? KS / 16 : KS / 8; // scale bytes/row
    static constexpr int NBOX = KS / 128;    // 128-byte swizzled column boxes per stage
    static constexpr int BOX_BYTES = kDecodeRows * 128;
    static constexpr int XROW = 4 * KS + 64; // 2*KS f16 per row, +64 B for LDS.128
    static constexpr int RS = MT + 1;        // reduction row stride (floats)
    static constexpr int RED_BYTES = kDecodeKParts * kDecodeRows * RS * 4; // per buffer
    static constexpr int BAR_BYTES = 256; // 8 full + 8 empty + 2 x kDecodeRedBufs reduction
    static constexpr int RHDR_BYTES = 16 * kDecodeRedBufs; // item headers for the epilogue
    static constexpr int ITEM_TAB = 512;  // item offsets of up to 511 experts, in shared memory
    static constexpr int OFF_W = 0;          // 1024-aligned: the 128-byte swizzle needs it
    static constexpr int OFF_SC = OFF_W + NBOX * BOX_BYTES;
    static constexpr int OFF_HDR = OFF_SC + kDecodeRows * SB;
    static constexpr int OFF_X = OFF_HDR + 16;
    static constexpr int STAGE_BYTES = (OFF_X + MT * XROW + 1023) / 1024 * 1024;
    static constexpr int HEAD_BYTES =
        (BAR_BYTES + RHDR_BYTES + kDecodeRedBufs * RED_BYTES + ITEM_TAB * 4 + 1023) / 1024 * 1024;
    static constexpr int OFF_ITEMS = BAR_BYTES + RHDR_BYTES + kDecodeRedBufs * RED_BYTES;
    static int smem_bytes(int nstages) { return HEAD_BYTES + nstages * STAGE_BYTES + 1024; }
};

template <int FMT, int KS> struct StageScales {
    // A warp covers KS/2 columns of a stage: MXFP4 KS/64 ue8m0 bytes per row,
    // int4 KS/128 f32 per row.
    static constexpr int WORDS = (FMT == MVLLM_FMT_MXFP4) ? (KS / 256) : (KS / 128);
    uint32_t r0[WORDS], r1[WORDS];
};

template <int FMT, int KS>
__device__ __forceinline__ void lds_scales(StageScales<FMT, KS> &sc, const uint8_t *a0,
                                           const uint8_t *a1) {
    constexpr int W = StageScales<FMT, KS>::WORDS;
    if constexpr (W == 1) {
        sc.r0[0] = *reinterpret_cast<const uint32_t *>(a0);
        sc.r1[0] = *reinterpret_cast<const uint32_t *>(a1);
    } else if constexpr (W == 2) {
        const uint2 x = *reinterpret_cast<const uint2 *>(a0);
        const uint2 y = *reinterpret_cast<const uint2 *>(a1);
        sc.r0[0] = x.x, sc.r0[1] = x.y, sc.r1[0] = y.x, sc.r1[1] = y.y;
    } else {
        const uint4 x = *reinterpret_cast<const uint4 *>(a0);
        const uint4 y = *reinterpret_cast<const uint4 *>(a1);
        sc.r0[0] = x.x, sc.r0[1] = x.y, sc.r0[2] = x.z, sc.r0[3] = x.w;
        sc.r1[0] = y.x, sc.r1[1] = y.y, sc.r1[2] = y.z, sc.r1[3] = y.w;
    }
}

// The MXFP4 single-tile stage split in two: every shared-memory operand of
// the warp's quarter (weights, token fragments) goes to registers first, so
// the warp can release the stage before it computes; the producer then
// refills the slot while the math runs.
template <int KS> struct Mx4StageRegs {
    static constexpr int NG = KS / 64;
    uint32_t w0[NG], w1[NG];
    uint4 xb[NG];
};

template <int KS>
__device__ __forceinline__ void mx4_stage_load(const uint8_t *wl, const uint32_t (&swz)[KS / 64],
                                               const uint8_t *xl, Mx4StageRegs<KS> &r) {
    constexpr int kRow8 = 8 * 128;
#pragma unroll
    for (int j = 0; j < Mx4StageRegs<KS>::NG; ++j) {
        const uint8_t *a = wl + swz[j];
        r.w0[j] = *reinterpret_cast<const uint32_t *>(a);
        r.w1[j] = *reinterpret_cast<const uint32_t *>(a + kRow8);
        r.xb[j] = *reinterpret_cast<const uint4 *>(xl + j * 64);
    }
}

template <int KS>
__device__ __forceinline__ void mx4_stage_math(const Mx4StageRegs<KS> &r,
                                               const StageScales<MVLLM_FMT_MXFP4, KS> &sc,
                                               float (&acc)[1][4]) {
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < Mx4StageRegs<KS>::NG; ++j) {
        uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
        e2m1x8_to_f16x8(r.w0[j], p0, p1, p2, p3);
        e2m1x8_to_f16x8(r.w1[j], q0, q1, q2, q3);
        const float s0 = ue8m0_byte(sc.r0[j >> 2], j & 3);
        const float s1 = ue8m0_byte(sc.r1[j >> 2], j & 3);
        float tmp[4];
        mma_f16_16816(tmp, p0, q0, p1, q1, r.xb[j].x, r.xb[j].y, zero);
        mma_f16_16816(tmp, p2, q2, p3, q3, r.xb[j].z, r.xb[j].w, tmp);
        ffma2(acc[0][0], acc[0][1], tmp[0], tmp[1], s0);
        ffma2(acc[0][2], acc[0][3], tmp[2], tmp[3], s1);
    }
}

// One stage of one consumer warp.  wl: this lane's first weight row (R0) in
// its quarter's swizzled box, plus 4*t; row R0 + 8 is 1024 bytes further and
// shares the swizzle phase.  swz[c]: byte offset of this warp's c-th 16-byte
// chunk in the lane's row (chunk XOR row%8, precomputed per lane).  xl: the
// lane's token row and column offset in the stage's operand rows.  All loads
// are plain shared-memory reads the compiler may schedule freely; every token
// tile is computed (columns beyond the item's tokens are never stored).
template <int FMT, int KS, int NT>
__device__ __forceinline__ void decode_stage_compute(const uint8_t *wl,
                                                     const uint32_t (&swz)[KS / 64],
                                                     const uint8_t *xl,
                                                     const StageScales<FMT, KS> &sc,
                                                     float (&acc)[NT][4]) {
    using L = DecodeLayout<FMT, KS, NT>;
    constexpr int kRow8 = 8 * 128;
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (FMT == MVLLM_FMT_MXFP4) {
        constexpr int NG = KS / 64; // 16-byte groups in this warp's quarter of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint8_t *a = wl + swz[j];
            const uint32_t w0 = *reinterpret_cast<const uint32_t *>(a);
            const uint32_t w1 = *reinterpret_cast<const uint32_t *>(a + kRow8);
            uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
            e2m1x8_to_f16x8(w0, p0, p1, p2, p3);
            e2m1x8_to_f16x8(w1, q0, q1, q2, q3);
            const float s0 = ue8m0_byte(sc.r0[j >> 2], j & 3);
            const float s1 = ue8m0_byte(sc.r1[j >> 2], j & 3);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint4 xb = *reinterpret_cast<const uint4 *>(xl + nt * 8 * L::XROW + j * 64);
                float tmp[4];
                mma_f16_16816(tmp, p0, q0, p1, q1, xb.x, xb.y, zero);
                mma_f16_16816(tmp, p2, q2, p3, q3, xb.z, xb.w, tmp);
                ffma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], s0);
                ffma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], s1);
            }
        }
    } else {
        constexpr int NG = KS / 128; // 32-byte groups in this warp's quarter of the stage
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const uint8_t *aa = wl + swz[2 * j], *ab = wl + swz[2 * j + 1];
            const uint32_t w0a = *reinterpret_cast<const uint32_t *>(aa);
            const uint32_t w0b = *reinterpret_cast<const uint32_t *>(ab);
            const uint32_t w1a = *reinterpret_cast<const uint32_t *>(aa + kRow8);
            const uint32_t w1b = *reinterpret_cast<const uint32_t *>(ab + kRow8);
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
                const uint8_t *xa = xl + nt * 8 * L::XROW + j * 128;
                const uint4 xlo = *reinterpret_cast<const uint4 *>(xa);
                const uint4 xhi = *reinterpret_cast<const uint4 *>(xa + 64);
                float tmp[4];
                mma_f16_16816(tmp, p0, q0, p1, q1, xlo.x, xlo.y, zero);
                mma_f16_16816(tmp, p2, q2, p3, q3, xlo.z, xlo.w, tmp);
                mma_f16_16816(tmp, u0, v0, u1, v1, xhi.x, xhi.y, tmp);
                mma_f16_16816(tmp, u2, v2, u3, v3, xhi.z, xhi.w, tmp);
                ffma2(acc[nt][0], acc[nt][1], tmp[0], tmp[1], s0);
                ffma2(acc[nt][2], acc[nt][3], tmp[2], tmp[3], s1);
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

// Items are resolved one ahead by the producer in two halves: at the start of
// item i it finds the next item's expert (binary search over the item offsets,
// kept in shared memory when they fit) and issues that expert's three loads;
// their values are first used at the start of the next item, so the producer
// never waits on them.
struct PendingItem {
    int i, e, off, cnt, xrow, orow;
};

__device__ __forceinline__ int find_owner_smem(const int *off, int nb, int i) {
    int lo = 0, hi = nb;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off[mid] <= i)
            lo = mid;
        else
            hi = mid;
    }
    return lo;
}

__device__ __forceinline__ PendingItem issue_item(const DecodeArgs &p, const int *off_s, int i) {
    PendingItem q;
    q.i = i;
    q.e = off_s ? find_owner_smem(off_s, p.nb, i) : find_owner(p.item_off, p.nb, i);
    q.off = off_s ? off_s[q.e] : __ldg(p.item_off + q.e);
    q.cnt = __ldg(p.cnt + q.e);
    q.xrow = __ldg(p.xrow + q.e);
    q.orow = __ldg(p.orow + q.e);
    return q;
}

template <int NT> __device__ __forceinline__ DecodeItem finish_item(const DecodeArgs &p,
                                                                    const PendingItem &q) {
    constexpr int MT = 8 * NT;
    const int local = q.i - q.off;
    const int chunks = (q.cnt + MT - 1) / MT;
    const int rb = local / chunks, chunk = local - rb * chunks;
    const int n0 = chunk * MT;
    DecodeItem it;
    it.rb = rb;
    it.nv = min(MT, q.cnt - n0);
    it.tm = p.tmaps + static_cast<size_t>(q.e) * kTmCount * kTmBytes;
    it.x = p.x + static_cast<size_t>(q.xrow + n0) * p.K;
    it.orow0 = q.orow + n0;
    return it;
}

template <int FMT, int PHASE, int KS, int NT>
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_ffn_kernel(const DecodeArgs p) {
    // Phase 1 lets phase 2 start as soon as its own inputs are complete:
    // phase 2's item table, tensor maps and weights come from the kernels
    // before phase 1, so its weight warp streams the first stages while
    // phase 1 finishes; only phase 2's token rows (h, phase 1's output) wait
    // for phase 1 (the side warp's griddepcontrol.wait below).  Every global
    // write of phase 2 follows a stage that holds h.
    if (p.enable) { // a redo launch: the word comes from the kernel before it
        pdl_wait();
        if (load_volatile(p.enable) == 0)
            return;
    }
    if constexpr (PHASE == 1) {
        pdl_wait();
        pdl_trigger();
    }
    static_assert(KS == 256 || KS == 512, "stage K-slice");
    using L = DecodeLayout<FMT, KS, NT>;
    extern __shared__ uint8_t smem_raw[];
    // Align by pointer arithmetic on the __shared__ array (not an integer round
    // trip), so every derived pointer stays a shared-memory pointer (LDS, 32-bit
    // addresses) for the compiler.
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 8;
    uint64_t *rfull = full + 16; // reduction buffer filled (16 consumer warps)
    uint64_t *rempty = rfull + kDecodeRedBufs; // reduction buffer drained (64 epilogue threads)
    int4 *rhdr = reinterpret_cast<int4 *>(smem + L::BAR_BYTES);
    float *red = reinterpret_cast<float *>(smem + L::BAR_BYTES + L::RHDR_BYTES);
    uint8_t *stages = smem + L::HEAD_BYTES;
    int *items_s = reinterpret_cast<int *>(smem + L::OFF_ITEMS);
    const bool items_in_smem = p.nb + 1 <= L::ITEM_TAB;
    if (items_in_smem)
        for (int e = threadIdx.x; e <= p.nb; e += blockDim.x)
            items_s[e] = __ldg(p.item_off + e);

    const int NS = p.nstages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 2); // both producer warps' expect_tx arrivals; the rest is tx bytes
            mbar_init(&empty[s], kDecodeConsumerWarps);
        }
        for (int b = 0; b < kDecodeRedBufs; ++b) {
            mbar_init(&rfull[b], kDecodeConsumerWarps);
            mbar_init(&rempty[b], kDecodeEpilogue);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int total = __ldg(p.item_off + p.nb);
    const int nks = (p.K / 2) / KS; // K-slices per item
    // Scale-box x coordinate per K-slice, in scale elements (bytes / f32).
    constexpr int SX = (FMT == MVLLM_FMT_MXFP4) ? L::SB : L::SB / 4;

    if (warp == kDecodeProducerWarp || warp == kDecodeSideWarp) {
        // ----------------------------- producers ------------------------------
        // Both warps walk the same items and stages.  The weight warp issues
        // nothing but the weight boxes, back to back; the side warp issues
        // the header, the scale boxes and the token rows.  (With one warp
        // doing all of it the weight copies waited behind the small ones:
        // the split measured 10-15% faster on config[1].)
        const bool wprod = warp == kDecodeProducerWarp;
        if (PHASE == 2 && !wprod)
            pdl_wait(); // phase 1's output rows
        const uint64_t pol_w = policy_evict_first(); // weights: read once per step
        const uint64_t pol_x = policy_evict_last();  // operand rows: re-read per item
        uint32_t it = 0;
        bool ok = true;
        int i = blockIdx.x;
        const int G = gridDim.x;
        const bool fence_maps = __ldg(p.tmaps_dirty) != 0;
        const int *off_s = items_in_smem ? items_s : nullptr;
        DecodeItem nxt{};
        PendingItem pend{};
        if (i < total) {
            nxt = finish_item<NT>(p, issue_item(p, off_s, i));
            if (fence_maps)
                tmap_acquire(nxt.tm + (lane % kTmCount) * kTmBytes);
        }
        for (; i < total && ok; i += G) {
            const DecodeItem cur = nxt;
            const bool more = i + G < total;
            if (more) // the next item's loads fly while this item streams
                pend = issue_item(p, off_s, i + G);
            const uint8_t *tm_w0 = cur.tm + (PHASE == 1 ? kTmGateP : kTmDownP) * kTmBytes;
            const uint8_t *tm_w1 = cur.tm + kTmUpP * kTmBytes;
            const uint8_t *tm_s0 = cur.tm + (PHASE == 1 ? kTmGateS : kTmDownS) * kTmBytes;
            const uint8_t *tm_s1 = cur.tm + kTmUpS * kTmBytes;
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
                    if (!wprod)
                        *reinterpret_cast<int4 *>(st + L::OFF_HDR) =
                            make_int4(cur.rb, cur.nv, cur.orow0, 0);
                    mbar_arrive_expect_tx(&full[slot], wprod ? kDecodeRows * KS
                                                             : kDecodeRows * L::SB +
                                                                   cur.nv * 4 * KS);
                }
                __syncwarp();
                if (!wprod) {
                    // side warp: below
                } else if (p.wbox3d) {
                    // One box per matrix: [column chunk][rows][128 B] -- phase 1
                    // puts the gate rows' chunks first, then the up rows'.
                    if (lane == 0)
                        tma_load_3d(st + L::OFF_W, tm_w0, 0, row0, ks * L::NBOX, &full[slot],
                                    pol_w);
                    else if (lane == 1 && PHASE == 1)
                        tma_load_3d(st + L::OFF_W + L::NBOX * 32 * 128, tm_w1, 0, row0,
                                    ks * L::NBOX, &full[slot], pol_w);
                } else if (lane < L::NBOX) {
                    uint8_t *dst = st + L::OFF_W + lane * L::BOX_BYTES;
                    const int x = ks * KS + lane * 128;
                    if (PHASE == 1) {
                        tma_load_2d(dst, tm_w0, x, row0, &full[slot], pol_w);
                        tma_load_2d(dst + 32 * 128, tm_w1, x, row0, &full[slot], pol_w);
                    } else {
                        tma_load_2d(dst, tm_w0, x, row0, &full[slot], pol_w);
                    }
                }
                if (wprod) {
                    // weight warp: above
                } else if (lane == 8) {
                    tma_load_2d(st + L::OFF_SC, tm_s0, ks * SX, row0, &full[slot], pol_w);
                } else if (lane == 9 && PHASE == 1) {
                    tma_load_2d(st + L::OFF_SC + 32 * L::SB, tm_s1, ks * SX, row0, &full[slot],
                                pol_w);
                }
                if (!wprod && lane >= 16 && lane - 16 < cur.nv) {
                    const int r = lane - 16;
                    bulk_g2s(st + L::OFF_X + r * L::XROW,
                             cur.x + static_cast<size_t>(r) * p.K +
                                 static_cast<size_t>(ks) * 2 * KS,
                             4 * KS, &full[slot], pol_x);
                }
                __syncwarp();
                // With the item's last stage on its way: finish the next item
                // (its loads landed while this item streamed) and acquire its
                // tensor maps (one convergent fence per lane).
                if (ks == nks - 1 && more) {
                    nxt = finish_item<NT>(p, pend);
                    if (fence_maps)
                        tmap_acquire(nxt.tm + (lane % kTmCount) * kTmBytes);
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

    if (warp > kDecodeSideWarp) {
        // ------------------------------ epilogue ------------------------------
        const int et = threadIdx.x - (kDecodeConsumers + 64); // 0..63
        uint32_t n_items = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < total; i += gridDim.x, ++n_items) {
            const int rs = n_items % kDecodeRedBufs;
            if (ok && !mbar_wait(&rfull[rs], (n_items / kDecodeRedBufs) & 1u, p.err))
                ok = false;
            if (ok) {
                const int4 h = rhdr[rs];
                const int rb = h.x, nv = h.y, orow0 = h.z;
                const float *rd = red + rs * (L::RED_BYTES / 4);
                if (PHASE == 1) {
                    __half *hp = static_cast<__half *>(p.out);
                    for (int idx = et; idx < 32 * nv; idx += kDecodeEpilogue) {
                        const int f = idx & 31, n = idx >> 5;
                        float gt = 0.f, up = 0.f;
#pragma unroll
                        for (int q = 0; q < kDecodeKParts; ++q) {
                            gt += rd[(q * kDecodeRows + f) * L::RS + n];
                            up += rd[(q * kDecodeRows + 32 + f) * L::RS + n];
                        }
                        const float hv = apply_act(gt, up, p.act, p.act_a, p.act_b);
                        if (beyond_f16(hv))
                            set_error(p.err, MVLLM_ERR_ACT_RANGE);
                        hp[static_cast<size_t>(orow0 + n) * p.O + stage_pos(rb * 32 + f, FMT)] =
                            __float2half_rn(hv);
                    }
                } else {
                    __half *y = static_cast<__half *>(p.out); // f16 rows of y
                    for (int idx = et; idx < kDecodeRows * nv; idx += kDecodeEpilogue) {
                        const int r = idx & 63, n = idx >> 6;
                        float v = 0.f;
#pragma unroll
                        for (int q = 0; q < kDecodeKParts; ++q)
                            v += rd[(q * kDecodeRows + r) * L::RS + n];
                        if (beyond_f16(v))
                            set_error(p.err, MVLLM_ERR_ACT_RANGE);
                        y[static_cast<size_t>(orow0 + n) * p.O + rb * 64 + r] =
                            __float2half_rn(v);
                    }
                }
            }
            mbar_arrive(&rempty[rs]); // every epilogue thread, also on the error path
        }
        return;
    }

    // ------------------------------- consumers --------------------------------
    // Consumer warps touch no global memory at all.
    const int mb = warp & 3, kp = warp >> 2; // row block, K quarter
    const int g = lane >> 2, t = lane & 3;
    const int R0 = mb * 16 + g, R1 = R0 + 8;
    constexpr int KQ = KS / 2; // columns of one K quarter of a stage
    // Lane-constant pieces of the swizzled weight addresses (R0 % 8 == g).
    const int qbyte = kp * (KS / 4);
    uint32_t swz[KS / 64];
#pragma unroll
    for (int c = 0; c < KS / 64; ++c)
        swz[c] = static_cast<uint32_t>(((((qbyte & 127) >> 4) + c) & 7) ^ g) << 4;
    // Weight rows of the stage: 2-D boxes give [chunk][64 rows][128 B]; the
    // 3-D phase-1 boxes give [chunk][32 gate rows][128 B] then the same for
    // the up rows.  Both keep 128-byte rows, so the swizzle phase is row % 8.
    const int wl_off =
        (PHASE == 1 && p.wbox3d)
            ? L::OFF_W + (R0 >= 32 ? L::NBOX * 32 * 128 : 0) + (qbyte >> 7) * 32 * 128 +
                  (R0 & 31) * 128 + 4 * t
            : L::OFF_W + (qbyte >> 7) * L::BOX_BYTES + R0 * 128 + 4 * t;
    const int xl_off = L::OFF_X + g * L::XROW + (kp * KQ + t * 8) * 2;
    const int s0_off = L::OFF_SC + R0 * L::SB + kp * (L::SB / 4);
    uint32_t it = 0, n_items = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < total; i += gridDim.x, ++n_items) {
        int4 hdr = make_int4(0, 0, 0, 0);
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
                if (ks == 0)
                    hdr = *reinterpret_cast<const int4 *>(st + L::OFF_HDR);
                StageScales<FMT, KS> sc;
                lds_scales<FMT, KS>(sc, st + s0_off, st + s0_off + 8 * L::SB);
                if constexpr (FMT == MVLLM_FMT_MXFP4 && NT == 1) {
                    Mx4StageRegs<KS> r;
                    mx4_stage_load<KS>(st + wl_off, swz, st + xl_off, r);
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive(&empty[slot]); // operands are in registers
                    mx4_stage_math<KS>(r, sc, acc);
                    continue;
                } else {
                    decode_stage_compute<FMT, KS, NT>(st + wl_off, swz, st + xl_off, sc, acc);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[slot]);
        }
        // Hand the partial sums to the epilogue warps and move on.
        const int rs = n_items % kDecodeRedBufs;
        if (ok && !mbar_wait(&rempty[rs], ((n_items / kDecodeRedBufs) & 1u) ^ 1u, p.err))
            ok = false;
        if (ok) {
            float *rd = red + rs * (L::RED_BYTES / 4);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float *r0 = rd + (kp * kDecodeRows + R0) * L::RS + nt * 8 + 2 * t;
                float *r1 = rd + (kp * kDecodeRows + R1) * L::RS + nt * 8 + 2 * t;
                r0[0] = acc[nt][0];
                r0[1] = acc[nt][1];
                r1[0] = acc[nt][2];
                r1[1] = acc[nt][3];
            }
            if (warp == 0 && lane == 0)
                rhdr[rs] = hdr;
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&rfull[rs]); // also on the error path: the epilogue never hangs
    }
}

} // namespace mvb
