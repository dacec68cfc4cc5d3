// tc_mx.cuh -- block-scaled tensor-core expert FFN (tcgen05 kind::mxf4 /
// kind::mxf8f6f4 with ue8m0 block scales in tensor memory) for MXFP4 experts
// with many rows (prefill chunks, skewed routing).
//
// Same contract, items and epilogue as tc_ffn.cuh: phase 1 computes
//   h[r, j] = act(sum_k x[r,k] g[j,k], sum_k x[r,k] u[j,k])   (f16)
// and phase 2 computes
//   y[r, n] = sum_j h[r,j] d[n,j]           (f32 sums, stored as f16)
// for the rows r the plan gave to the tensor-core path (reference:
// moe_block's per-expert loop, metal_ops.cpp:278-342, through matmul_mxfp4,
// quant.cpp:298-321).
//
// What differs from tc_ffn: the weights are never dequantised.  The packed
// e2m1 rows go from HBM into shared memory by TMA and straight into the MMA,
// which applies each row's ue8m0 scale per 32 elements itself -- exactly the
// reference's MXFP4 scale granularity, so the weight operand is exact.  The
// other operand must then be block-scaled too.  Token rows x (and h for
// phase 2) are written as a sum of NTERM block-scaled terms,
//   x ~ s_1 q_1 + s_2 q_2 + ... ,  q_t e2m1 (mxf4) or e4m3 (mxf8f6f4),
//   s_t = 2^(c_t - 127), one ue8m0 code c_t per 32 elements of a row,
// each term quantising what the earlier ones left over (mx_terms_kernel).
// The terms accumulate into one f32 accumulator.  Measured on B200 over the
// config[3] layer (relative L2 / max-abs against f64): mxf4 x1 2.2e-1 / 1.5,
// x2 2.8e-2 / 1.9e-1, x3 2.7e-3 / 1.9e-2; e4m3 x1 4.7e-2 / 3.5e-1, x2 7e-4 /
// 5.7e-3.  Three mxf4 terms cost 3/4 of the f16 tensor time and need no
// dequantisation; two e4m3 terms cost the f16 tensor time.
//
// Layout (per CTA; a CTA pair splits M = 256 weight rows 128/128 and the
// token tile N/2 / N/2 as tc_ffn does):
// - A (weights): 128 rows x 128 bytes per stage, K-major, 128-byte swizzle.
//   mxf4: 256 packed e2m1 per row (TMA of the packed bytes as they are);
//   mxf8f6f4: 128 e2m1 per row in the padded 16 x 4-bit + 8-byte-gap form
//   the MMA needs, expanded by the TMA (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B).
//   Phase 1 takes 16 gate rows then 16 up rows per TMEM lane quadrant (eight
//   16-row boxes), so the accumulator lanes match tc_ffn's epilogue.
// - B (token terms): NTERM planes of TOK_ROWS rows x 128 bytes per stage.
// - Scales: 16-byte windows per row (16 ue8m0 codes = 512 elements) by TMA;
//   four SF warps (one per TMEM lane quadrant) move them into tensor memory
//   with tcgen05.st in the layout the MMA reads: for an M = 128 operand, row
//   m's four codes of a 128-element group at lane m, column base + m / 32;
//   for the token operand, token n's codes at column base + n / 32 of every
//   quadrant.
//
// Warp roles (pair 480 threads, one CTA per SM; solo 352, two per SM):
//   warps 0..E-1   epilogue (tc_epilogue, shared with tc_ffn)
//   4 warps        SF warps: scale windows -> tensor memory
//   1 warp         token producer: TMA of the term planes and their scales
//   1 warp         MMA issuer (one thread of the pair's even CTA), TMEM owner
//   1 warp         weight producer: TMA of packed weight rows and scales
#pragma once

#include "tc_ffn.cuh"

namespace mvb {

enum { kMxF4 = 0, kMxF8 = 1 }; // MMA kind: mxf4 (block32) or mxf8f6f4 (e2m1 x e4m3)

// Two forms, as tc_ffn: CTA pairs (M = 256 weight rows per MMA, token tiles
// of up to 256 rows: an N = 256 pair MMA runs at the tensor rate; the token
// terms accumulate through separate MMAs) and single CTAs for the rest tiles
// of at most 64 rows.  A narrow MMA costs almost as much tensor-pipe time as
// a 128-wide one (about 46 cycles at N <= 64 on B200), so the single-CTA form
// stacks a tile's terms along N instead: term t's 64 token rows are rows
// 64t..64t+63 of one B operand, one MMA per K step covers all terms, and the
// epilogue adds the terms' accumulator columns.  The three operand rings
// (weights, token terms, block scales in TMEM) advance one K stage at a
// time; one "stage consumed" commit per stage frees a stage's slot in all
// three (a tcgen05.commit costs about as much as an MMA to issue).
template <int KIND, int NTERM, bool PAIR> struct MxCfg {
    static constexpr int EPI_WARPS = TcCfg<PAIR>::EPI_WARPS;
    static constexpr int SF_WARP0 = EPI_WARPS;
    static constexpr int TOK_WARP = SF_WARP0 + 4;
    static constexpr int MMA_WARP = TOK_WARP + 1;
    static constexpr int W_WARP = TOK_WARP + 2;
    static constexpr int THREADS = (W_WARP + 1) * 32;     // pair 480, single 352
    static constexpr int TSHIFT = 8;                      // pair tiles of 256 rows
    static constexpr int NT = TcCfg<PAIR>::NT;            // 256 / 64
    // Stacking pays where it cuts three or more MMAs to one (measured); the
    // stacked accumulators need a whole SM's TMEM, the unstacked single-CTA
    // form runs two CTAs per SM (two issuing threads).
    static constexpr bool STACK = !PAIR && NTERM >= 3;
    static constexpr int CTAS_PER_SM = (PAIR || STACK) ? 1 : 2;
    // Columns of one accumulator buffer (a pair tile wider than 128 takes both).
    static constexpr int ACC_COLS = STACK ? NTERM * NT : TcCfg<PAIR>::ACC_HALF;
    static constexpr int ACC_HALF = TcCfg<PAIR>::ACC_HALF;
    static constexpr int KSTAGE = KIND == kMxF4 ? 256 : 128; // K elements per stage
    static constexpr int G = KSTAGE / 128;                  // 4-code scale groups per stage
    static constexpr int WST = 512 / KSTAGE;                // stages per 16-byte scale window
    static constexpr int TOK_ROWS = PAIR ? NT / 2 : NT;     // token rows one CTA holds
    static constexpr int PLANE = TOK_ROWS * 128;            // one term's rows, one stage
    static constexpr int B_SLOT = NTERM * PLANE;
    static constexpr int A_SLOT = 128 * 128;
    static constexpr int SB = PAIR ? (B_SLOT <= 16384 ? 4 : 3)
                                   : STACK ? 4 : (B_SLOT <= 8192 ? 3 : 2);
    static constexpr int NSC = 2;                           // scale-window ring depth
    static constexpr int SCA_SLOT = 128 * 16;               // weight rows' windows
    static constexpr int SCB_SLOT = NTERM * NT * 16;        // every token of the tile (full N)
    // Token-code columns per (term, group): pairs N / 32 (a whole block of
    // 8); single CTAs 2 (64 rows), the terms of a group adjacent.
    static constexpr int NBMAX = PAIR ? NT / 32 : STACK ? 2 : 4;
    static constexpr int SF_COLS = 4 * G + NTERM * G * NBMAX;
    static constexpr int SSF = 3;                           // scale stages in tensor memory
    static constexpr int TMEM_COLS = CTAS_PER_SM == 1 ? 512 : 256;
    static constexpr int SF_BASE = PAIR ? 2 * ACC_HALF : 2 * ACC_COLS;
    static_assert(SF_BASE + SSF * SF_COLS <= TMEM_COLS, "TMEM budget");
    static constexpr int SMEM_BUDGET = 232448 / CTAS_PER_SM;
    static constexpr int ITEM_TAB = 512;
    static constexpr int FIXED = SB * B_SLOT + NSC * (SCA_SLOT + SCB_SLOT) + 2 * ITEM_TAB * 4 +
                                 1024 + 512;
    static constexpr int SA_FIT = (SMEM_BUDGET - FIXED) / A_SLOT;
    static constexpr int SA = SA_FIT > 8 ? 8 : SA_FIT;      // weight ring depth
    static_assert(SA >= 3, "weight ring");
    static constexpr int OFF_A = SB * B_SLOT;
    static constexpr int OFF_SCA = OFF_A + SA * A_SLOT;
    static constexpr int OFF_SCB = OFF_SCA + NSC * SCA_SLOT;
    static constexpr int OFF_BAR = OFF_SCB + NSC * SCB_SLOT;
    static constexpr int SD = SA > SB ? (SA > SSF ? SA : SSF) : (SB > SSF ? SB : SSF);
    static constexpr int NBARS = SA + SB + SSF + SD + 4 * NSC + 4 + 1;
    static_assert(NBARS * 8 + 16 <= 512, "barrier area");
    static constexpr int OFF_ITEMS = OFF_BAR + 512;
    static constexpr int SMEM = OFF_ITEMS + 2 * ITEM_TAB * 4 + 1024;
    static_assert(SMEM <= SMEM_BUDGET, "dynamic shared memory per SM");
    // Arrivals on the leader's scale-stage barrier: SF warps of both CTAs.
    static constexpr int SF_ARRIVALS = PAIR ? 8 : 4;
};

enum { kMxGateP = 0, kMxUpP, kMxDownP, kMxGateS, kMxUpS, kMxDownS, kMxMapCount };

struct MxArgs {
    TcArgs t;              // items, rows, output, activation, error word (as tc_ffn)
    const uint8_t *tmaps;  // [nb][kMxMapCount] weight maps (device-built)
};

// ---- PTX wrappers ----------------------------------------------------------
// Instruction descriptor of a block-scaled MMA: A/B formats [7,10)/[10,13)
// (mxf4: e2m1 = 1; mxf8f6f4: e2m1 = 5, e4m3 = 0), both K-major, N >> 3 at
// [17,23), ue8m0 scales (bit 23), M >> 4 at [24,29), and the byte of the
// scale column where A's / B's codes start at [29,31) / [4,6).
__device__ __forceinline__ uint32_t mx_idesc(int kind, int m, int n, uint32_t sf_id) {
    const uint32_t af = kind == kMxF4 ? 1u : 5u, bf = kind == kMxF4 ? 1u : 0u;
    return (sf_id << 4) | (af << 7) | (bf << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (1u << 23) | (static_cast<uint32_t>(m >> 4) << 24) | (sf_id << 29);
}
template <int KIND, bool PAIR>
__device__ __forceinline__ void mx_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate, uint32_t sfa, uint32_t sfb) {
    if (KIND == kMxF4) {
        if (PAIR)
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, "
                         "%3, [%5], [%6], p;\n\t}\n" ::"r"(d),
                         "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
                         : "memory");
        else
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, "
                         "%3, [%5], [%6], p;\n\t}\n" ::"r"(d),
                         "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
                         : "memory");
    } else {
        if (PAIR)
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, "
                         "[%5], [%6], p;\n\t}\n" ::"r"(d),
                         "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
                         : "memory");
        else
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, "
                         "[%5], [%6], p;\n\t}\n" ::"r"(d),
                         "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
                         : "memory");
    }
}
__device__ __forceinline__ void tc_st1(uint32_t taddr, uint32_t v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v)
                 : "memory");
}
__device__ __forceinline__ void tc_st2(uint32_t taddr, uint32_t v0, uint32_t v1) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(v0),
                 "r"(v1)
                 : "memory");
}
__device__ __forceinline__ void tc_st4(uint32_t taddr, const uint32_t (&v)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
                 : "memory");
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::
                     "r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                 "r"(v[7])
                 : "memory");
}
// 3-D tensor box into this CTA's shared memory, completion counted on a
// barrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const void *tmap, int x, int y, int z,
                                                 uint32_t cluster_bar, uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx"
                 "::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
                 "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(cluster_bar), "l"(policy)
                 : "memory");
}

// ---- token terms -----------------------------------------------------------
// Value of an e2m1 code (bit 3 sign, bits 2..1 exponent, bit 0 mantissa):
// 0, 0.5, 1, 1.5, 2, 3, 4, 6 and their negatives.
__device__ __forceinline__ float e2m1_value(uint32_t n) {
    const uint32_t e = (n >> 1) & 3u;
    const float mag = e == 0u ? 0.5f * static_cast<float>(n & 1u)
                              : __uint_as_float((e + 126u) << 23) * ((n & 1u) ? 1.5f : 1.f);
    return (n & 8u) ? -mag : mag;
}

// Rows of `src` (f16, [rows, K], K % 32 == 0) as NTERM block-scaled terms:
// planes [NTERM][rows][K/2] packed e2m1 (low nibble = even element) or
// [NTERM][rows][K] e4m3, and codes [NTERM][rows][K/32] ue8m0.  Term t
// quantises the residual the terms before it left: its code is the smallest
// c with 2^(c-127) >= amax/6 (e2m1) or amax/448 (e4m3) over the block's 32
// residuals, and its values are the residuals / 2^(c-127) rounded to nearest
// (cvt.rn.satfinite).  A block of zeros gets code 0 and zero values (the
// MMA reads code 0 as 2^-127, times zero).  A thread handles 8 elements; the
// 4 threads of a block are adjacent lanes.
template <int KIND, int NTERM>
__global__ void __launch_bounds__(256) mx_terms_kernel(const __half *__restrict__ src, int rows,
                                                       int K, uint8_t *__restrict__ planes,
                                                       uint8_t *__restrict__ codes) {
    const int per_row = K >> 3;
    const long long total = static_cast<long long>(rows) * per_row;
    const float inv_top = KIND == kMxF4 ? (1.f / 6.f) : (1.f / 448.f);
    const size_t plane_rows = static_cast<size_t>(rows);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(i / per_row);
        const int col = static_cast<int>(i - static_cast<long long>(row) * per_row) * 8;
        const uint4 raw = *reinterpret_cast<const uint4 *>(src + static_cast<size_t>(row) * K + col);
        float v[8];
        {
            const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h[j]);
                v[2 * j] = f.x;
                v[2 * j + 1] = f.y;
            }
        }
#pragma unroll
        for (int t = 0; t < NTERM; ++t) {
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                amax = fmaxf(amax, fabsf(v[j]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            uint32_t code;
            if (!(amax <= 3.402823466e38f)) {
                code = 255u; // inf / NaN rows: the MMA's NaN scale carries them
            } else if (amax == 0.f) {
                code = 0u;
            } else {
                const uint32_t b = __float_as_uint(amax * inv_top);
                const int ex = static_cast<int>(b >> 23);
                int e = ex == 0 ? -126 : ex - 127 + ((b & 0x7FFFFFu) ? 1 : 0);
                if (ex == 0 && b <= 0x00400000u)
                    e = -127; // 2^-127 already covers it
                code = static_cast<uint32_t>(max(0, min(253, e + 127)));
            }
            // inv = 2^(127 - code), s = 2^(code - 127): exact powers of two.
            const float inv = code <= 253u ? __uint_as_float((254u - min(code, 253u)) << 23) : 0.f;
            const float s = code == 0u ? __uint_as_float(0x00400000u)
                                       : __uint_as_float(min(code, 254u) << 23);
            const size_t prow = static_cast<size_t>(t) * plane_rows + row;
            if (KIND == kMxF4) {
                // Byte j holds elements 2j (low nibble) and 2j+1: cvt puts its
                // first source in the upper half.
                uint32_t word;
                asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
                    "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
                    "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
                    "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
                    "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
                    "mov.b32 %0, {b0, b1, b2, b3};\n\t}\n"
                    : "=r"(word)
                    : "f"(v[0] * inv), "f"(v[1] * inv), "f"(v[2] * inv), "f"(v[3] * inv),
                      "f"(v[4] * inv), "f"(v[5] * inv), "f"(v[6] * inv), "f"(v[7] * inv));
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    v[j] -= e2m1_value((word >> (4 * j)) & 15u) * s;
                *reinterpret_cast<uint32_t *>(planes + prow * (K / 2) + col / 2) = word;
            } else {
                uint32_t w[2] = {0, 0};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint16_t q;
                    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
                        : "=h"(q)
                        : "f"(v[2 * j + 1] * inv), "f"(v[2 * j] * inv));
                    w[j >> 1] |= static_cast<uint32_t>(q) << (16 * (j & 1));
                    uint32_t hh;
                    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hh) : "h"(q));
                    const float2 dq = __half22float2(*reinterpret_cast<const __half2 *>(&hh));
                    v[2 * j] -= dq.x * s;
                    v[2 * j + 1] -= dq.y * s;
                }
                *reinterpret_cast<uint2 *>(planes + prow * K + col) = make_uint2(w[0], w[1]);
            }
            if ((threadIdx.x & 3) == 0)
                codes[prow * (K / 32) + col / 32] = static_cast<uint8_t>(code);
        }
    }
}

// ---- tensor-pipe rate ----------------------------------------------------------
// Back-to-back MMAs of one kind on a resident tile (zeros, block scales of
// code 0): the tensor pipe's own rate for the kinds the expert FFN issues,
// measured in the same run as the kernels that use it.  KIND 0: mxf4 (K 64
// per MMA), 1: mxf8f6f4 (K 32), 2: f16 (K 16).  One CTA (or CTA pair) per SM,
// 128 threads; `iters` MMAs per CTA, then one commit and a bounded wait.
template <int KIND, bool PAIR>
__global__ void __launch_bounds__(128) mma_rate_kernel(int n, int iters, int *err) {
    __shared__ __align__(1024) uint8_t tile[2 * 128 * 128];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tslot;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 2 * 128 * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(tile)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        if (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&tslot)),
                         "r"(512)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&tslot)),
                         "r"(512)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    if (PAIR)
        cluster_sync();
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(&tslot);
    // Block scales (codes 0) in columns 256..271 of every lane quadrant.
    const uint32_t lane_addr = static_cast<uint32_t>(32 * warp) << 16;
    const uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    tc_st8(tmem + lane_addr + 256, z);
    tc_st8(tmem + lane_addr + 264, z);
    tc_wait_st();
    tc_fence_before();
    if (PAIR)
        cluster_sync();
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    bool ok = true;
    if (threadIdx.x == 0 && rank == 0) {
        const uint32_t a0 = smem_u32(tile), b0 = smem_u32(tile + 128 * 128);
        const int M = PAIR ? 256 : 128;
        for (int it = 0; it < iters; ++it) {
            const int kk = it & 3;
            const uint64_t ad = tc_desc_sw128(a0 + kk * 32), bd = tc_desc_sw128(b0 + kk * 32);
            if (KIND == 2) { // single-CTA form only (the host launches no f16 pair)
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::
                                     "r"(tmem),
                                 "l"(ad), "l"(bd), "r"(tc_idesc(M, n)), "r"(it != 0 ? 1u : 0u)
                                 : "memory");
            } else {
                mx_mma<KIND == 0 ? kMxF4 : kMxF8, PAIR>(tmem, ad, bd, mx_idesc(KIND == 0 ? kMxF4 : kMxF8, M, n, 0u),
                                                       it != 0, tmem + 256, tmem + 264);
            }
        }
        if (PAIR) {
            tc_commit_pair(cluster_addr(&bar, 0));
            tc_commit_pair(cluster_addr(&bar, 1));
        } else {
            tc_commit_solo(&bar);
        }
        ok = mbar_wait(&bar, 0, err);
    } else if ((threadIdx.x & 31) == 0) {
        ok = mbar_wait(&bar, 0, err);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    // An MMA that never completed leaves its TMEM alone (the error word says so).
    if (!__syncthreads_and(ok))
        return;
    tc_fence_before();
    if (PAIR)
        cluster_sync();
    else
        __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        if (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(512)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(512)
                         : "memory");
    }
}

// ---- the block-scaled expert FFN -------------------------------------------
// A ring slot of depth `depth` may be refilled for stage k once stage
// k - depth is consumed: wait for that stage's phase of the stage-empty ring
// (SD >= depth barriers, so the barrier cannot have moved on a whole phase
// past it: the MMAs cannot pass stage k before this slot is refilled).
template <int SD>
__device__ __forceinline__ bool mx_slot_free(uint64_t *st_empty, uint32_t k, uint32_t depth,
                                             int *err) {
    if (k < depth)
        return true;
    const uint32_t j = k - depth;
    return mbar_wait(&st_empty[j % SD], (j / SD) & 1u, err);
}

template <int KIND, int NTERM, int PHASE, bool PAIR>
__global__ void __launch_bounds__(MxCfg<KIND, NTERM, PAIR>::THREADS,
                                  MxCfg<KIND, NTERM, PAIR>::CTAS_PER_SM)
    tc_mx_kernel(const MxArgs ma, const __grid_constant__ CUtensorMap tok_map,
                 const __grid_constant__ CUtensorMap tsc_map) {
    using C = MxCfg<KIND, NTERM, PAIR>;
    const TcArgs &p = ma.t;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *a_full = bars, *b_full = a_full + C::SA, *sf_full = b_full + C::SB;
    uint64_t *st_empty = sf_full + C::SSF; // [SD]: stage k consumed (k % SD)
    uint64_t *sa_full = st_empty + C::SD, *sa_empty = sa_full + C::NSC;
    uint64_t *sb_full = sa_empty + C::NSC, *sb_empty = sb_full + C::NSC;
    uint64_t *acc_full = sb_empty + C::NSC, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    int *off_s = reinterpret_cast<int *>(smem + C::OFF_ITEMS);
    int *cnt_s = off_s + C::ITEM_TAB;
    const bool tab_in_smem = p.nb + 1 <= C::ITEM_TAB;
    if (tab_in_smem) {
        for (int e = threadIdx.x; e <= p.nb; e += blockDim.x) {
            off_s[e] = __ldg(p.item_off + e);
            cnt_s[e] = e < p.nb ? __ldg(p.cnt + e) : 0;
        }
    }
    const TcItemTab tab{tab_in_smem ? off_s : p.item_off, tab_in_smem ? cnt_s : p.cnt};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int unit = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
    const int nunits = PAIR ? static_cast<int>(nclusters_x()) : static_cast<int>(gridDim.x);
    const int total = __ldg(p.item_off + p.nb);
    if (unit >= total)
        return; // no item (for a pair: both CTAs leave) -- before touching TMEM

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::SA; ++s)
            mbar_init(&a_full[s], 1); // the weight producer's expect_tx (leader: both CTAs' bytes)
        for (int s = 0; s < C::SB; ++s)
            mbar_init(&b_full[s], 1);
        for (int s = 0; s < C::SSF; ++s)
            mbar_init(&sf_full[s], C::SF_ARRIVALS);
        for (int s = 0; s < C::SD; ++s)
            mbar_init(&st_empty[s], 1); // the (leader's) tcgen05.commit of the stage
        for (int s = 0; s < C::NSC; ++s) {
            mbar_init(&sa_full[s], 1);
            mbar_init(&sa_empty[s], 4);
            mbar_init(&sb_full[s], 1);
            mbar_init(&sb_empty[s], 4);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TcCfg<PAIR>::ACC_EMPTY_ARRIVALS);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == C::MMA_WARP) {
        if (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"(C::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"(C::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    if (PAIR)
        cluster_sync();
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    const int nk = p.K / C::KSTAGE; // stages per item

    if (warp == C::TOK_WARP) {
        // --------------------------------------- token producer (terms + codes)
        if (lane == 0) {
            const uint64_t pol_t = policy_evict_last();
            uint32_t b_it = 0, w_it = 0;
            bool ok = true;
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR>(p, tab, i, it);
                if (C::STACK)
                    it.nmma = C::NT; // stacked terms: whole 64-row planes
                const int rows = PAIR ? it.nmma >> 1 : it.nmma; // this CTA's token rows
                const int xr0 = __ldg(p.xrow + it.e) + it.t0;
                const int xr = xr0 + static_cast<int>(rank) * rows;
                const int nbox = (rows + kTcTokBox - 1) / kTcTokBox;
                const int nsbox = (it.nmma + kTcTokBox - 1) / kTcTokBox; // codes: the full tile
                for (int kb = 0; kb < nk; ++kb) {
                    if (kb % C::WST == 0) {
                        const uint32_t w = w_it % C::NSC;
                        if (!mbar_wait(&sb_empty[w], ((w_it / C::NSC) & 1u) ^ 1u, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&sb_full[w], NTERM * nsbox * kTcTokBox * 16);
                        uint8_t *sdst = smem + C::OFF_SCB + w * C::SCB_SLOT;
                        const int xs = (kb / C::WST) * 16;
                        for (int t = 0; t < NTERM; ++t)
                            for (int j = 0; j < nsbox; ++j)
                                tma_load_3d(sdst + (t * C::NT + j * kTcTokBox) * 16, &tsc_map, xs,
                                            xr0 + j * kTcTokBox, t, &sb_full[w], pol_t);
                        ++w_it;
                    }
                    const uint32_t s = b_it % C::SB;
                    if (!mx_slot_free<C::SD>(st_empty, b_it, C::SB, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst = smem + s * C::B_SLOT;
                    const int xb = kb * 128; // byte column of a term row
                    if (PAIR) {
                        if (rank == 0)
                            mbar_arrive_expect_tx(&b_full[s], 2u * NTERM * nbox * kTcTokBox * 128);
                        const uint32_t fb = cluster_addr(&b_full[s], 0);
                        for (int t = 0; t < NTERM; ++t)
                            for (int j = 0; j < nbox; ++j)
                                tma_load_3d_pair(dst + t * C::PLANE + j * kTcTokBox * 128, &tok_map,
                                                 xb, xr + j * kTcTokBox, t, fb, pol_t);
                    } else {
                        mbar_arrive_expect_tx(&b_full[s], NTERM * nbox * kTcTokBox * 128);
                        for (int t = 0; t < NTERM; ++t)
                            for (int j = 0; j < nbox; ++j)
                                tma_load_3d(dst + t * C::PLANE + j * kTcTokBox * 128, &tok_map, xb,
                                            xr + j * kTcTokBox, t, &b_full[s], pol_t);
                    }
                    ++b_it;
                }
            }
            if (!ok || load_volatile(p.err) != 0) {
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
            // Every code window in flight has landed before the CTA ends.
            for (uint32_t j = w_it > C::NSC ? w_it - C::NSC : 0; j < w_it; ++j)
                mbar_wait(&sb_full[j % C::NSC], (j / C::NSC) & 1u, nullptr);
        }
    } else if (warp == C::W_WARP) {
        // ----------------------------------------- weight producer (rows + codes)
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const bool fence_maps = __ldg(p.tmaps_dirty) != 0;
            uint32_t a_it = 0, w_it = 0;
            bool ok = true;
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR>(p, tab, i, it);
                const uint8_t *tm = ma.tmaps + static_cast<size_t>(it.e) * kMxMapCount * kTcMapBytes;
                if (fence_maps)
                    for (int m = 0; m < kMxMapCount; ++m)
                        tmap_acquire(tm + m * kTcMapBytes);
                const int r0 = it.c0 + static_cast<int>(rank) * tc_cols_per_item<PHASE, false>();
                for (int kb = 0; kb < nk; ++kb) {
                    if (kb % C::WST == 0) {
                        const uint32_t w = w_it % C::NSC;
                        if (!mbar_wait(&sa_empty[w], ((w_it / C::NSC) & 1u) ^ 1u, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&sa_full[w], C::SCA_SLOT);
                        uint8_t *sdst = smem + C::OFF_SCA + w * C::SCA_SLOT;
                        const int xs = (kb / C::WST) * 16;
                        if (PHASE == 1) {
                            tma_load_2d(sdst, tm + kMxGateS * kTcMapBytes, xs, r0, &sa_full[w], pol_w);
                            tma_load_2d(sdst + 1024, tm + kMxUpS * kTcMapBytes, xs, r0, &sa_full[w],
                                        pol_w);
                        } else {
                            tma_load_2d(sdst, tm + kMxDownS * kTcMapBytes, xs, r0, &sa_full[w], pol_w);
                        }
                        ++w_it;
                    }
                    const uint32_t s = a_it % C::SA;
                    if (!mx_slot_free<C::SD>(st_empty, a_it, C::SA, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst = smem + C::OFF_A + s * C::A_SLOT;
                    // x of the weight maps: bytes (mxf4, packed) or 4-bit elements (mxf8f6f4).
                    const int xa = kb * 128;
                    // Transaction bytes: the packed bytes read (the padded form
                    // of mxf8f6f4 counts its global size).
                    constexpr uint32_t ABYTES = KIND == kMxF4 ? 128u * 128u : 128u * 64u;
                    uint32_t fb = 0;
                    if (PAIR) {
                        if (rank == 0)
                            mbar_arrive_expect_tx(&a_full[s], 2u * ABYTES);
                        fb = cluster_addr(&a_full[s], 0);
                    } else {
                        mbar_arrive_expect_tx(&a_full[s], ABYTES);
                    }
                    if (PHASE == 1) {
                        // Quadrant q: gate rows r0+16q.. at 32q, up rows at 32q+16.
                        for (int q = 0; q < 4; ++q) {
                            for (int gu = 0; gu < 2; ++gu) {
                                uint8_t *d = dst + (32 * q + 16 * gu) * 128;
                                const void *m = tm + (gu ? kMxUpP : kMxGateP) * kTcMapBytes;
                                if (PAIR)
                                    tma_load_2d_pair(d, m, xa, r0 + 16 * q, fb, pol_w);
                                else
                                    tma_load_2d(d, m, xa, r0 + 16 * q, &a_full[s], pol_w);
                            }
                        }
                    } else {
                        const void *m = tm + kMxDownP * kTcMapBytes;
                        if (PAIR)
                            tma_load_2d_pair(dst, m, xa, r0, fb, pol_w);
                        else
                            tma_load_2d(dst, m, xa, r0, &a_full[s], pol_w);
                    }
                    ++a_it;
                }
            }
            if (!ok || load_volatile(p.err) != 0) {
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
            for (uint32_t j = w_it > C::NSC ? w_it - C::NSC : 0; j < w_it; ++j)
                mbar_wait(&sa_full[j % C::NSC], (j / C::NSC) & 1u, nullptr);
        }
    } else if (warp == C::MMA_WARP) {
        // ------------------------------------ MMA issuer (a pair's leader only)
        if (lane == 0 && rank == 0) {
            uint32_t a_it = 0, b_it = 0, f_it = 0;
            TcAccState acc;
            bool ok = true;
            const uint32_t b_base = smem_u32(smem);
            const uint32_t a_base = smem_u32(smem + C::OFF_A);
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR>(p, tab, i, it);
                const int b = acc.take(!C::STACK && it.nmma > C::ACC_HALF);
                if (b != 1 && !mbar_wait(&acc_empty[0], (acc.use[0] & 1u) ^ 1u, p.err))
                    ok = false;
                if (ok && b != 0 && !mbar_wait(&acc_empty[1], (acc.use[1] & 1u) ^ 1u, p.err))
                    ok = false;
                if (!ok)
                    break;
                tc_fence_after();
                const uint32_t d = tmem + (b == 1 ? static_cast<uint32_t>(C::ACC_COLS) : 0u);
                // Everything an MMA needs is a per-item or per-stage base plus a
                // compile-time offset: instruction descriptors for the two
                // scale-byte positions, the operand descriptors (address >> 4
                // in the low bits) and the scale columns.
                const uint32_t id0 =
                    mx_idesc(KIND, PAIR ? 256 : 128, C::STACK ? NTERM * C::NT : it.nmma, 0u);
                constexpr uint32_t kSfStep = (1u << 4) | (1u << 29); // sf_id += 1 for A and B
                // Ring bases as descriptors (start address >> 4 in bits 0..13;
                // every address stays below 256 KB, so offsets add in place).
                const uint64_t adesc_base = tc_desc_sw128(a_base), bdesc_base = tc_desc_sw128(b_base);
                for (int kb = 0; kb < nk; ++kb) {
                    const uint32_t sa = a_it % C::SA, sb = b_it % C::SB, sf = f_it % C::SSF;
                    if (!mbar_wait(&a_full[sa], (a_it / C::SA) & 1u, p.err) ||
                        !mbar_wait(&b_full[sb], (b_it / C::SB) & 1u, p.err) ||
                        !mbar_wait(&sf_full[sf], (f_it / C::SSF) & 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = adesc_base + ((sa * C::A_SLOT) >> 4);
                    const uint64_t bd = bdesc_base + ((sb * C::B_SLOT) >> 4);
                    const uint32_t sfa0 = tmem + C::SF_BASE + sf * C::SF_COLS;
                    const uint32_t sfb0 = sfa0 + 4 * C::G;
                    const uint32_t acc0 = kb != 0 ? 1u : 0u;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t g = KIND == kMxF4 ? static_cast<uint32_t>(kk >> 1) : 0u;
                        const uint32_t id = KIND == kMxF4 ? static_cast<uint32_t>(kk & 1) * 2u
                                                          : static_cast<uint32_t>(kk);
                        const uint32_t idesc = id0 + id * kSfStep;
                        const uint32_t tsfa = (sfa0 + 4 * g) | (id << 30);
                        if (C::STACK) {
                            // All terms in one MMA: B rows 64t.. are term t's tokens.
                            const uint32_t tsfb = (sfb0 + g * NTERM * C::NBMAX) | (id << 30);
                            mx_mma<KIND, PAIR>(d, ad + 2 * kk, bd + 2 * kk, idesc,
                                               kk != 0 ? 1u : acc0, tsfa, tsfb);
                        } else {
#pragma unroll
                            for (int t = 0; t < NTERM; ++t) {
                                const uint32_t tsfb =
                                    (sfb0 + (t * C::G + g) * C::NBMAX) | (id << 30);
                                mx_mma<KIND, PAIR>(d, ad + 2 * kk,
                                                   bd + ((t * C::PLANE) >> 4) + 2 * kk, idesc,
                                                   (kk | t) != 0 ? 1u : acc0, tsfa, tsfb);
                            }
                        }
                    }
                    const uint32_t se = a_it % C::SD; // a_it == b_it == f_it: the stage index
                    if (PAIR) {
                        tc_commit_pair(cluster_addr(&st_empty[se], 0));
                        tc_commit_pair(cluster_addr(&st_empty[se], 1));
                    } else {
                        tc_commit_solo(&st_empty[se]);
                    }
                    ++a_it;
                    ++b_it;
                    ++f_it;
                }
                if (!ok)
                    break;
                for (int h = 0; h < 2; ++h) {
                    if (b == 1 - h)
                        continue;
                    if (PAIR) {
                        tc_commit_pair(cluster_addr(&acc_full[h], 0));
                        tc_commit_pair(cluster_addr(&acc_full[h], 1));
                    } else {
                        tc_commit_solo(&acc_full[h]);
                    }
                    ++acc.use[h];
                }
            }
            if (PAIR)
                tc_commit_pair(cluster_addr(done, 0));
            else
                tc_commit_solo(done);
            mbar_wait(done, 0, nullptr);
        }
    } else if (warp >= C::SF_WARP0 && warp < C::SF_WARP0 + 4) {
        // -------------------------------------------- SF warps: codes -> TMEM
        const int q = warp & 3;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
        // This lane's weight row inside the CTA's 128 (its TMEM lane): phase 1
        // gate rows in lanes 0-15 of a quadrant, up rows in 16-31.
        int sa_off;
        if (PHASE == 1)
            sa_off = (lane < 16 ? 0 : 1024) + (16 * q + (lane & 15)) * 16;
        else
            sa_off = (32 * q + lane) * 16;
        uint32_t f_it = 0, w_it = 0;
        bool ok = true;
        for (int i = unit; ok && i < total; i += nunits) {
            TcItem it;
            tc_item<PHASE, PAIR>(p, tab, i, it);
            if (C::STACK)
                it.nmma = C::NT;
            const int nb = (it.nmma + 31) >> 5; // token-code columns in use
            uint32_t wa = 0, wb = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int ks = kb % C::WST;
                if (ks == 0) {
                    wa = w_it % C::NSC;
                    wb = wa;
                    const uint32_t par = (w_it / C::NSC) & 1u;
                    if (!__all_sync(0xffffffffu, mbar_wait(&sa_full[wa], par, p.err) &&
                                                     mbar_wait(&sb_full[wb], par, p.err))) {
                        ok = false;
                        break;
                    }
                }
                const uint32_t sf = f_it % C::SSF;
                if (!__all_sync(0xffffffffu, mx_slot_free<C::SD>(st_empty, f_it, C::SSF, p.err))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t col0 = tmem + lane_addr + C::SF_BASE + sf * C::SF_COLS;
                const uint8_t *wina = smem + C::OFF_SCA + wa * C::SCA_SLOT + sa_off;
                const uint8_t *winb = smem + C::OFF_SCB + wb * C::SCB_SLOT;
#pragma unroll
                for (int g = 0; g < C::G; ++g) {
                    const int word = ks * C::G + g; // 4-code group inside the 16-byte window
                    const uint32_t va = lds32(smem_u32(wina + 4 * word));
                    // 255 would be NaN to the MMA but +inf to the reference.
                    if (__vcmpeq4(va, 0xFFFFFFFFu))
                        flag_range(p);
                    tc_st1(col0 + 4 * g + q, va);
#pragma unroll
                    for (int t = 0; t < NTERM; ++t) {
                        const uint32_t cb = col0 + 4 * C::G +
                                            (C::STACK ? (g * NTERM + t) : (t * C::G + g)) * C::NBMAX;
                        if (PAIR) {
                            uint32_t vb[8];
#pragma unroll
                            for (int n1 = 0; n1 < 8; ++n1)
                                vb[n1] = n1 < nb ? lds32(smem_u32(
                                                       winb + ((t * C::NT) + lane + 32 * n1) * 16 +
                                                       4 * word))
                                                 : 0u;
                            tc_st8(cb, vb);
                        } else {
                            const uint32_t v0 =
                                lds32(smem_u32(winb + ((t * C::NT) + lane) * 16 + 4 * word));
                            const uint32_t v1 =
                                nb > 1 ? lds32(smem_u32(winb + ((t * C::NT) + lane + 32) * 16 +
                                                        4 * word))
                                       : 0u;
                            tc_st2(cb, v0, v1);
                        }
                    }
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR)
                        mbar_arrive_cluster(cluster_addr(&sf_full[sf], 0));
                    else
                        mbar_arrive(&sf_full[sf]);
                    if (ks == C::WST - 1) {
                        mbar_arrive(&sa_empty[wa]);
                        mbar_arrive(&sb_empty[wb]);
                    }
                }
                if (ks == C::WST - 1)
                    ++w_it;
                ++f_it;
            }
        }
    } else if (warp < C::EPI_WARPS) {
        if (C::STACK)
            tc_epilogue<MVLLM_FMT_MXFP4, PHASE, PAIR, NTERM, C::NT, C::ACC_COLS, C::NT>(
                p, tab, unit, nunits, total, tmem, rank, acc_full, acc_empty, warp, lane);
        else
            tc_epilogue<MVLLM_FMT_MXFP4, PHASE, PAIR>(p, tab, unit, nunits, total, tmem, rank,
                                                      acc_full, acc_empty, warp, lane);
    }

    tc_fence_before();
    if (PAIR)
        cluster_sync();
    else
        __syncthreads();
    if (warp == C::MMA_WARP) {
        tc_fence_after();
        if (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(C::TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(C::TMEM_COLS)
                         : "memory");
    }
}

} // namespace mvb
