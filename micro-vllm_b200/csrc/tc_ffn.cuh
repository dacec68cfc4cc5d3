// tc_ffn.cuh -- tensor-core expert FFN (tcgen05 + TMEM, CTA pairs) for experts
// with many rows (prefill chunks, skewed routing).
//
// Same contract as the decode kernels (decode_ffn.cuh): phase 1 computes
//   h[r, j] = act(sum_k x[r,k] g[j,k], sum_k x[r,k] u[j,k])   (f16, stage_pos order)
// and phase 2 computes
//   y[r, n] = sum_j h[r,j] d[n,j]           (f32 sums, stored as f16)
// for the rows r of every expert the plan gave to this path
// (reference: moe_block's per-expert loop, metal_ops.cpp:466-509, through
// matmul_mxfp4 / matmul_int4_g64 in quant.cpp:104-123 / 61-102).
//
// The product is computed transposed, weights as the MMA's M side, by a pair
// of CTAs on the two SMs of a TPC (tcgen05 cta_group::2):
//   D[w, t] = sum_k W[w, k] * X[t, k]    M = 256 weight rows, N <= 256 tokens.
// - W (A operand) lives in tensor memory, 128 rows in each CTA of the pair.
//   Dequant warps read the packed rows (TMA box, 64-byte swizzle) and the
//   group scales, convert e2m1 / int4 to f16 with the scale folded in, and
//   store them with tcgen05.st: the weights never pass through shared memory.
// - X (B operand) is a token tile in shared memory, N/2 rows in each CTA:
//   TMA boxes of the staged f16 rows (128-byte swizzle, K-major) read by the
//   MMA through a matrix descriptor.  N is the tile's row count rounded up to
//   32, so an expert with 20 rows pays for 32, not for a 256-row tile.
// - D accumulates in f32 in tensor memory, 128 rows x N columns per CTA.
// One MMA instruction covers 256 x N x 16 on two SMs, so a pair issues half
// the instructions of two single-CTA MMAs and each SM reads and fills only
// half of the token tile: both limits (one issuing thread, 128 B/clk of
// shared memory) sit below the tensor rate at N = 256.
//
// Exactness of the folded scale: an MXFP4 weight is e2m1 * 2^(s-127).  As an
// f16 product it is exact for s in [104, 140] and for s = 0 (+0) and 255 (inf,
// as the reference decodes it).  Codes below 104 lose bits below 2^-24
// (absolute error under 2^-25 per weight).  Codes 141..254 would overflow:
// the dequant warps raise the call's redo word and the decode kernels
// recompute the call's tensor-core experts (f32 scale arithmetic).  int4-g64 weights are (q-8) * scale rounded once to f16.
//
// Warp roles (608 threads per CTA, one CTA per SM, both CTAs of a pair walk
// the pair's item list):
//   warps 0-7   epilogue: TMEM -> registers -> activation -> global
//   warps 8-15  dequant: packed weights -> f16 -> TMEM (A operand); the two
//               groups of four take even and odd k-blocks
//   warp 16     token producer: TMA of this CTA's half of the token tile
//   warp 17     MMA issuer (one thread of the pair's even CTA) and TMEM allocator
//   warp 18     weight producer: TMA of packed weight rows, which run up to
//               16 k-blocks ahead of the MMAs (their HBM latency is longer),
//               and of the rows' scale windows (16 bytes per row); the
//               dequant warps issue no global loads, so their cluster-scope
//               release arrivals wait on nothing but their own TMEM stores
// A warp may only touch the TMEM lanes of its quadrant (warp id % 4), which
// is why epilogue and dequant warps come in groups of four.
//
// Barriers that gather the pair live in the even CTA ("leader"): its stage
// `full` barriers receive both CTAs' token bytes (TMA .cta_group::2) and both
// CTAs' dequant arrivals; its accumulator `empty` barriers both CTAs'
// epilogue arrivals.  The leader's commits arrive on the `empty` and
// accumulator `full` barriers of both CTAs.
#pragma once

#include "common.cuh"

namespace mvb {

constexpr int kTcKb = 64;         // k elements per k-block: one 128-byte swizzle atom of f16
constexpr int kTcTokBox = 64;     // token rows per TMA box
constexpr int kTcPkSlots = 8;     // packed-weight ring depth (2 k-blocks per slot)
constexpr int kTcScSlots = 3;     // scale ring depth (one 16-byte window per row per slot)
constexpr int kTcSoloMax = 64;    // token tiles of at most this many rows run on single CTAs
constexpr int kTcWideMax = 192;   // ... of at most this many on wide single CTAs (one per SM)

// The three forms of the kernel.  PAIR: CTA pairs, M = 256 weight rows per
// MMA, token tiles of up to 256 rows, one CTA per SM.  Solo: one CTA, M = 128,
// token tiles of up to 64 rows, two CTAs per SM.  WIDE solo: one CTA per SM,
// M = 128, token tiles of up to kTcWideMax rows, eight dequant and eight
// epilogue warps.  A pair MMA takes about 108 cycles to issue whatever its N
// (measured on B200), a single-CTA MMA about 45: the pair wins at N = 256 (it
// runs at the tensor rate), a tile of a few dozen tokens is bound by issue,
// so it runs on single CTAs, two per SM, each with its own issuing thread;
// between the two (a 65..192-row rest, e.g. 171 rows per expert at config[4]),
// one CTA per SM (about 123 cycles per N = 176 MMA) beats a pair bound by its
// issue.  The wide tile is bound by shared-memory bandwidth: per MMA its
// token slice (5.6 KB) is written by TMA and read by the MMA, with 1 KB of
// packed weights read by the dequant warps, about 96 cycles at 128 B/clk;
// the tensor pipe alone would take 88.
template <bool PAIR, bool WIDE = false> struct TcCfg {
    static constexpr bool BIG = PAIR || WIDE;     // one CTA per SM, 8 + 8 warps
    static constexpr int EPI_WARPS = BIG ? 8 : 4; // quadrant = warp % 4, chunk half = warp / 4
    static constexpr int DQ_SETS = BIG ? 2 : 1;   // sets of 4 dequant warps (k-block parity)
    static constexpr int DQ_WARP0 = EPI_WARPS;
    static constexpr int DQ_WARPS = 4 * DQ_SETS;
    static constexpr int PROD_WARP = DQ_WARP0 + DQ_WARPS;
    static constexpr int MMA_WARP = PROD_WARP + 1;
    static constexpr int PK_WARP = PROD_WARP + 2;
    static constexpr int THREADS = (PK_WARP + 1) * 32; // 608 / 352
    static constexpr int CTAS_PER_SM = BIG ? 1 : 2;
    static constexpr int NT = PAIR ? 256 : WIDE ? kTcWideMax : kTcSoloMax; // item token tile
    static constexpr int NALIGN = PAIR ? 32 : 16;      // MMA N granularity
    static constexpr int ACC_HALF = BIG ? 128 : 64;    // TMEM columns of one accumulator half
    static constexpr int A_BASE = 2 * ACC_HALF;
    static constexpr int STAGES = PAIR ? 4 : WIDE ? 3 : 2; // token + A ring (2 k-blocks each)
    static constexpr int PK_SLOTS = kTcPkSlots;        // packed-weight ring depth
    static constexpr int TMEM_COLS = BIG ? 512 : 256;
    static constexpr int TOK_ROWS = PAIR ? NT / 2 : NT; // token rows one CTA holds
    static constexpr int FULL_ARRIVALS = 1 + (PAIR ? 16 : DQ_WARPS); // producer + dequant warps
    static constexpr int ACC_EMPTY_ARRIVALS = PAIR ? 2 * EPI_WARPS : EPI_WARPS;
    static_assert(A_BASE + STAGES * 64 <= TMEM_COLS, "TMEM budget");
    static_assert(NT <= 2 * ACC_HALF, "accumulator columns");
};
enum { kTcGateP = 0, kTcUpP, kTcDownP, kTcGateS, kTcUpS, kTcDownS, kTcMapCount };
constexpr int kTcMapBytes = 128;

struct TcArgs {
    const uint8_t *tmaps;     // [nb][kTcMapCount] packed-weight maps (device-built)
    const int *tmaps_dirty;   // non-zero: maps were rewritten, acquire before use
    const void *const *s0;    // phase 1: gate scales, phase 2: down scales
    const void *const *s1;    // phase 1: up scales
    const int *xrow;          // per expert: first operand row (token map row)
    const int *orow;          // per expert: first output row
    const int *cnt;           // per expert: rows on this path (0 = decode path)
    const int *item_off;      // [nb + 1] item prefix of this list
    int small_max;            // rest tiles of at most this many rows are single-CTA items
    int wide_max;             // ... of at most this many (above small_max) wide items
    int tshift;               // pair token tiles are 2^tshift rows (the plan's split)
    int nb;
    int K, O;                 // reduction length, output width (I or D)
    void *out;                // phase 1: f16 h [rows, I]; phase 2: f16 y [rows, D]
    int act;
    float act_a, act_b;
    int *err;
    int *range;               // raised for scale codes this kernel cannot represent: the
                              // decode kernels then redo the call's tensor-core experts
};

// Scale codes the operands cannot represent: with a redo word the call's
// tensor-core experts are recomputed on the decode kernels; without one the
// call fails with MVLLM_ERR_RANGE.
__device__ __forceinline__ void flag_range(const TcArgs &p) {
    if (p.range)
        *reinterpret_cast<volatile int *>(p.range) = 1;
    else
        set_error(p.err, MVLLM_ERR_RANGE);
}

// Per CTA: TMEM columns [0, 2 * ACC_HALF) accumulators -- one buffer of both
// halves for a tile wider than a half, or two halves that alternate between
// narrower tiles (the epilogue of one overlaps the MMAs of the next); then
// one 64-column A stage (128 weight rows x 128 f16: two k-blocks) per ring
// stage.  A stage holds two k-blocks so that one wait and one commit cover
// eight MMAs.
template <bool PAIR, bool WIDE = false> struct TcLayout {
    using C = TcCfg<PAIR, WIDE>;
    static constexpr int TOK_KB = C::TOK_ROWS * 128;   // this CTA's token rows, one k-block
    static constexpr int TOK_STAGE = 2 * TOK_KB;        // a stage holds two k-blocks
    static constexpr int PK_STAGE = 128 * 64;           // 128 weight rows x 64 B (2 k-blocks)
    static constexpr int SC_STAGE = 128 * 16;           // 128 weight rows x one scale window
    static constexpr int A_COLS = 64; // two k-blocks of 128 rows x 64 f16
    static constexpr int OFF_PK = C::STAGES * TOK_STAGE;
    static constexpr int OFF_SC = OFF_PK + C::PK_SLOTS * PK_STAGE;
    static constexpr int OFF_BAR = OFF_SC + kTcScSlots * SC_STAGE;
    static constexpr int NBARS = 2 * C::STAGES + 2 * C::PK_SLOTS + 2 * kTcScSlots + 4 + 1;
    static constexpr int ITEM_TAB = 512; // item offsets and row counts of up to 511 experts
    static constexpr int OFF_ITEMS = OFF_BAR + NBARS * 8 + 16;
    static constexpr int SMEM = OFF_ITEMS + 2 * ITEM_TAB * 4 + 1024; // + alignment
    static_assert(SMEM * C::CTAS_PER_SM <= 232448, "dynamic shared memory per SM");
};

// Output columns per item: phase 1 takes 64 h columns (64 gate + 64 up rows)
// per 128 weight rows, phase 2 takes 128 down rows; a pair item holds twice
// that, half in each CTA.
template <int PHASE, bool PAIR> __host__ __device__ constexpr int tc_cols_per_item() {
    return (PHASE == 1 ? 64 : 128) * (PAIR ? 2 : 1);
}


// k-blocks per 16-byte scale window of a row: 8 for MXFP4 (two ue8m0 bytes per
// k-block), 4 for int4-g64 (one f32 per k-block).
template <int FMT> __host__ __device__ constexpr int tc_kb_per_window() {
    return FMT == MVLLM_FMT_MXFP4 ? 8 : 4;
}

// ---- cluster / CTA-pair helpers -------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// One arrival on a barrier of either CTA of the pair.  The data it publishes
// is tensor memory, ordered by tcgen05.wait::st + tcgen05.fence pairs around
// the barrier, so the arrival keeps the default CTA-scope release: a
// cluster-scope release measured about 1000 cycles per arrival here.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Barriers the other CTA of the pair arrives on are waited on like local ones.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *err) {
    return mbar_wait(bar, parity, err);
}
// Tensor TMA box into this CTA's shared memory whose completion is counted
// on a barrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *tmap, int x, int y,
                                                 uint32_t cluster_bar, uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx"
                 "::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
                 "l"(tmap), "r"(x), "r"(y), "r"(cluster_bar), "l"(policy)
                 : "memory");
}

// ---- tcgen05 wrappers ---------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrival on a barrier of either CTA once this thread's earlier pair MMAs completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     cluster_bar)
                 : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T over the CTA pair, f16 in, f32 accumulate.
__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
                 "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
__device__ __forceinline__ void tc_commit_solo(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T on this CTA, f16 in, f32 accumulate.
__device__ __forceinline__ void tc_mma_solo(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
                 "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

#define MVB_R32(v)                                                                             \
    "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),     \
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),     \
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),   \
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),   \
        "r"(v[29]), "r"(v[30]), "r"(v[31])
#define MVB_W32(v)                                                                             \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),         \
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),            \
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),         \
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),         \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),         \
        "=r"(v[31])

// This warp's 32 lanes x 32 consecutive columns, one row (lane) per thread.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, "
                 "%9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, "
                 "%25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
                 MVB_R32(v)
                 : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, "
                 "%9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, "
                 "%25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : MVB_W32(v)
                 : "r"(taddr)
                 : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start >> 4 [0,14), leading offset >> 4 [16,30) (unused by this
// swizzle, 1), stride offset >> 4 [32,46), version 1 [46,48), layout 2
// (128-byte swizzle) [61,64).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: f32 accumulate [4,6)=1, A and B f16 (0), both
// K-major, N >> 3 at [17,23), M >> 4 at [24,29) (256 over a pair, else 128).
__device__ __forceinline__ uint32_t tc_idesc(int m, int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Word i (0..3) of v without a local-memory array.
__device__ __forceinline__ uint32_t sel4(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct TcItem {
    int e;     // expert
    int t0;    // first row of the item's token tile (relative to the expert)
    int n;     // real rows in the tile
    int nmma;  // MMA N: n rounded up to the MMA's granularity
    int c0;    // first output column of the item (h column or y column)
};

// Item i of a list: experts in plan order; inside an expert the weight tile
// varies slowest and the token tile fastest, so CTAs working at the same
// time share the weight rows through L2.  Pair lists hold an expert's
// 256-row tiles (and a wider rest); solo lists its narrow rest, if any.
// The item offsets and row counts live in shared memory (when the experts
// fit the table), so the binary search costs no global round trips: every
// role resolves every item itself.
struct TcItemTab {
    const int *off; // [nb + 1] item offsets of this list
    const int *cnt; // [nb] rows per expert
};

template <int PHASE, bool PAIR, bool WIDE = false>
__device__ __forceinline__ void tc_item(const TcArgs &p, const TcItemTab &tab, int i, TcItem &it) {
    using C = TcCfg<PAIR, WIDE>;
    int lo = 0, hi = p.nb;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tab.off[mid] <= i)
            lo = mid;
        else
            hi = mid;
    }
    const int e = lo;
    const int local = i - tab.off[e];
    const int c = tab.cnt[e];
    int npair, nsolo, nwide;
    tc_tiles3(c, p.small_max, p.wide_max, p.tshift, npair, nsolo, nwide);
    const int ntt = PAIR ? npair : 1;
    const int wg = local / ntt, tt = local - wg * ntt;
    it.e = e;
    it.t0 = PAIR ? tt << p.tshift : (c >> p.tshift) << p.tshift;
    it.n = min(PAIR ? (1 << p.tshift) : C::NT, c - it.t0);
    it.nmma = (it.n + C::NALIGN - 1) & ~(C::NALIGN - 1);
    it.c0 = wg * tc_cols_per_item<PHASE, PAIR>();
}

// Accumulator buffers: a tile of more than 128 tokens takes both 128-column
// halves (one 256-column accumulator), smaller tiles alternate between them.
// The MMA issuer and the epilogue walk the same item sequence and keep this
// state identically.
struct TcAccState {
    uint32_t use[2] = {0, 0}; // completed uses of each half
    uint32_t next = 0;        // half the next small tile takes
    __device__ __forceinline__ int take(bool full) { // returns 0/1 (half) or 2 (both)
        if (full) {
            next = 0;
            return 2;
        }
        const int b = static_cast<int>(next);
        next ^= 1u;
        return b;
    }
};

// Dequantized A operand for one k-block of one weight row: 32 f16x2 words.
template <int FMT>
__device__ __forceinline__ void tc_dequant_row(const uint4 &w0, const uint4 &w1, __half2 sc0,
                                               __half2 sc1, uint32_t (&v)[32]) {
    const uint32_t pw[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t h[4];
        if (FMT == MVLLM_FMT_MXFP4)
            e2m1x8_to_f16x8(pw[c], h[0], h[1], h[2], h[3]);
        else
            int4x8_to_f16x8(pw[c], h[0], h[1], h[2], h[3]);
        const __half2 sc = c < 4 ? sc0 : sc1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&h[j]), sc);
            v[4 * c + j] = *reinterpret_cast<const uint32_t *>(&r);
        }
    }
}

// Epilogue warps (quadrant = warp % 4, chunk half = warp / 4): per item,
// wait for the accumulator, read it (tcgen05.ld), release it, and write
// phase 1's activations (f16, stage_pos order) or phase 2's rows (f16).  The
// MMA issuer and this loop walk the same item sequence, so both keep the
// accumulator-half state (TcAccState) identically.
// NSUM > 1 (the block-scaled kernel's single-CTA form): the accumulator of a
// tile holds NSUM column groups SUM_STRIDE apart, one per token term, and a
// token's value is their sum; ACC_STRIDE is the column offset of the second
// accumulator buffer.  With the defaults the layout is tc_ffn's.
template <int FMT, int PHASE, bool PAIR, int NSUM = 1, int SUM_STRIDE = 0,
          int ACC_STRIDE = TcCfg<PAIR>::ACC_HALF, int MAXN = TcCfg<PAIR>::NT, bool WIDE = false>
__device__ __forceinline__ void tc_epilogue(const TcArgs &p, const TcItemTab &tab, int unit,
                                            int nunits, int total, uint32_t tmem, uint32_t rank,
                                            uint64_t *acc_full, uint64_t *acc_empty, int warp,
                                            int lane) {
    using C = TcCfg<PAIR, WIDE>;
    const int q = warp & 3, whalf = warp >> 2;
    constexpr int CH_STEP = 32 * (C::EPI_WARPS / 4);
    const float ia = 1.f / p.act_a, ib = 1.f / p.act_b; // SiTU's divisions, once
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    TcAccState acc;
    bool ok = true;
    for (int i = unit; ok && i < total; i += nunits) {
        TcItem it;
        tc_item<PHASE, PAIR, WIDE>(p, tab, i, it);
        const int b = acc.take(NSUM == 1 && it.nmma > C::ACC_HALF);
        bool got = true;
        if (b != 1)
            got = mbar_wait(&acc_full[0], acc.use[0] & 1u, p.err);
        if (got && b != 0)
            got = mbar_wait(&acc_full[1], acc.use[1] & 1u, p.err);
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const int orow = __ldg(p.orow + it.e) + it.t0;
        const uint32_t accb = tmem + lane_addr + (b == 1 ? static_cast<uint32_t>(ACC_STRIDE) : 0u);
        // The accumulator is released as soon as it has been read, so the
        // next tile's MMAs need not wait for the global stores: phase 1
        // keeps every chunk's activations in registers (two tokens per
        // word) and stores them after the release; phase 2 stores the rows
        // of all chunks but the last as they are read, and the last after
        // the release.
        constexpr int MAXCH = (MAXN + CH_STEP - 1) / CH_STEP;
        uint32_t hpk[PHASE == 1 ? MAXCH * 8 : 1];
        uint32_t v[32];
        int nch = 0;
        const bool gate = lane < 16;
#pragma unroll
        for (int j = 0; j < MAXCH; ++j) {
            const int ch = 32 * whalf + j * CH_STEP;
            if (ch >= it.n)
                break;
            tc_ld32(accb + ch, v);
            if (NSUM > 1) {
                uint32_t w[32];
#pragma unroll
                for (int t = 1; t < NSUM; ++t) {
                    tc_ld32(accb + ch + t * SUM_STRIDE, w);
                    tc_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        v[k] = __float_as_uint(__uint_as_float(v[k]) + __uint_as_float(w[k]));
                }
            }
            tc_wait_ld();
            ++nch;
            if (PHASE == 1) {
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const float mine_lo = __uint_as_float(v[t]);
                    const float mine_hi = __uint_as_float(v[16 + t]);
                    const float other =
                        __shfl_xor_sync(0xffffffffu, gate ? mine_hi : mine_lo, 16);
                    const float g = gate ? mine_lo : other;
                    const float u = gate ? other : mine_hi;
                    const float hv = apply_act_fast(g, u, p.act, p.act_a, p.act_b, ia, ib);
                    if (beyond_f16(hv))
                        set_error(p.err, MVLLM_ERR_ACT_RANGE);
                    const uint32_t hb = __half_as_ushort(__float2half_rn(hv));
                    if (t & 1)
                        hpk[j * 8 + (t >> 1)] |= hb << 16;
                    else
                        hpk[j * 8 + (t >> 1)] = hb;
                }
            } else if (ch + CH_STEP < it.n) {
                __half *yp = static_cast<__half *>(p.out); // f16 rows of y
                const int col = it.c0 + static_cast<int>(rank) * 128 + 32 * q + lane;
                bool big = false;
#pragma unroll
                for (int t = 0; t < 32; ++t)
                    if (ch + t < it.n) {
                        const float yv = __uint_as_float(v[t]);
                        big |= beyond_f16(yv);
                        yp[static_cast<size_t>(orow + ch + t) * p.O + col] = __float2half_rn(yv);
                    }
                if (big)
                    set_error(p.err, MVLLM_ERR_ACT_RANGE);
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            for (int h = 0; h < 2; ++h) {
                if (b == 1 - h)
                    continue;
                if (PAIR)
                    mbar_arrive_cluster(cluster_addr(&acc_empty[h], 0));
                else
                    mbar_arrive(&acc_empty[h]);
            }
        }
        if (PHASE == 1) {
            const int col = it.c0 + static_cast<int>(rank) * 64 + 16 * q + (lane & 15);
            __half *hp = static_cast<__half *>(p.out);
#pragma unroll
            for (int j = 0; j < MAXCH; ++j) {
                if (j >= nch)
                    break;
                const int tb = 32 * whalf + j * CH_STEP + (gate ? 0 : 16);
#pragma unroll
                for (int t = 0; t < 16; ++t)
                    if (tb + t < it.n)
                        hp[static_cast<size_t>(orow + tb + t) * p.O + stage_pos(col, FMT)] =
                            __ushort_as_half(static_cast<unsigned short>(
                                hpk[j * 8 + (t >> 1)] >> (16 * (t & 1))));
            }
        } else if (nch > 0) {
            const int ch = 32 * whalf + (nch - 1) * CH_STEP;
            __half *yp = static_cast<__half *>(p.out);
            const int col = it.c0 + static_cast<int>(rank) * 128 + 32 * q + lane;
            bool big = false;
#pragma unroll
            for (int t = 0; t < 32; ++t)
                if (ch + t < it.n) {
                    const float yv = __uint_as_float(v[t]);
                    big |= beyond_f16(yv);
                    yp[static_cast<size_t>(orow + ch + t) * p.O + col] = __float2half_rn(yv);
                }
            if (big)
                set_error(p.err, MVLLM_ERR_ACT_RANGE);
        }
        if (b != 1)
            ++acc.use[0];
        if (b != 0)
            ++acc.use[1];
    }
}

template <int FMT, int PHASE, bool PAIR, bool WIDE = false>
__global__ void __launch_bounds__(TcCfg<PAIR, WIDE>::THREADS, TcCfg<PAIR, WIDE>::CTAS_PER_SM)
    tc_ffn_kernel(const TcArgs p, const __grid_constant__ CUtensorMap tok_map) {
    using C = TcCfg<PAIR, WIDE>;
    using L = TcLayout<PAIR, WIDE>;
    constexpr int S = C::STAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *full = bars, *empty = bars + S; // tokens + A stage
    uint64_t *pk_full = empty + S, *pk_empty = pk_full + C::PK_SLOTS;
    uint64_t *sc_full = pk_empty + C::PK_SLOTS, *sc_empty = sc_full + kTcScSlots;
    uint64_t *acc_full = sc_empty + kTcScSlots, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    int *off_s = reinterpret_cast<int *>(smem + L::OFF_ITEMS);
    int *cnt_s = off_s + L::ITEM_TAB;
    const bool tab_in_smem = p.nb + 1 <= L::ITEM_TAB;
    if (tab_in_smem) {
        for (int e = threadIdx.x; e <= p.nb; e += blockDim.x) {
            off_s[e] = __ldg(p.item_off + e);
            cnt_s[e] = e < p.nb ? __ldg(p.cnt + e) : 0;
        }
    }
    const TcItemTab tab{tab_in_smem ? off_s : p.item_off, tab_in_smem ? cnt_s : p.cnt};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // A pair's CTAs walk the pair's list together; rank 0 is the leader.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const int unit = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
    const int nunits = PAIR ? static_cast<int>(nclusters_x()) : static_cast<int>(gridDim.x);
    const int total = __ldg(p.item_off + p.nb);
    if (unit >= total)
        return; // no item (for a pair: both CTAs leave) -- before touching TMEM

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            // Producer's expect_tx (a pair's leader counts both CTAs' token
            // bytes) + the k-block's dequant warps (both CTAs' for a pair; the
            // other CTA's copy of this barrier is unused).
            mbar_init(&full[s], C::FULL_ARRIVALS);
            mbar_init(&empty[s], 1); // the (leader's) tcgen05.commit
        }
        for (int s = 0; s < C::PK_SLOTS; ++s) {
            mbar_init(&pk_full[s], 1);
            mbar_init(&pk_empty[s], C::DQ_WARPS);
        }
        for (int s = 0; s < kTcScSlots; ++s) {
            mbar_init(&sc_full[s], 1);
            mbar_init(&sc_empty[s], C::DQ_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], C::ACC_EMPTY_ARRIVALS);
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
        cluster_sync(); // barriers of both CTAs initialised, TMEM allocated
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    const int nk = p.K / kTcKb;

    if (warp == C::PROD_WARP) {
        // ---------------------------------------------------- token producer
        if (lane == 0) {
            const uint64_t pol_t = policy_evict_last();
            uint32_t st_it = 0;
            bool ok = true;
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR, WIDE>(p, tab, i, it);
                const int rows = PAIR ? it.nmma >> 1 : it.nmma; // this CTA's token rows
                const int xr = __ldg(p.xrow + it.e) + it.t0 + static_cast<int>(rank) * rows;
                const int nbox = (rows + kTcTokBox - 1) / kTcTokBox;
                for (int kb = 0; kb < nk; kb += 2) {
                    const uint32_t s = st_it % S, par = (st_it / S) & 1u;
                    if (!mbar_wait(&empty[s], par ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst = smem + s * L::TOK_STAGE;
                    if (PAIR) {
                        if (rank == 0)
                            mbar_arrive_expect_tx(&full[s], 2u * 2u * nbox * kTcTokBox * 128);
                        const uint32_t fb = cluster_addr(&full[s], 0);
                        for (int kk = 0; kk < 2; ++kk)
                            for (int j = 0; j < nbox; ++j)
                                tma_load_2d_pair(dst + kk * L::TOK_KB + j * kTcTokBox * 128,
                                                 &tok_map, (kb + kk) * kTcKb, xr + j * kTcTokBox,
                                                 fb, pol_t);
                    } else {
                        mbar_arrive_expect_tx(&full[s], 2u * nbox * kTcTokBox * 128);
                        for (int kk = 0; kk < 2; ++kk)
                            for (int j = 0; j < nbox; ++j)
                                tma_load_2d(dst + kk * L::TOK_KB + j * kTcTokBox * 128, &tok_map,
                                            (kb + kk) * kTcKb, xr + j * kTcTokBox, &full[s],
                                            pol_t);
                    }
                    ++st_it;
                }
            }
            if (!ok || load_volatile(p.err) != 0) {
                // A stage's full barrier also waits for dequant arrivals, which
                // do not come on an error path: give copies in flight time to
                // land before the CTA ends.
                const uint64_t t0 = globaltimer_ns();
                while (globaltimer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == C::PK_WARP) {
        // ------------------------------------------- packed-weight producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const bool fence_maps = __ldg(p.tmaps_dirty) != 0;
            uint32_t pk_it = 0, sc_it = 0;
            bool ok = true;
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR, WIDE>(p, tab, i, it);
                const uint8_t *tm = p.tmaps + static_cast<size_t>(it.e) * kTcMapCount * kTcMapBytes;
                if (fence_maps)
                    for (int m = 0; m < kTcMapCount; ++m)
                        tmap_acquire(tm + m * kTcMapBytes);
                // This CTA's 128 weight rows: 64 gate + 64 up, or 128 down.
                const int r0 = it.c0 + static_cast<int>(rank) * tc_cols_per_item<PHASE, false>();
                for (int kb = 0; kb < nk; kb += 2) {
                    if (kb % tc_kb_per_window<FMT>() == 0) {
                        // The rows' next scale window (16 bytes per row).
                        const uint32_t w = sc_it % kTcScSlots, wpar = (sc_it / kTcScSlots) & 1u;
                        if (!mbar_wait(&sc_empty[w], wpar ^ 1u, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&sc_full[w], L::SC_STAGE);
                        uint8_t *sdst = smem + L::OFF_SC + w * L::SC_STAGE;
                        const int xs = (kb / tc_kb_per_window<FMT>()) *
                                       (FMT == MVLLM_FMT_MXFP4 ? 16 : 4); // in map elements
                        if (PHASE == 1) {
                            tma_load_2d(sdst, tm + kTcGateS * kTcMapBytes, xs, r0, &sc_full[w],
                                        pol_w);
                            tma_load_2d(sdst + 1024, tm + kTcUpS * kTcMapBytes, xs, r0,
                                        &sc_full[w], pol_w);
                        } else {
                            tma_load_2d(sdst, tm + kTcDownS * kTcMapBytes, xs, r0, &sc_full[w],
                                        pol_w);
                        }
                        ++sc_it;
                    }
                    const uint32_t s = pk_it % C::PK_SLOTS, par = (pk_it / C::PK_SLOTS) & 1u;
                    if (!mbar_wait(&pk_empty[s], par ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&pk_full[s], L::PK_STAGE);
                    uint8_t *dst = smem + L::OFF_PK + s * L::PK_STAGE;
                    const int xb = kb * (kTcKb / 2); // byte column of the packed rows
                    if (PHASE == 1) {
                        tma_load_2d(dst, tm + kTcGateP * kTcMapBytes, xb, r0, &pk_full[s], pol_w);
                        tma_load_2d(dst + 4096, tm + kTcUpP * kTcMapBytes, xb, r0, &pk_full[s],
                                    pol_w);
                    } else {
                        tma_load_2d(dst, tm + kTcDownP * kTcMapBytes, xb, r0, &pk_full[s], pol_w);
                    }
                    ++pk_it;
                }
            }
            // Drain: wait for every copy still in flight before the CTA ends.
            for (uint32_t j = pk_it > C::PK_SLOTS ? pk_it - C::PK_SLOTS : 0; j < pk_it; ++j)
                mbar_wait(&pk_full[j % C::PK_SLOTS], (j / C::PK_SLOTS) & 1u, nullptr);
            for (uint32_t j = sc_it > kTcScSlots ? sc_it - kTcScSlots : 0; j < sc_it; ++j)
                mbar_wait(&sc_full[j % kTcScSlots], (j / kTcScSlots) & 1u, nullptr);
        }
    } else if (warp == C::MMA_WARP) {
        // ------------------------------------ MMA issuer (a pair's leader only)
        if (lane == 0 && rank == 0) {
            uint32_t st_it = 0;
            TcAccState acc;
            bool ok = true;
            const uint32_t tok_base = smem_u32(smem);
            for (int i = unit; ok && i < total; i += nunits) {
                TcItem it;
                tc_item<PHASE, PAIR, WIDE>(p, tab, i, it);
                const int b = acc.take(it.nmma > C::ACC_HALF);
                if (b != 1 && !mbar_wait(&acc_empty[0], (acc.use[0] & 1u) ^ 1u, p.err))
                    ok = false;
                if (ok && b != 0 && !mbar_wait(&acc_empty[1], (acc.use[1] & 1u) ^ 1u, p.err))
                    ok = false;
                if (!ok)
                    break;
                tc_fence_after();
                const uint32_t d = tmem + (b == 1 ? static_cast<uint32_t>(C::ACC_HALF) : 0u);
                const uint32_t idesc = tc_idesc(PAIR ? 256 : 128, it.nmma);
                for (int kb = 0; kb < nk; kb += 2) {
                    const uint32_t s = st_it % S;
                    if (!mbar_wait(&full[s], (st_it / S) & 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = tmem + C::A_BASE + s * L::A_COLS;
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint64_t bdesc =
                            tc_desc_sw128(tok_base + s * L::TOK_STAGE + kk * L::TOK_KB);
                        const uint32_t ak = a0 + kk * 32;
                        if (PAIR) {
                            tc_mma_pair(d, ak, bdesc, idesc, (kb | kk) != 0);
                            tc_mma_pair(d, ak + 8, bdesc + 2, idesc, 1u);
                            tc_mma_pair(d, ak + 16, bdesc + 4, idesc, 1u);
                            tc_mma_pair(d, ak + 24, bdesc + 6, idesc, 1u);
                        } else {
                            tc_mma_solo(d, ak, bdesc, idesc, (kb | kk) != 0);
                            tc_mma_solo(d, ak + 8, bdesc + 2, idesc, 1u);
                            tc_mma_solo(d, ak + 16, bdesc + 4, idesc, 1u);
                            tc_mma_solo(d, ak + 24, bdesc + 6, idesc, 1u);
                        }
                    }
                    if (PAIR) {
                        tc_commit_pair(cluster_addr(&empty[s], 0));
                        tc_commit_pair(cluster_addr(&empty[s], 1));
                    } else {
                        tc_commit_solo(&empty[s]);
                    }
                    ++st_it;
                }
                if (!ok)
                    break;
                for (int h = 0; h < 2; ++h) {
                    if (b == 1 - h)
                        continue; // the other half
                    if (PAIR) {
                        tc_commit_pair(cluster_addr(&acc_full[h], 0));
                        tc_commit_pair(cluster_addr(&acc_full[h], 1));
                    } else {
                        tc_commit_solo(&acc_full[h]);
                    }
                    ++acc.use[h];
                }
            }
            // Every MMA this thread issued has completed once `done` flips.
            if (PAIR)
                tc_commit_pair(cluster_addr(done, 0));
            else
                tc_commit_solo(done);
            mbar_wait(done, 0, nullptr);
        }
    } else if (warp >= C::DQ_WARP0 && warp < C::DQ_WARP0 + C::DQ_WARPS) {
        // -------------------------------------------------------------- dequant
        const int q = warp & 3, set = (warp - C::DQ_WARP0) >> 2;
        uint32_t pk_it = 0, sc_it = 0, st_it = 0;
        bool ok = true;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
        constexpr int KPW = tc_kb_per_window<FMT>();
        // This thread's weight row inside the CTA's 128: its packed-slot and
        // scale-slot offsets (phase 1: gate rows in lanes 0-15, up rows in
        // 16-31 of each quadrant; phase 2: one down row per lane).
        int pk_off, sc_off;
        if (PHASE == 1) {
            const int j = 16 * q + (lane & 15);
            pk_off = (lane < 16 ? 0 : 4096) + j * 64;
            sc_off = (lane < 16 ? 0 : 1024) + j * 16;
        } else {
            const int j = 32 * q + lane;
            pk_off = j * 64;
            sc_off = j * 16;
        }
        // SW64: 16-byte chunk c of box row j sits at chunk c ^ ((j >> 1) & 3).
        const uint32_t sw = static_cast<uint32_t>((((pk_off & 4095) >> 6) >> 1) & 3);
        uint4 win = make_uint4(0, 0, 0, 0);
        for (int i = unit; ok && i < total; i += nunits) {
            for (int sl = 0; sl < nk / 2 && ok; ++sl) {
                if ((2 * sl) % KPW == 0) {
                    // First slot of a scale window: this row's 16 bytes to registers.
                    const uint32_t w = sc_it % kTcScSlots;
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&sc_full[w], (sc_it / kTcScSlots) & 1u, p.err))) {
                        ok = false;
                        break;
                    }
                    win = lds128(smem_u32(smem + L::OFF_SC + w * L::SC_STAGE + sc_off));
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive(&sc_empty[w]);
                    ++sc_it;
                }
                const uint32_t ps = pk_it % C::PK_SLOTS;
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&pk_full[ps], (pk_it / C::PK_SLOTS) & 1u, p.err))) {
                    ok = false;
                    break;
                }
                const uint32_t pk_addr = smem_u32(smem + L::OFF_PK + ps * L::PK_STAGE + pk_off);
                // The slot's two k-blocks: one each for two sets, both for one.
                uint4 w0[2], w1[2];
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (C::DQ_SETS == 2 && jj != set)
                        continue;
                    w0[jj] = lds128(pk_addr + ((static_cast<uint32_t>(2 * jj) ^ sw) << 4));
                    w1[jj] = lds128(pk_addr + ((static_cast<uint32_t>(2 * jj + 1) ^ sw) << 4));
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&pk_empty[ps]); // the slot's bytes are in registers
                ++pk_it;
                // Convert and store this warp's k-blocks of the slot, then wait
                // for the stores once (the registers are free at issue).
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    if (C::DQ_SETS == 2 && jj != set)
                        continue;
                    const int kw = (2 * sl + jj) % KPW;
                    __half2 sc0, sc1;
                    if (FMT == MVLLM_FMT_MXFP4) {
                        const uint32_t word = sel4(win, kw >> 1);
                        const uint32_t e0 = (word >> (16 * (kw & 1))) & 0xFFu;
                        const uint32_t e1 = (word >> (16 * (kw & 1) + 8)) & 0xFFu;
                        if ((e0 > 140u && e0 != 255u) || (e1 > 140u && e1 != 255u))
                            flag_range(p);
                        sc0 = __float2half2_rn(ue8m0_to_f32(e0));
                        sc1 = __float2half2_rn(ue8m0_to_f32(e1));
                    } else {
                        sc0 = __float2half2_rn(__uint_as_float(sel4(win, kw)));
                        sc1 = sc0;
                    }
                    uint32_t v[32];
                    tc_dequant_row<FMT>(w0[jj], w1[jj], sc0, sc1, v);
                    // The slot's stage of the shared ring; k-block jj is its
                    // 32-column half.
                    const uint32_t s = st_it % S;
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&empty[s], ((st_it / S) & 1u) ^ 1u, p.err))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tc_st32(tmem + lane_addr + C::A_BASE + s * L::A_COLS + jj * 32, v);
                }
                if (!ok)
                    break;
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    const uint32_t s = st_it % S;
                    if (PAIR)
                        mbar_arrive_cluster(cluster_addr(&full[s], 0));
                    else
                        mbar_arrive(&full[s]);
                }
                ++st_it;
            }
        }
    } else if (warp < C::EPI_WARPS) {
        tc_epilogue<FMT, PHASE, PAIR, 1, 0, C::ACC_HALF, C::NT, WIDE>(
            p, tab, unit, nunits, total, tmem, rank, acc_full, acc_empty,
                                      warp, lane);
    }

    tc_fence_before();
    if (PAIR)
        cluster_sync(); // the pair's MMAs, copies and remote arrivals are all done
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
