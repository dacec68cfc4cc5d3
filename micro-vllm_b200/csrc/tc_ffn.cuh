// tc_ffn.cuh -- tensor-core expert FFN (tcgen05 + TMEM, CTA pairs) for experts
// with many rows (prefill chunks, skewed routing).
//
// Same contract as the decode kernels (decode_ffn.cuh): phase 1 computes
//   h[r, j] = act(sum_k x[r,k] g[j,k], sum_k x[r,k] u[j,k])   (f16, stage_pos order)
// and phase 2 computes
//   y[r, n] = sum_j h[r,j] d[n,j]                             (f32)
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
// the dequant warps record MVLLM_ERR_RANGE and the host reruns the call on
// the decode path.  int4-g64 weights are (q-8) * scale rounded once to f16.
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

constexpr int kTcEpiWarps = 8;             // warps 0-7: quadrant = warp % 4, column half = warp / 4
constexpr int kTcDqWarp0 = 8, kTcDqWarps = 8; // warps 8-15: quadrant = warp % 4, k-block parity set
constexpr int kTcProdWarp = 16, kTcMmaWarp = 17, kTcPkWarp = 18;
constexpr int kTcThreads = 19 * 32;
constexpr int kTcKb = 64;         // k elements per k-block: one 128-byte swizzle atom of f16
constexpr int kTcTokBox = 64;     // token rows per TMA box
constexpr int kTcNT = 256;        // token tile of a pair: the largest MMA N
constexpr int kTcTmemCols = 512;  // whole TMEM of the SM
constexpr int kTcStages = 7;      // token half-tile + A operand ring (k-blocks)
constexpr int kTcPkSlots = 8;     // packed-weight ring depth (2 k-blocks per slot)
constexpr int kTcScSlots = 3;     // scale ring depth (one 16-byte window per row per slot)
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
    const int *item_off;      // [nb + 1] item prefix of this path
    int nb;
    int K, O;                 // reduction length, output width (I or D)
    void *out;                // phase 1: f16 h [rows, I]; phase 2: f32 y [rows, D]
    int act;
    float act_a, act_b;
    int *err;
};

// Per CTA: TMEM columns [0, 256) accumulators -- one 256-column buffer for a
// tile of more than 128 tokens, or two 128-column buffers that alternate
// between smaller tiles (the epilogue of one overlaps the MMAs of the next);
// then one 32-column A stage (128 weight rows x 64 f16) per ring stage.
struct TcLayout {
    static constexpr int TOK_STAGE = (kTcNT / 2) * 128; // this CTA's half tile, one k-block
    static constexpr int PK_STAGE = 128 * 64;           // 128 weight rows x 64 B (2 k-blocks)
    static constexpr int SC_STAGE = 128 * 16;           // 128 weight rows x one scale window
    static constexpr int A_BASE = 256;
    static constexpr int A_COLS = 32;
    static constexpr int OFF_PK = kTcStages * TOK_STAGE;
    static constexpr int OFF_SC = OFF_PK + kTcPkSlots * PK_STAGE;
    static constexpr int OFF_BAR = OFF_SC + kTcScSlots * SC_STAGE;
    static constexpr int NBARS = 2 * kTcStages + 2 * kTcPkSlots + 2 * kTcScSlots + 4 + 1;
    static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16 + 1024; // + tmem slot + alignment
    static_assert(A_BASE + kTcStages * A_COLS <= kTcTmemCols, "TMEM budget");
    static_assert(SMEM <= 232448, "dynamic shared memory of one CTA");
};

// Weight rows per item of a pair: phase 1 takes 128 h columns (128 gate + 128
// up rows), phase 2 takes 256 down rows; each CTA holds half.
template <int PHASE> __host__ __device__ constexpr int tc_cols_per_item() {
    return PHASE == 1 ? 128 : 256;
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
// K-major, N >> 3 at [17,23), M >> 4 at [24,29); M = 256 over the pair.
__device__ __forceinline__ uint32_t tc_idesc(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
}

// Word i (0..3) of v without a local-memory array.
__device__ __forceinline__ uint32_t sel4(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct TcItem {
    int e;     // expert
    int t0;    // first row of the pair's token tile (relative to the expert)
    int n;     // real rows in the pair's tile
    int nmma;  // MMA N: n rounded up to 32
    int c0;    // first output column of the pair's item (h column or y column)
};

// Item i of the path: experts in plan order; inside an expert the weight tile
// varies slowest and the token tile fastest, so pairs working at the same
// time share the weight rows through L2.
template <int PHASE>
__device__ __forceinline__ void tc_item(const TcArgs &p, int i, TcItem &it) {
    const int e = find_owner(p.item_off, p.nb, i);
    const int local = i - __ldg(p.item_off + e);
    const int c = __ldg(p.cnt + e);
    const int ntt = (c + kTcNT - 1) / kTcNT;
    const int wg = local / ntt, tt = local - wg * ntt;
    it.e = e;
    it.t0 = tt * kTcNT;
    it.n = min(kTcNT, c - it.t0);
    it.nmma = (it.n + 31) & ~31;
    it.c0 = wg * tc_cols_per_item<PHASE>();
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

template <int FMT, int PHASE>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_ffn_kernel(const TcArgs p, const __grid_constant__ CUtensorMap tok_map) {
    using L = TcLayout;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *full = bars, *empty = bars + kTcStages;              // tokens + A stage
    uint64_t *pk_full = empty + kTcStages, *pk_empty = pk_full + kTcPkSlots;
    uint64_t *sc_full = pk_empty + kTcPkSlots, *sc_empty = sc_full + kTcScSlots;
    uint64_t *acc_full = sc_empty + kTcScSlots, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();           // 0 = leader of the pair
    const int pair = static_cast<int>(cluster_id_x()), npairs = static_cast<int>(nclusters_x());
    const int total = __ldg(p.item_off + p.nb);
    if (pair >= total)
        return; // no item for this pair (both CTAs leave): before touching TMEM

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            // Leader: its producer's expect_tx (both halves' bytes) + the
            // k-block's 4 dequant warps of each CTA.  The other CTA's copy of
            // this barrier is unused.
            mbar_init(&full[s], 1 + 8);
            mbar_init(&empty[s], 1); // the leader's tcgen05.commit
        }
        for (int s = 0; s < kTcPkSlots; ++s) {
            mbar_init(&pk_full[s], 1);
            mbar_init(&pk_empty[s], kTcDqWarps);
        }
        for (int s = 0; s < kTcScSlots; ++s) {
            mbar_init(&sc_full[s], 1);
            mbar_init(&sc_empty[s], kTcDqWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);                   // the leader's tcgen05.commit
            mbar_init(&acc_empty[b], 2 * kTcEpiWarps);    // leader: both CTAs' epilogue warps
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync(); // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    const int nk = p.K / kTcKb;

    if (warp == kTcProdWarp) {
        // ---------------------------------------------------- token producer
        if (lane == 0) {
            const uint64_t pol_t = policy_evict_last();
            uint32_t st_it = 0;
            bool ok = true;
            for (int i = pair; ok && i < total; i += npairs) {
                TcItem it;
                tc_item<PHASE>(p, i, it);
                const int half = it.nmma >> 1; // this CTA's token rows
                const int xr = __ldg(p.xrow + it.e) + it.t0 + static_cast<int>(rank) * half;
                const int nbox = (half + kTcTokBox - 1) / kTcTokBox;
                for (int kb = 0; kb < nk; ++kb) {
                    const uint32_t s = st_it % kTcStages, par = (st_it / kTcStages) & 1u;
                    if (!mbar_wait_cluster(&empty[s], par ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0)
                        mbar_arrive_expect_tx(&full[s], 2u * nbox * kTcTokBox * 128);
                    const uint32_t fb = cluster_addr(&full[s], 0);
                    uint8_t *dst = smem + s * L::TOK_STAGE;
                    for (int j = 0; j < nbox; ++j)
                        tma_load_2d_pair(dst + j * kTcTokBox * 128, &tok_map, kb * kTcKb,
                                         xr + j * kTcTokBox, fb, pol_t);
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
    } else if (warp == kTcPkWarp) {
        // ------------------------------------------- packed-weight producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const bool fence_maps = __ldg(p.tmaps_dirty) != 0;
            uint32_t pk_it = 0, sc_it = 0;
            bool ok = true;
            for (int i = pair; ok && i < total; i += npairs) {
                TcItem it;
                tc_item<PHASE>(p, i, it);
                const uint8_t *tm = p.tmaps + static_cast<size_t>(it.e) * kTcMapCount * kTcMapBytes;
                if (fence_maps)
                    for (int m = 0; m < kTcMapCount; ++m)
                        tmap_acquire(tm + m * kTcMapBytes);
                // This CTA's 128 weight rows: 64 gate + 64 up, or 128 down.
                const int r0 = it.c0 + static_cast<int>(rank) * (tc_cols_per_item<PHASE>() / 2);
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
                    const uint32_t s = pk_it % kTcPkSlots, par = (pk_it / kTcPkSlots) & 1u;
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
            for (uint32_t j = pk_it > kTcPkSlots ? pk_it - kTcPkSlots : 0; j < pk_it; ++j)
                mbar_wait(&pk_full[j % kTcPkSlots], (j / kTcPkSlots) & 1u, nullptr);
            for (uint32_t j = sc_it > kTcScSlots ? sc_it - kTcScSlots : 0; j < sc_it; ++j)
                mbar_wait(&sc_full[j % kTcScSlots], (j / kTcScSlots) & 1u, nullptr);
        }
    } else if (warp == kTcMmaWarp) {
        // ------------------------------------------- MMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            uint32_t st_it = 0;
            TcAccState acc;
            bool ok = true;
            const uint32_t tok_base = smem_u32(smem);
            for (int i = pair; ok && i < total; i += npairs) {
                TcItem it;
                tc_item<PHASE>(p, i, it);
                const int b = acc.take(it.nmma > 128);
                if (b != 1 && !mbar_wait_cluster(&acc_empty[0], (acc.use[0] & 1u) ^ 1u, p.err))
                    ok = false;
                if (ok && b != 0 &&
                    !mbar_wait_cluster(&acc_empty[1], (acc.use[1] & 1u) ^ 1u, p.err))
                    ok = false;
                if (!ok)
                    break;
                tc_fence_after();
                const uint32_t d = tmem + (b == 1 ? 128u : 0u);
                const uint32_t idesc = tc_idesc(it.nmma);
                for (int kb = 0; kb < nk; ++kb) {
                    const uint32_t s = st_it % kTcStages;
                    if (!mbar_wait_cluster(&full[s], (st_it / kTcStages) & 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = tc_desc_sw128(tok_base + s * L::TOK_STAGE);
                    const uint32_t a0 = tmem + L::A_BASE + s * L::A_COLS;
                    tc_mma_pair(d, a0, bdesc, idesc, kb != 0);
                    tc_mma_pair(d, a0 + 8, bdesc + 2, idesc, 1u);
                    tc_mma_pair(d, a0 + 16, bdesc + 4, idesc, 1u);
                    tc_mma_pair(d, a0 + 24, bdesc + 6, idesc, 1u);
                    tc_commit_pair(cluster_addr(&empty[s], 0));
                    tc_commit_pair(cluster_addr(&empty[s], 1));
                    ++st_it;
                }
                if (!ok)
                    break;
                for (int h = 0; h < 2; ++h) {
                    if (b == 1 - h)
                        continue; // the other half
                    tc_commit_pair(cluster_addr(&acc_full[h], 0));
                    tc_commit_pair(cluster_addr(&acc_full[h], 1));
                    ++acc.use[h];
                }
            }
            // Every MMA this thread issued has completed once `done` flips.
            tc_commit_pair(cluster_addr(done, 0));
            mbar_wait(done, 0, nullptr);
        }
    } else if (warp >= kTcDqWarp0 && warp < kTcDqWarp0 + kTcDqWarps) {
        // -------------------------------------------------------------- dequant
        const int q = warp & 3, set = (warp - kTcDqWarp0) >> 2;
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
        for (int i = pair; ok && i < total; i += npairs) {
            for (int sl = 0; sl < nk / 2 && ok; ++sl) {
                const int kb = 2 * sl + set;
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
                const uint32_t ps = pk_it % kTcPkSlots;
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&pk_full[ps], (pk_it / kTcPkSlots) & 1u, p.err))) {
                    ok = false;
                    break;
                }
                const uint32_t pk_addr = smem_u32(smem + L::OFF_PK + ps * L::PK_STAGE + pk_off);
                const uint4 w0 = lds128(pk_addr + ((static_cast<uint32_t>(2 * set) ^ sw) << 4));
                const uint4 w1 = lds128(pk_addr + ((static_cast<uint32_t>(2 * set + 1) ^ sw) << 4));
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&pk_empty[ps]); // the slot's bytes are in registers
                ++pk_it;
                const int kw = kb % KPW;
                __half2 sc0, sc1;
                if (FMT == MVLLM_FMT_MXFP4) {
                    const uint32_t word = sel4(win, kw >> 1);
                    const uint32_t e0 = (word >> (16 * (kw & 1))) & 0xFFu;
                    const uint32_t e1 = (word >> (16 * (kw & 1) + 8)) & 0xFFu;
                    if ((e0 > 140u && e0 != 255u) || (e1 > 140u && e1 != 255u))
                        set_error(p.err, MVLLM_ERR_RANGE);
                    sc0 = __float2half2_rn(ue8m0_to_f32(e0));
                    sc1 = __float2half2_rn(ue8m0_to_f32(e1));
                } else {
                    sc0 = __float2half2_rn(__uint_as_float(sel4(win, kw)));
                    sc1 = sc0;
                }
                uint32_t v[32];
                tc_dequant_row<FMT>(w0, w1, sc0, sc1, v);
                // This set's k-block is stage st_it + set of the shared ring.
                const uint32_t sidx = st_it + static_cast<uint32_t>(set);
                const uint32_t s = sidx % kTcStages;
                if (!__all_sync(0xffffffffu, mbar_wait_cluster(&empty[s],
                                                               ((sidx / kTcStages) & 1u) ^ 1u,
                                                               p.err))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tc_st32(tmem + lane_addr + L::A_BASE + s * L::A_COLS, v);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive_cluster(cluster_addr(&full[s], 0));
                st_it += 2;
            }
        }
    } else if (warp < kTcEpiWarps) {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3, whalf = warp >> 2;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
        TcAccState acc;
        bool ok = true;
        for (int i = pair; ok && i < total; i += npairs) {
            TcItem it;
            tc_item<PHASE>(p, i, it);
            const int b = acc.take(it.nmma > 128);
            bool got = true;
            if (b != 1)
                got = mbar_wait_cluster(&acc_full[0], acc.use[0] & 1u, p.err);
            if (got && b != 0)
                got = mbar_wait_cluster(&acc_full[1], acc.use[1] & 1u, p.err);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int orow = __ldg(p.orow + it.e) + it.t0;
            const uint32_t accb = tmem + lane_addr + (b == 1 ? 128u : 0u);
#pragma unroll 1
            for (int ch = 32 * whalf; ch < it.n; ch += 64) {
                uint32_t v[32];
                tc_ld32(accb + ch, v);
                tc_wait_ld();
                if (PHASE == 1) {
                    const bool gate = lane < 16;
                    const int col = it.c0 + static_cast<int>(rank) * 64 + 16 * q + (lane & 15);
                    const int tb = ch + (gate ? 0 : 16);
                    __half *hp = static_cast<__half *>(p.out);
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const float mine_lo = __uint_as_float(v[t]);
                        const float mine_hi = __uint_as_float(v[16 + t]);
                        const float other =
                            __shfl_xor_sync(0xffffffffu, gate ? mine_hi : mine_lo, 16);
                        const float g = gate ? mine_lo : other;
                        const float u = gate ? other : mine_hi;
                        if (tb + t < it.n)
                            hp[static_cast<size_t>(orow + tb + t) * p.O + stage_pos(col, FMT)] =
                                __float2half_rn(apply_act(g, u, p.act, p.act_a, p.act_b));
                    }
                } else {
                    float *yp = static_cast<float *>(p.out);
                    const int col = it.c0 + static_cast<int>(rank) * 128 + 32 * q + lane;
#pragma unroll
                    for (int t = 0; t < 32; ++t)
                        if (ch + t < it.n)
                            yp[static_cast<size_t>(orow + ch + t) * p.O + col] =
                                __uint_as_float(v[t]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (b != 1)
                    mbar_arrive_cluster(cluster_addr(&acc_empty[0], 0));
                if (b != 0)
                    mbar_arrive_cluster(cluster_addr(&acc_empty[1], 0));
            }
            if (b != 1)
                ++acc.use[0];
            if (b != 0)
                ++acc.use[1];
        }
    }

    tc_fence_before();
    cluster_sync(); // the pair's MMAs, copies and remote arrivals are all done
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTcTmemCols)
                     : "memory");
    }
}

} // namespace mvb
