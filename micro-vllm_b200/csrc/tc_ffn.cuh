// tc_ffn.cuh -- tensor-core expert FFN (tcgen05 + TMEM) for experts with many
// rows (prefill chunks, skewed routing).
//
// Same contract as the decode kernels (decode_ffn.cuh): phase 1 computes
//   h[r, j] = act(sum_k x[r,k] g[j,k], sum_k x[r,k] u[j,k])   (f16, stage_pos order)
// and phase 2 computes
//   y[r, n] = sum_j h[r,j] d[n,j]                             (f32)
// for the rows r of every expert the plan gave to this path
// (reference: moe_block's per-expert loop, metal_ops.cpp:466-509, through
// matmul_mxfp4 / matmul_int4_g64 in quant.cpp:104-123 / 61-102).
//
// The product is computed transposed, weights as the MMA's M side:
//   D[w, t] = sum_k W[w, k] * X[t, k]      M = 128 weight rows, N = tokens.
// - W (A operand) lives in tensor memory.  Dequant warps read the packed rows
//   (TMA box, 64-byte swizzle) and the group scales, convert e2m1 / int4 to
//   f16 with the scale folded in, and write them with tcgen05.st: no shared
//   memory round trip for the weights.
// - X (B operand) is a token tile in shared memory: TMA boxes of the staged f16
//   rows (128-byte swizzle, K-major), read by tcgen05.mma through a matrix
//   descriptor.  N is the expert's row count rounded up to 16, so an expert
//   with 20 rows pays for 32, not for a 128-row tile.
// - D accumulates in f32 in tensor memory, double buffered: the epilogue of
//   one item overlaps the MMAs of the next.
//
// Exactness of the folded scale: an MXFP4 weight is e2m1 * 2^(s-127).  As an
// f16 product it is exact for s in [104, 140] and for s = 0 (+0) and 255 (inf,
// as the reference decodes it).  Codes below 104 lose bits below 2^-24
// (absolute error under 2^-25 per weight).  Codes 141..254 would overflow:
// the dequant warps record MVLLM_ERR_RANGE and the host reruns the call on
// the decode path.  int4-g64 weights are (q-8) * scale rounded once to f16.
//
// Warp roles (448 threads, one CTA per SM, persistent over the item list):
//   warps 0-3   epilogue: TMEM -> registers -> activation -> global
//   warps 4-11  dequant: packed weights -> f16 -> TMEM (A operand)
//   warp 12     producer: TMA of packed weights and token tiles
//   warp 13     MMA issuer (one thread) and TMEM allocator
// A warp may only touch the TMEM lanes of its quadrant (warp id % 4), which
// is why epilogue and dequant warps come in groups of four.
#pragma once

#include "common.cuh"

namespace mvb {

constexpr int kTcThreads = 448;
constexpr int kTcEpiWarps = 4;
constexpr int kTcDqWarp0 = 4, kTcDqWarps = 8;
constexpr int kTcProdWarp = 12, kTcMmaWarp = 13;
constexpr int kTcKb = 64;         // k elements per k-block: one 128-byte swizzle atom of f16
constexpr int kTcTokBox = 64;     // token rows per TMA box
constexpr int kTcTmemCols = 512;  // whole TMEM of the SM
constexpr int kTcStages = 8;      // token ring depth (k-blocks)
constexpr int kTcPkSlots = 8;     // packed-weight ring depth (2 k-blocks per slot)
constexpr int kTcWt = 1;          // weight tiles (128 rows each) per item
enum { kTcGateP = 0, kTcUpP, kTcDownP, kTcMapCount };
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

template <int WT> struct TcLayout {
    static constexpr int NT = 128 / WT;                // token tile = largest MMA N
    static constexpr int TOK_STAGE = NT * 128;         // bytes of one k-block of tokens
    static constexpr int PK_STAGE = WT * 128 * 64;     // WT weight tiles x 128 rows x 64 B
    static constexpr int ACC_COLS = WT * NT;           // TMEM columns per accumulator buffer
    static constexpr int A_COLS = WT * 32;             // TMEM columns per A stage (64 f16)
    static constexpr int A_BASE = 2 * ACC_COLS;        // first A-stage column
    // One A stage of the columns is left unused so that every MMA operand
    // stays well inside the allocation.
    static constexpr int SA = (kTcTmemCols - A_BASE) / A_COLS - 1;
    static constexpr int OFF_PK = kTcStages * TOK_STAGE;
    static constexpr int OFF_BAR = OFF_PK + kTcPkSlots * PK_STAGE;
    static constexpr int NBARS = 2 * kTcStages + 2 * kTcPkSlots + 2 * SA + 4 + 1;
    static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16 + 1024; // + tmem slot + alignment
    static_assert(SA >= 2 && SA <= 16, "A ring");
};

// Rows of weights per item: phase 1 takes 64 h columns (64 gate + 64 up rows)
// per weight tile, phase 2 takes 128 down rows.
template <int PHASE> __host__ __device__ constexpr int tc_cols_per_tile() {
    return PHASE == 1 ? 64 : 128;
}

// ---- tcgen05 wrappers ---------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, f16 inputs, f32 accumulate.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
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
// K-major, N >> 3 at [17,23), M >> 4 at [24,29).
__device__ __forceinline__ uint32_t tc_idesc(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

// Word i (0..3) of v without a local-memory array.
__device__ __forceinline__ uint32_t sel4(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct TcItem {
    int e;     // expert
    int t0;    // first row of the token tile (relative to the expert)
    int n;     // real rows in the tile
    int nmma;  // MMA N: n rounded up to 16
    int c0;    // first output column of the item (h column or y column)
};

template <int PHASE, int WT>
__device__ __forceinline__ void tc_item(const TcArgs &p, int i, TcItem &it) {
    using L = TcLayout<WT>;
    const int e = find_owner(p.item_off, p.nb, i);
    const int local = i - __ldg(p.item_off + e);
    const int c = __ldg(p.cnt + e);
    const int ntt = (c + L::NT - 1) / L::NT;
    const int wg = local / ntt, tt = local - wg * ntt;
    it.e = e;
    it.t0 = tt * L::NT;
    it.n = min(L::NT, c - it.t0);
    it.nmma = (it.n + 15) & ~15;
    it.c0 = wg * WT * tc_cols_per_tile<PHASE>();
}

template <int FMT, int PHASE, int WT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_ffn_kernel(const TcArgs p, const __grid_constant__ CUtensorMap tok_map) {
    using L = TcLayout<WT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *tok_full = bars, *tok_empty = bars + kTcStages;
    uint64_t *pk_full = tok_empty + kTcStages, *pk_empty = pk_full + kTcPkSlots;
    uint64_t *a_full = pk_empty + kTcPkSlots, *a_empty = a_full + L::SA;
    uint64_t *acc_full = a_empty + L::SA, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = __ldg(p.item_off + p.nb);
    if (static_cast<int>(blockIdx.x) >= total)
        return; // no item for this CTA: leave before touching TMEM

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&tok_full[s], 1);
            mbar_init(&tok_empty[s], 1);
        }
        for (int s = 0; s < kTcPkSlots; ++s) {
            mbar_init(&pk_full[s], 1);
            mbar_init(&pk_empty[s], kTcDqWarps);
        }
        for (int s = 0; s < L::SA; ++s) {
            mbar_init(&a_full[s], WT == 1 ? 4 : 8);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kTcEpiWarps);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    const int nk = p.K / kTcKb;

    if (warp == kTcProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first(), pol_t = policy_evict_last();
            const bool fence_maps = __ldg(p.tmaps_dirty) != 0;
            uint32_t tok_it = 0, pk_it = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && i < total; i += gridDim.x) {
                TcItem it;
                tc_item<PHASE, WT>(p, i, it);
                const uint8_t *tm = p.tmaps + static_cast<size_t>(it.e) * kTcMapCount * kTcMapBytes;
                if (fence_maps)
                    for (int m = 0; m < kTcMapCount; ++m)
                        tmap_acquire(tm + m * kTcMapBytes);
                const int xr = __ldg(p.xrow + it.e) + it.t0;
                const int nbox = (it.nmma + kTcTokBox - 1) / kTcTokBox;
                for (int kb = 0; kb < nk && ok; ++kb) {
                    if ((kb & 1) == 0) {
                        const uint32_t s = pk_it % kTcPkSlots, par = (pk_it / kTcPkSlots) & 1u;
                        if (!mbar_wait(&pk_empty[s], par ^ 1u, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&pk_full[s], L::PK_STAGE);
                        uint8_t *dst = smem + L::OFF_PK + s * L::PK_STAGE;
                        const int xb = kb * (kTcKb / 2); // byte column of the packed rows
                        for (int wt = 0; wt < WT; ++wt) {
                            if (PHASE == 1) {
                                const int r = it.c0 + wt * 64;
                                tma_load_2d(dst + wt * 8192, tm + kTcGateP * kTcMapBytes, xb, r,
                                            &pk_full[s], pol_w);
                                tma_load_2d(dst + wt * 8192 + 4096, tm + kTcUpP * kTcMapBytes, xb,
                                            r, &pk_full[s], pol_w);
                            } else {
                                tma_load_2d(dst + wt * 8192, tm + kTcDownP * kTcMapBytes, xb,
                                            it.c0 + wt * 128, &pk_full[s], pol_w);
                            }
                        }
                        ++pk_it;
                    }
                    const uint32_t s = tok_it % kTcStages, par = (tok_it / kTcStages) & 1u;
                    if (!mbar_wait(&tok_empty[s], par ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&tok_full[s], nbox * kTcTokBox * 128);
                    uint8_t *dst = smem + s * L::TOK_STAGE;
                    for (int j = 0; j < nbox; ++j)
                        tma_load_2d(dst + j * kTcTokBox * 128, &tok_map, kb * kTcKb,
                                    xr + j * kTcTokBox, &tok_full[s], pol_t);
                    ++tok_it;
                }
            }
            // Drain: wait for every copy still in flight before the CTA ends.
            for (uint32_t j = tok_it > kTcStages ? tok_it - kTcStages : 0; j < tok_it; ++j)
                mbar_wait(&tok_full[j % kTcStages], (j / kTcStages) & 1u, nullptr);
            for (uint32_t j = pk_it > kTcPkSlots ? pk_it - kTcPkSlots : 0; j < pk_it; ++j)
                mbar_wait(&pk_full[j % kTcPkSlots], (j / kTcPkSlots) & 1u, nullptr);
        }
    } else if (warp == kTcMmaWarp) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t tok_it = 0, a_it = 0, li = 0;
            bool ok = true;
            const uint32_t tok_base = smem_u32(smem);
            for (int i = blockIdx.x; ok && i < total; i += gridDim.x, ++li) {
                TcItem it;
                tc_item<PHASE, WT>(p, i, it);
                const uint32_t buf = li & 1u;
                if (!mbar_wait(&acc_empty[buf], ((li >> 1) & 1u) ^ 1u, p.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + buf * L::ACC_COLS;
                const uint32_t idesc = tc_idesc(it.nmma);
                for (int kb = 0; kb < nk; ++kb) {
                    const uint32_t ts = tok_it % kTcStages, as = a_it % L::SA;
                    if (!mbar_wait(&tok_full[ts], (tok_it / kTcStages) & 1u, p.err) ||
                        !mbar_wait(&a_full[as], (a_it / L::SA) & 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = tc_desc_sw128(tok_base + ts * L::TOK_STAGE);
                    const uint32_t a0 = tmem + L::A_BASE + as * L::A_COLS;
#pragma unroll
                    for (int wt = 0; wt < WT; ++wt)
#pragma unroll
                        for (int k = 0; k < kTcKb / 16; ++k)
                            tc_mma_ts(d + wt * L::NT, a0 + wt * 32 + k * 8, bdesc + 2 * k, idesc,
                                      (kb | k) != 0);
                    tc_commit(&tok_empty[ts]);
                    tc_commit(&a_empty[as]);
                    ++tok_it;
                    ++a_it;
                }
                if (ok)
                    tc_commit(&acc_full[buf]);
            }
            // Every MMA this thread issued has completed once `done` flips.
            tc_commit(done);
            mbar_wait(done, 0, nullptr);
        }
    } else if (warp >= kTcDqWarp0) {
        // -------------------------------------------------------------- dequant
        const int q = warp & 3, set = (warp - kTcDqWarp0) >> 2;
        const int wt = WT == 2 ? set : 0;
        uint32_t pk_it = 0, a_it = 0;
        bool ok = true;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
        for (int i = blockIdx.x; ok && i < total; i += gridDim.x) {
            TcItem it;
            tc_item<PHASE, WT>(p, i, it);
            // The weight row this thread converts and its place in the packed slot.
            int row, pk_row_off;
            const void *const *stab;
            if (PHASE == 1) {
                const bool gate = lane < 16;
                const int j = 16 * q + (lane & 15);
                row = it.c0 + wt * 64 + j;
                pk_row_off = wt * 8192 + (gate ? 0 : 4096) + j * 64;
                stab = gate ? p.s0 : p.s1;
                // SW64: 16-byte chunk c of box row j sits at chunk c ^ ((j >> 1) & 3).
            } else {
                const int j = 32 * q + lane;
                row = it.c0 + wt * 128 + j;
                pk_row_off = wt * 8192 + j * 64;
                stab = p.s0;
            }
            const int jrow = (pk_row_off & 4095) >> 6; // row inside its box
            const uint32_t sw = static_cast<uint32_t>((jrow >> 1) & 3);
            // Scales of this row: 16-byte windows (8 k-blocks of ue8m0 pairs or
            // 4 k-blocks of f32), the next window fetched one window ahead.
            constexpr int KB_PER_WIN = FMT == MVLLM_FMT_MXFP4 ? 8 : 4;
            const size_t srow_bytes = FMT == MVLLM_FMT_MXFP4 ? size_t(p.K) / 32 : size_t(p.K) / 16;
            const uint8_t *srow = static_cast<const uint8_t *>(stab[it.e]) +
                                  static_cast<size_t>(row) * srow_bytes;
            const int nwin = nk / KB_PER_WIN;
            uint4 win = ldg_stream128(srow), nxt = nwin > 1 ? ldg_stream128(srow + 16) : win;
            int cur_w = 0;
            for (int sl = 0; sl < nk / 2 && ok; ++sl) {
                const uint32_t s = pk_it % kTcPkSlots;
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&pk_full[s], (pk_it / kTcPkSlots) & 1u, p.err))) {
                    ok = false;
                    break;
                }
                const uint32_t pk_addr = smem_u32(smem + L::OFF_PK + s * L::PK_STAGE + pk_row_off);
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const int kb = 2 * sl + jj;
                    const bool mine = WT == 2 || (jj == set);
                    if (mine) {
                        const uint4 w0 = lds128(pk_addr + ((static_cast<uint32_t>(2 * jj) ^ sw) << 4));
                        const uint4 w1 =
                            lds128(pk_addr + ((static_cast<uint32_t>(2 * jj + 1) ^ sw) << 4));
                        const int wi = kb / KB_PER_WIN;
                        if (wi != cur_w) {
                            win = nxt;
                            cur_w = wi;
                            if (wi + 1 < nwin)
                                nxt = ldg_stream128(srow + 16 * (wi + 1));
                        }
                        const int kw = kb - wi * KB_PER_WIN;
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
                        const uint32_t pw[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                        uint32_t v[32];
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            uint32_t h0, h1, h2, h3;
                            if (FMT == MVLLM_FMT_MXFP4)
                                e2m1x8_to_f16x8(pw[c], h0, h1, h2, h3);
                            else
                                int4x8_to_f16x8(pw[c], h0, h1, h2, h3);
                            const __half2 sc = c < 4 ? sc0 : sc1;
                            const __half2 r0 = __hmul2(*reinterpret_cast<__half2 *>(&h0), sc);
                            const __half2 r1 = __hmul2(*reinterpret_cast<__half2 *>(&h1), sc);
                            const __half2 r2 = __hmul2(*reinterpret_cast<__half2 *>(&h2), sc);
                            const __half2 r3 = __hmul2(*reinterpret_cast<__half2 *>(&h3), sc);
                            v[4 * c + 0] = *reinterpret_cast<const uint32_t *>(&r0);
                            v[4 * c + 1] = *reinterpret_cast<const uint32_t *>(&r1);
                            v[4 * c + 2] = *reinterpret_cast<const uint32_t *>(&r2);
                            v[4 * c + 3] = *reinterpret_cast<const uint32_t *>(&r3);
                        }
                        const uint32_t as = a_it % L::SA;
                        if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[as],
                                                               ((a_it / L::SA) & 1u) ^ 1u, p.err))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        tc_st32(tmem + lane_addr + L::A_BASE + as * L::A_COLS + wt * 32, v);
                        tc_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0)
                            mbar_arrive(&a_full[as]);
                    }
                    ++a_it;
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&pk_empty[s]);
                ++pk_it;
            }
        }
    } else {
        // ------------------------------------------------------------- epilogue
        const int q = warp; // quadrant
        const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
        uint32_t li = 0;
        bool ok = true;
        for (int i = blockIdx.x; ok && i < total; i += gridDim.x, ++li) {
            TcItem it;
            tc_item<PHASE, WT>(p, i, it);
            const uint32_t buf = li & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (li >> 1) & 1u, p.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int orow = __ldg(p.orow + it.e) + it.t0;
#pragma unroll 1
            for (int wt = 0; wt < WT; ++wt) {
                const uint32_t acc = tmem + lane_addr + buf * L::ACC_COLS + wt * L::NT;
#pragma unroll 1
                for (int ch = 0; ch < it.n; ch += 32) {
                    uint32_t v[32];
                    tc_ld32(acc + ch, v);
                    tc_wait_ld();
                    if (PHASE == 1) {
                        const bool gate = lane < 16;
                        const int col = it.c0 + wt * 64 + 16 * q + (lane & 15);
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
                        const int col = it.c0 + wt * 128 + 32 * q + lane;
#pragma unroll
                        for (int t = 0; t < 32; ++t)
                            if (ch + t < it.n)
                                yp[static_cast<size_t>(orow + ch + t) * p.O + col] =
                                    __uint_as_float(v[t]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&acc_empty[buf]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTcTmemCols)
                     : "memory");
    }
}

} // namespace mvb
