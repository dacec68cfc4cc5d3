// mvllm_moe.cu -- host side of the sm_100a MoE block: the C ABI of
// include/mvllm_moe.h, the device-resident expert cache, and the launch
// sequence plan -> operand staging -> expert phase 1 -> phase 2 -> ordered
// combine.  No CPU fallback: every entry either runs the CUDA path or
// returns an error code.
#include "aux_kernels.cuh"
#include "decode_ffn.cuh"
#include "tc_ffn.cuh"
#include "tc_mx.cuh"
#include "ep_kernels.cuh"
#include "route_kernels.cuh"
#include "dense_ffn.cuh"
#include "epilogue.cuh"
#include "expert_tier.hpp"

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

using namespace mvb;

namespace {

// ------------------------------------------------------------------ context --
struct CacheEntry {
    void *dev = nullptr;
    size_t bytes = 0;
    uint64_t generation = 0;
};

struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
};

struct Context {
    std::mutex mu;
    bool inited = false;
    int device = -1;
    int sms = 0;
    int sm_limit = 0; // SMs the persistent expert kernels may fill (0: all)
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[4] = {};
    DevBuf ws;        // workspace of the host-pointer entries
    DevBuf transient; // per-call copies of unregistered weight arrays
    void *pinned = nullptr;
    size_t pinned_bytes = 0;
    std::map<uintptr_t, CacheEntry> cache; // host start -> device copy
    size_t cache_bytes = 0;
    // Device expert tier: bound host blobs, streamed into equal VRAM slots.
    TierPolicy tier;
    void *tier_arena = nullptr;
    std::map<uintptr_t, size_t> host_reg; // caller buffers page-locked by host_register
    cudaStream_t copy_stream = nullptr; // stream-ins of cold blobs, caller rows of layer_host
    cudaEvent_t copy_done = nullptr;
    cudaEvent_t call_start = nullptr, x_in = nullptr, out_in = nullptr; // caller-row copies
    cudaEvent_t x_head = nullptr; // moe_block: the head part of xg is on the device
    uint64_t calls = 0, experts = 0, rows = 0;
    double h2d_ms = 0, kernel_ms = 0, d2h_ms = 0;
};

Context &ctx() {
    static Context c;
    return c;
}

// SMs the layer's persistent kernels are sized for: all of them, or the
// limit a caller set to leave SMs to concurrent work (an NCCL exchange on
// another stream that should overlap the expert kernels).
int launch_sms(const Context &c) {
    return c.sm_limit > 0 ? std::max(2, std::min(c.sms, c.sm_limit)) : c.sms;
}

thread_local std::string g_last_error;

// ------------------------------------------------------------- profiling --
// Optional per-phase device timing of the device-pointer entries: a CUDA
// event is recorded on the launch stream after each phase; durations are the
// elapsed times between consecutive events of one call.
enum ProfPhase { kPhStart = -1, kPhPermute = 0, kPhGather, kPhPlan, kPhExpert1, kPhExpert2,
                 kPhCombine, kPhCount };
struct Prof {
    std::mutex mu;
    bool on = false;
    std::vector<cudaEvent_t> pool;
    std::vector<std::pair<cudaEvent_t, int>> marks;
    size_t used = 0;
};
Prof &prof() {
    static Prof p;
    return p;
}
void prof_mark(cudaStream_t st, int phase) {
    Prof &p = prof();
    if (!p.on)
        return;
    std::lock_guard<std::mutex> lk(p.mu);
    if (p.used == p.pool.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess)
            return;
        p.pool.push_back(e);
    }
    cudaEvent_t e = p.pool[p.used++];
    cudaEventRecord(e, st);
    p.marks.push_back({e, phase});
}

// A launch that may begin while the previous kernel on the stream finishes
// (programmatic dependent launch): the kernel waits in pdl_wait() before it
// reads that kernel's results, so only launch latency is overlapped.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess)                                                                  \
            return fail(MVLLM_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));        \
    } while (0)

int ensure_dev(DevBuf &b, size_t bytes) {
    if (b.bytes >= bytes)
        return MVLLM_OK;
    if (b.p)
        cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
    const size_t want = std::max(bytes, size_t(1) << 20);
    if (cudaMalloc(&b.p, want) != cudaSuccess) {
        cudaGetLastError();
        return fail(MVLLM_ERR_NOMEM, "cudaMalloc(%zu) failed", want);
    }
    b.bytes = want;
    return MVLLM_OK;
}

int ensure_pinned(Context &c, size_t bytes) {
    if (c.pinned_bytes >= bytes)
        return MVLLM_OK;
    if (c.pinned)
        cudaFreeHost(c.pinned);
    c.pinned = nullptr;
    c.pinned_bytes = 0;
    const size_t want = std::max(bytes, size_t(1) << 20);
    if (cudaMallocHost(&c.pinned, want) != cudaSuccess) {
        cudaGetLastError();
        return fail(MVLLM_ERR_NOMEM, "cudaMallocHost(%zu) failed", want);
    }
    c.pinned_bytes = want;
    return MVLLM_OK;
}

// Bump allocator over a caller- or context-owned workspace.
struct Carve {
    uint8_t *base;
    size_t cap, used = 0;
    bool overflow = false;
    Carve(void *b, size_t c) : base(static_cast<uint8_t *>(b)), cap(c) {}
    template <typename T> T *take(size_t n) {
        used = (used + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base ? base + used : nullptr);
        used += n * sizeof(T);
        if (used > cap)
            overflow = true;
        return p;
    }
};

// ------------------------------------------------------------ shapes / plan --
size_t row_bytes_packed(int fmt, int cols) {
    return fmt == MVLLM_FMT_F32 ? size_t(cols) * 4 : size_t((cols + 1) / 2);
}
size_t scale_row_bytes(int fmt, int cols) {
    if (fmt == MVLLM_FMT_INT4_G64)
        return size_t((cols + 63) / 64) * 4;
    if (fmt == MVLLM_FMT_MXFP4)
        return size_t((cols + 31) / 32);
    return 0;
}

bool fast_path_ok(int fmt, int D, int I) {
    if (fmt != MVLLM_FMT_INT4_G64 && fmt != MVLLM_FMT_MXFP4)
        return false;
    if (getenv("MVLLM_FORCE_GENERIC"))
        return false;
    return D >= 512 && I >= 512 && D % 512 == 0 && I % 512 == 0;
}

// Token tiles per item: 8 tokens, or 16 when experts average more than 8
// rows (prefill-like); experts with more rows are split into chunks, whose
// items run back to back so the repeated weight rows come from L2.
int chunk_tiles(int avg_rows) { return avg_rows > 8 ? 2 : 1; }
// Stage K-slice of the decode kernels (bytes of packed row per stage):
// 512 when the row divides, else 256; MVLLM_DECODE_KS=256 forces the smaller
// slice (twice the stages in the same shared memory).
int pick_ks(int K) {
    static const int forced = [] {
        const char *s = getenv("MVLLM_DECODE_KS");
        return s ? atoi(s) : 0;
    }();
    if (forced == 256 && (K / 2) % 256 == 0)
        return 256;
    return ((K / 2) % 512 == 0) ? 512 : 256;
}

struct RunWs {
    int *base, *cnt, *off1, *off2, *total_rows, *err;
    int *toff1, *toff2; // tensor-core path, CTA-pair item offsets [nb + 1]
    int *soff1, *soff2; // tensor-core path, single-CTA item offsets [nb + 1]
    int *woff1, *woff2; // tensor-core path, wide single-CTA item offsets [nb + 1]
    uint8_t *tc_tmaps;  // fast path: [nb][kTcMapCount] tensor maps
    int h_rows;         // rows of h and y
    int *tmaps_dirty; // set when build_tmaps_kernel rewrote a map this call
    uint8_t *tmaps;   // fast path: [nb][6] tensor maps
    void *xs; // staged operand (fast: f16, generic: f32)
    void *h;  // fast: f16 [rows, I]; generic: f32 [rows, I]
    float *y; // [rows, D]: f16 rows on the fast path (y16), f32 on the generic path
    bool y16;
    // Block-scaled tensor-core path (fast path only): per-expert weight maps,
    // and the token operands as block-scaled terms (planes + ue8m0 codes) of
    // x [x_rows, D] and h [h_rows, I], sized for the widest mode.
    uint8_t *mx_tmaps;
    uint8_t *xq, *xc, *hq, *hc;
    // Redo of the tensor-core experts on the decode kernels (fast path only):
    // their decode item offsets [nb + 1] per phase, and the word a
    // tensor-core kernel raises for scale codes it cannot represent.
    int *roff1, *roff2, *range;
};

// Carves the expert-run workspace; x_rows = operand rows to stage (0 when the
// operand is already staged by the caller of run_experts).
void carve_run(Carve &cv, RunWs &w, int nb, int D, int I, bool fast, int rows_cap, int x_rows) {
    w.base = cv.take<int>(nb);
    w.cnt = cv.take<int>(nb);
    w.off1 = cv.take<int>(nb + 1);
    w.off2 = cv.take<int>(nb + 1);
    w.total_rows = cv.take<int>(1);
    w.err = cv.take<int>(1);
    w.tmaps_dirty = cv.take<int>(1);
    w.tmaps = fast ? cv.take<uint8_t>(size_t(nb) * kTmapsPerExpert * 128) : nullptr;
    w.toff1 = cv.take<int>(nb + 1);
    w.toff2 = cv.take<int>(nb + 1);
    w.soff1 = cv.take<int>(nb + 1);
    w.soff2 = cv.take<int>(nb + 1);
    w.woff1 = cv.take<int>(nb + 1);
    w.woff2 = cv.take<int>(nb + 1);
    w.tc_tmaps = fast ? cv.take<uint8_t>(size_t(nb) * kTcMapCount * kTcMapBytes) : nullptr;
    w.h_rows = std::max(rows_cap, 1);
    const size_t esz = fast ? 2 : 4;
    w.xs = cv.take<uint8_t>(size_t(std::max(x_rows, 1)) * D * esz);
    w.h = cv.take<uint8_t>(size_t(std::max(rows_cap, 1)) * I * esz);
    w.y = cv.take<float>(size_t(std::max(rows_cap, 1)) * D);
    w.mx_tmaps = w.xq = w.xc = w.hq = w.hc = nullptr;
    w.roff1 = w.roff2 = w.range = nullptr;
    if (fast) {
        w.roff1 = cv.take<int>(nb + 1);
        w.roff2 = cv.take<int>(nb + 1);
        w.range = cv.take<int>(1);
        // Widest modes: two e4m3 terms (2 bytes per element) or three e2m1
        // terms (3 codes per 32 elements).
        const size_t xr = size_t(std::max(x_rows, 1)), hr = size_t(std::max(rows_cap, 1));
        w.mx_tmaps = cv.take<uint8_t>(size_t(nb) * kMxMapCount * kTcMapBytes);
        w.xq = cv.take<uint8_t>(xr * D * 2);
        w.xc = cv.take<uint8_t>(xr * (D / 32) * 3);
        w.hq = cv.take<uint8_t>(hr * I * 2);
        w.hc = cv.take<uint8_t>(hr * (I / 32) * 3);
    }
}

// ------------------------------------------------- prefill (tensor-core) mode --
// How experts on the tensor-core path compute with MXFP4 weights (header:
// MVLLM_PREFILL_*): dequantised to f16 (kind::f16), or block-scaled with the
// token operand as 1-3 e2m1 terms (kind::mxf4) or 1-2 e4m3 terms
// (kind::mxf8f6f4).  Set by mvllm_moe_set_prefill_mode or MVLLM_PREFILL_MODE
// (f16, mxf4x1, mxf4x2, mxf4x3, mxf8x1, mxf8x2).
std::atomic<int> g_prefill_mode{-1};
int prefill_mode() {
    int m = g_prefill_mode.load();
    if (m >= 0)
        return m;
    m = MVLLM_PREFILL_DEFAULT;
    if (const char *e = getenv("MVLLM_PREFILL_MODE")) {
        static const char *names[] = {"f16", "mxf4x1", "mxf4x2", "mxf4x3", "mxf8x1", "mxf8x2"};
        for (int i = 0; i < 6; ++i)
            if (!strcmp(e, names[i]))
                m = i;
    }
    return m;
}

// Exact mode: the layer epilogue and the router scores keep the reference's
// summation order and roundings (bit-identical results, serial sums); off,
// they run the tolerance-mode kernels.  Set by mvllm_moe_set_exact or
// MVLLM_EXACT=1.
std::atomic<int> g_exact{-1};
bool exact_mode() {
    int m = g_exact.load();
    if (m < 0) {
        const char *e = getenv("MVLLM_EXACT");
        m = (e && *e && strcmp(e, "0")) ? 1 : 0;
    }
    return m != 0;
}

struct Tables {
    const void *const *g, *const *u, *const *d, *const *gs, *const *us, *const *ds;
};

// ---------------------------------------------------------- tensor maps --
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 2-D map over a row-major [rows, inner] matrix; box = box_inner x box_rows.
int encode_2d(CUtensorMap *m, CUtensorMapDataType dt, void *addr, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
    auto enc = tmap_encoder();
    if (!enc)
        return fail(MVLLM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(m, dt, 2, addr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(MVLLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return MVLLM_OK;
}

// 3-D map over a row-major [rows, row_bytes] u8 matrix seen as (128-byte
// column chunk, row, chunk index): box = 128 B x box_rows x box_chunks, so one
// copy brings box_chunks chunks of box_rows rows laid out chunk-major.
int encode_3d_rows(CUtensorMap *m, void *addr, uint64_t row_bytes, uint64_t rows,
                   uint32_t box_rows, uint32_t box_chunks) {
    auto enc = tmap_encoder();
    if (!enc)
        return fail(MVLLM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
    const cuuint64_t strides[2] = {row_bytes, 128};
    const cuuint32_t box[3] = {128, box_rows, box_chunks};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, addr, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MVLLM_OK : MVLLM_ERR_UNSUPPORTED;
}

// Templates for one (fmt, D, I) shape: phase-1 boxes are 32 rows (gate and up
// halves of an item), phase-2 boxes 64 rows; weights use the 128-byte swizzle
// the decode consumers read through, scales are dense.
// With *box3d set on entry, the weight maps are first tried as 3-D maps (one
// copy per matrix per stage); *box3d says on return which form was encoded.
int make_templates(TmapTemplates *t, int fmt, int D, int I, int ks1, int ks2, void *placeholder,
                   int *box3d) {
    const bool mx = fmt == MVLLM_FMT_MXFP4;
    const auto u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8, f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B, none = CU_TENSOR_MAP_SWIZZLE_NONE;
    int rc = 0;
    if (*box3d) {
        const int r3 = encode_3d_rows(&t->m[0], placeholder, D / 2, I, 32, ks1 / 128) |
                       encode_3d_rows(&t->m[1], placeholder, D / 2, I, 32, ks1 / 128) |
                       encode_3d_rows(&t->m[2], placeholder, I / 2, D, 64, ks2 / 128);
        if (r3 != MVLLM_OK)
            *box3d = 0; // the driver refused the chunk-major view: 2-D boxes
    }
    if (!*box3d) {
        rc |= encode_2d(&t->m[0], u8, placeholder, D / 2, I, D / 2, 128, 32, sw);
        rc |= encode_2d(&t->m[1], u8, placeholder, D / 2, I, D / 2, 128, 32, sw);
        rc |= encode_2d(&t->m[2], u8, placeholder, I / 2, D, I / 2, 128, 64, sw);
    }
    const int sb1 = mx ? ks1 / 16 : ks1 / 8, sb2 = mx ? ks2 / 16 : ks2 / 8; // bytes per row
    if (mx) {
        rc |= encode_2d(&t->m[3], u8, placeholder, D / 32, I, D / 32, sb1, 32, none);
        rc |= encode_2d(&t->m[4], u8, placeholder, D / 32, I, D / 32, sb1, 32, none);
        rc |= encode_2d(&t->m[5], u8, placeholder, I / 32, D, I / 32, sb2, 64, none);
    } else {
        rc |= encode_2d(&t->m[3], f32, placeholder, D / 64, I, D / 16, sb1 / 4, 32, none);
        rc |= encode_2d(&t->m[4], f32, placeholder, D / 64, I, D / 16, sb1 / 4, 32, none);
        rc |= encode_2d(&t->m[5], f32, placeholder, I / 64, D, I / 16, sb2 / 4, 64, none);
    }
    return rc ? MVLLM_ERR_CUDA : MVLLM_OK;
}

// Templates of the tensor-core path: packed rows in boxes of 64 bytes (two
// k-blocks) by 64 gate / up rows or 128 down rows with the 64-byte swizzle,
// and the rows' scales in 16-byte windows (8 k-blocks of ue8m0 pairs or 4
// k-blocks of f32), unswizzled.
int make_tc_templates(TmapSet<kTcMapCount> *t, int fmt, int D, int I, void *placeholder) {
    const auto u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8, f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_64B, none = CU_TENSOR_MAP_SWIZZLE_NONE;
    int rc = 0;
    rc |= encode_2d(&t->m[kTcGateP], u8, placeholder, D / 2, I, D / 2, 64, 64, sw);
    rc |= encode_2d(&t->m[kTcUpP], u8, placeholder, D / 2, I, D / 2, 64, 64, sw);
    rc |= encode_2d(&t->m[kTcDownP], u8, placeholder, I / 2, D, I / 2, 64, 128, sw);
    if (fmt == MVLLM_FMT_MXFP4) {
        rc |= encode_2d(&t->m[kTcGateS], u8, placeholder, D / 32, I, D / 32, 16, 64, none);
        rc |= encode_2d(&t->m[kTcUpS], u8, placeholder, D / 32, I, D / 32, 16, 64, none);
        rc |= encode_2d(&t->m[kTcDownS], u8, placeholder, I / 32, D, I / 32, 16, 128, none);
    } else {
        rc |= encode_2d(&t->m[kTcGateS], f32, placeholder, D / 64, I, D / 16, 4, 64, none);
        rc |= encode_2d(&t->m[kTcUpS], f32, placeholder, D / 64, I, D / 16, 4, 64, none);
        rc |= encode_2d(&t->m[kTcDownS], f32, placeholder, I / 64, D, I / 16, 4, 128, none);
    }
    return rc ? MVLLM_ERR_CUDA : MVLLM_OK;
}

// Token tiles of the tensor-core path: f16 rows of `cols` elements, boxes of
// 64 elements (one 128-byte swizzle atom) by 64 rows.
int make_tok_map(CUtensorMap *m, const void *rows_ptr, int cols, int rows) {
    return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<void *>(rows_ptr),
                     uint64_t(cols), uint64_t(std::max(rows, 1)), uint64_t(cols) * 2, kTcKb,
                     kTcTokBox, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int FMT, int PHASE, bool PAIR, bool WIDE = false>
int launch_tc_t(const TcArgs &a, const CUtensorMap &tok, cudaStream_t st, int sms) {
    using L = TcLayout<PAIR, WIDE>;
    auto kern = tc_ffn_kernel<FMT, PHASE, PAIR, WIDE>;
    static bool attr = false;
    if (!attr) {
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM));
        attr = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(TcCfg<PAIR, WIDE>::THREADS);
    cfg.dynamicSmemBytes = L::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    if (PAIR) {
        // CTA pairs: clusters of 2 on the two SMs of a TPC, one pair per TPC.
        cfg.gridDim = dim3(std::max(2, sms & ~1));
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    } else {
        cfg.gridDim = dim3(sms * TcCfg<PAIR, WIDE>::CTAS_PER_SM);
    }
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, tok));
    return MVLLM_OK;
}

template <int PHASE>
int launch_tc(int fmt, const TcArgs &pair, const TcArgs &solo, const TcArgs *wide,
              const CUtensorMap &tok, cudaStream_t st, int sms) {
    int rc = fmt == MVLLM_FMT_MXFP4
                 ? launch_tc_t<MVLLM_FMT_MXFP4, PHASE, true>(pair, tok, st, sms)
                 : launch_tc_t<MVLLM_FMT_INT4_G64, PHASE, true>(pair, tok, st, sms);
    if (rc)
        return rc;
    if (wide) {
        rc = fmt == MVLLM_FMT_MXFP4
                 ? launch_tc_t<MVLLM_FMT_MXFP4, PHASE, false, true>(*wide, tok, st, sms)
                 : launch_tc_t<MVLLM_FMT_INT4_G64, PHASE, false, true>(*wide, tok, st, sms);
        if (rc)
            return rc;
    }
    return fmt == MVLLM_FMT_MXFP4 ? launch_tc_t<MVLLM_FMT_MXFP4, PHASE, false>(solo, tok, st, sms)
                                  : launch_tc_t<MVLLM_FMT_INT4_G64, PHASE, false>(solo, tok, st, sms);
}

// Weight maps of the block-scaled path: packed rows in boxes of 128 bytes of
// one stage (mxf4: 256 packed e2m1; mxf8f6f4: 128 e2m1 as 16U4_ALIGN16B,
// expanded to the padded form in shared memory) by 16 gate / up rows or 128
// down rows, 128-byte swizzle; the rows' code windows as in tc_ffn.
int make_mx_templates(TmapSet<kMxMapCount> *t, int kind, int D, int I, void *placeholder) {
    const auto u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const auto none = CU_TENSOR_MAP_SWIZZLE_NONE, sw = CU_TENSOR_MAP_SWIZZLE_128B;
    int rc = 0;
    if (kind == kMxF4) {
        rc |= encode_2d(&t->m[kMxGateP], u8, placeholder, D / 2, I, D / 2, 128, 16, sw);
        rc |= encode_2d(&t->m[kMxUpP], u8, placeholder, D / 2, I, D / 2, 128, 16, sw);
        rc |= encode_2d(&t->m[kMxDownP], u8, placeholder, I / 2, D, I / 2, 128, 128, sw);
    } else {
        const auto u4 = CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B;
        rc |= encode_2d(&t->m[kMxGateP], u4, placeholder, D, I, D / 2, 128, 16, sw);
        rc |= encode_2d(&t->m[kMxUpP], u4, placeholder, D, I, D / 2, 128, 16, sw);
        rc |= encode_2d(&t->m[kMxDownP], u4, placeholder, I, D, I / 2, 128, 128, sw);
    }
    rc |= encode_2d(&t->m[kMxGateS], u8, placeholder, D / 32, I, D / 32, 16, 64, none);
    rc |= encode_2d(&t->m[kMxUpS], u8, placeholder, D / 32, I, D / 32, 16, 64, none);
    rc |= encode_2d(&t->m[kMxDownS], u8, placeholder, I / 32, D, I / 32, 16, 128, none);
    return rc ? MVLLM_ERR_CUDA : MVLLM_OK;
}

// 3-D map over NTERM planes of `rows` rows of `row_bytes` bytes each (term
// planes or their code rows): box = box_inner bytes x 64 rows x 1 plane.
int encode_planes(CUtensorMap *m, void *addr, uint64_t row_bytes, uint64_t rows, int nterm,
                  uint32_t box_inner, CUtensorMapSwizzle swz) {
    auto enc = tmap_encoder();
    if (!enc)
        return fail(MVLLM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const cuuint64_t dims[3] = {row_bytes, std::max<uint64_t>(rows, 1), uint64_t(nterm)};
    const cuuint64_t strides[2] = {row_bytes, row_bytes * std::max<uint64_t>(rows, 1)};
    const cuuint32_t box[3] = {box_inner, uint32_t(kTcTokBox), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, addr, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(MVLLM_ERR_CUDA, "cuTensorMapEncodeTiled (term planes) failed (%d)", int(r));
    return MVLLM_OK;
}

int mode_kind(int mode) { return mode >= MVLLM_PREFILL_MXF8_X1 ? kMxF8 : kMxF4; }
int mode_nterm(int mode) {
    return mode >= MVLLM_PREFILL_MXF8_X1 ? mode - MVLLM_PREFILL_MXF8_X1 + 1 : mode;
}

// Term planes of f16 rows [rows, K] for the block-scaled path.
int launch_terms(int mode, const void *src, int rows, int K, uint8_t *planes, uint8_t *codes,
                 cudaStream_t st, int sms) {
    const long long threads = static_cast<long long>(rows) * (K / 8);
    const int blocks = static_cast<int>(std::max<long long>(
        1, std::min<long long>((threads + 255) / 256, 16LL * sms)));
    const __half *x = static_cast<const __half *>(src);
    switch (mode) {
    case MVLLM_PREFILL_MXF4_X1: mx_terms_kernel<kMxF4, 1><<<blocks, 256, 0, st>>>(x, rows, K, planes, codes); break;
    case MVLLM_PREFILL_MXF4_X2: mx_terms_kernel<kMxF4, 2><<<blocks, 256, 0, st>>>(x, rows, K, planes, codes); break;
    case MVLLM_PREFILL_MXF4_X3: mx_terms_kernel<kMxF4, 3><<<blocks, 256, 0, st>>>(x, rows, K, planes, codes); break;
    case MVLLM_PREFILL_MXF8_X1: mx_terms_kernel<kMxF8, 1><<<blocks, 256, 0, st>>>(x, rows, K, planes, codes); break;
    case MVLLM_PREFILL_MXF8_X2: mx_terms_kernel<kMxF8, 2><<<blocks, 256, 0, st>>>(x, rows, K, planes, codes); break;
    default: return fail(MVLLM_ERR_INVALID, "unknown prefill mode %d", mode);
    }
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

template <int KIND, int NTERM, int PHASE, bool PAIR>
int launch_mx_t(const MxArgs &a, const CUtensorMap &tok, const CUtensorMap &tsc, cudaStream_t st,
                int sms) {
    using C = MxCfg<KIND, NTERM, PAIR>;
    auto kern = tc_mx_kernel<KIND, NTERM, PHASE, PAIR>;
    static bool attr = false;
    if (!attr) {
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    if (PAIR) {
        cfg.gridDim = dim3(std::max(2, sms & ~1));
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    } else {
        cfg.gridDim = dim3(sms * C::CTAS_PER_SM);
    }
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, tok, tsc));
    return MVLLM_OK;
}

template <int KIND, int NTERM, int PHASE>
int launch_mx_pair_solo(const MxArgs &pair, const MxArgs &solo, const CUtensorMap &tok,
                        const CUtensorMap &tsc, cudaStream_t st, int sms) {
    if (int rc = launch_mx_t<KIND, NTERM, PHASE, true>(pair, tok, tsc, st, sms))
        return rc;
    return launch_mx_t<KIND, NTERM, PHASE, false>(solo, tok, tsc, st, sms);
}

template <int PHASE>
int launch_mx(int mode, const MxArgs &pair, const MxArgs &solo, const CUtensorMap &tok,
              const CUtensorMap &tsc, cudaStream_t st, int sms) {
    switch (mode) {
    case MVLLM_PREFILL_MXF4_X1: return launch_mx_pair_solo<kMxF4, 1, PHASE>(pair, solo, tok, tsc, st, sms);
    case MVLLM_PREFILL_MXF4_X2: return launch_mx_pair_solo<kMxF4, 2, PHASE>(pair, solo, tok, tsc, st, sms);
    case MVLLM_PREFILL_MXF4_X3: return launch_mx_pair_solo<kMxF4, 3, PHASE>(pair, solo, tok, tsc, st, sms);
    case MVLLM_PREFILL_MXF8_X1: return launch_mx_pair_solo<kMxF8, 1, PHASE>(pair, solo, tok, tsc, st, sms);
    case MVLLM_PREFILL_MXF8_X2: return launch_mx_pair_solo<kMxF8, 2, PHASE>(pair, solo, tok, tsc, st, sms);
    default: return fail(MVLLM_ERR_INVALID, "unknown prefill mode %d", mode);
    }
}

// Which experts take the tensor-core path: calls with at least
// MVLLM_TC_MIN_TOTAL routed rows (default 1024: prefill chunks, not decode
// batches) send their experts with at least MVLLM_TC_MIN_ROWS rows (default
// 17) there.  Returns 0 when the path is off for this call.
int tc_min_rows(int total_rows) {
    const char *t = getenv("MVLLM_TC_MIN_TOTAL");
    const char *r = getenv("MVLLM_TC_MIN_ROWS");
    const int min_total = t ? atoi(t) : 1024;
    const int min_rows = r ? atoi(r) : 17;
    if (getenv("MVLLM_TC_OFF") || total_rows < min_total || min_rows <= 0)
        return 0;
    return min_rows;
}

template <int FMT, int PHASE, int KS, int NT>
int launch_decode_t(DecodeArgs a, cudaStream_t st, int sms) {
    using L = DecodeLayout<FMT, KS, NT>;
    auto kern = decode_ffn_kernel<FMT, PHASE, KS, NT>;
    static int budget_kb = [] {
        const char *s = getenv("MVLLM_DECODE_SMEM_KB");
        return s ? atoi(s) : 226;
    }();
    static int ns = 0, smem = 0, per_sm = 0; // per instantiation, set once
    if (per_sm == 0) {
        ns = (budget_kb * 1024 - L::HEAD_BYTES - 128) / L::STAGE_BYTES;
        ns = std::max(2, std::min(8, ns));
        smem = L::smem_bytes(ns);
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        int occ = 0;
        CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kDecodeThreads, smem));
        per_sm = std::max(occ, 1);
    }
    a.nstages = ns;
    CUDA_TRY(launch_pdl(kern, dim3(sms * std::max(per_sm, 1)), dim3(kDecodeThreads), smem, st, a));
    return MVLLM_OK;
}

template <int FMT, int PHASE>
int launch_decode(const DecodeArgs &a, int ks, int nt, cudaStream_t st, int sms) {
    if (ks == 512)
        return nt == 1 ? launch_decode_t<FMT, PHASE, 512, 1>(a, st, sms)
                       : launch_decode_t<FMT, PHASE, 512, 2>(a, st, sms);
    return nt == 1 ? launch_decode_t<FMT, PHASE, 256, 1>(a, st, sms)
                   : launch_decode_t<FMT, PHASE, 256, 2>(a, st, sms);
}

// The expert plan of a run: PlanArgs plus what the launches after it need.
struct ExpertPlan {
    PlanArgs pa;
    bool fast, mx;
    int tc_min, mode, nt;
};

ExpertPlan make_expert_plan(int nb, int D, int I, int fmt, const Tables &tb, const int *nr,
                            const int *xoff, int x_rows, int avg_rows, const RunWs &w,
                            bool allow_tc) {
    ExpertPlan ep{};
    const bool fast = fast_path_ok(fmt, D, I);
    const int tc_min = (fast && allow_tc) ? tc_min_rows(x_rows) : 0;
    // Block-scaled MMAs for MXFP4 experts on the tensor-core path (the mode's
    // term planes need the workspace's term buffers).
    const int mode = (tc_min && fmt == MVLLM_FMT_MXFP4 && w.xq) ? prefill_mode()
                                                                  : MVLLM_PREFILL_F16;
    const bool mx = mode != MVLLM_PREFILL_F16;
    const int nt = chunk_tiles(avg_rows);
    const int mt = 8 * nt;
    PlanArgs pa{};
    pa.nb = nb;
    pa.fmt = fmt;
    pa.nr = nr;
    pa.g = tb.g, pa.u = tb.u, pa.d = tb.d, pa.gs = tb.gs, pa.us = tb.us, pa.ds = tb.ds;
    if (fast) {
        pa.chunk1 = mt, pa.blocks1 = I / 32;
        pa.chunk2 = mt, pa.blocks2 = D / 64;
    } else {
        pa.chunk1 = 1 << 30, pa.blocks1 = (I + 7) / 8;
        pa.chunk2 = 1 << 30, pa.blocks2 = (D + 7) / 8;
    }
    pa.base = w.base, pa.cnt = w.cnt, pa.off1 = w.off1, pa.off2 = w.off2;
    pa.total_rows = w.total_rows;
    pa.xoff = xoff, pa.x_rows = x_rows, pa.err = w.err;
    pa.align_mask = fast ? ((mx && mode_kind(mode) == kMxF8) ? 31 : 15) : 0;
    pa.tc_min = tc_min;
    // 256-row pair tiles, rests of at most kTcSoloMax rows on single CTAs.
    pa.tc_small = getenv("MVLLM_TC_NO_SOLO") ? 0 : kTcSoloMax;
    pa.tc_shift = 8;
    pa.tc_blocks1 = I / tc_cols_per_item<1, true>();
    pa.tc_blocks2 = D / tc_cols_per_item<2, true>();
    pa.tc_sblocks1 = I / tc_cols_per_item<1, false>();
    pa.tc_sblocks2 = D / tc_cols_per_item<2, false>();
    pa.toff1 = w.toff1, pa.toff2 = w.toff2, pa.soff1 = w.soff1, pa.soff2 = w.soff2;
    // Rests of 65..192 rows on wide single CTAs (f16 mode; the block-scaled
    // kernels have pairs and single CTAs only).
    pa.tc_wide = (mx || getenv("MVLLM_TC_NO_WIDE")) ? 0 : kTcWideMax;
    pa.woff1 = w.woff1, pa.woff2 = w.woff2;
    pa.clear_word = fast ? w.tmaps_dirty : nullptr;
    if (tc_min) {
        pa.roff1 = w.roff1, pa.roff2 = w.roff2, pa.range_word = w.range;
    }
    ep.pa = pa;
    ep.fast = fast, ep.mx = mx, ep.tc_min = tc_min, ep.mode = mode, ep.nt = nt;
    return ep;
}

// Decode tensor-map templates per shape, encoded once (the address is swapped
// in on the device, so the placeholder address does not matter).
int decode_templates(TmapTemplates *tpl, int fmt, int D, int I, void *placeholder, int *box3d) {
    struct Key {
        int fmt, D, I, want3d;
        bool operator<(const Key &o) const {
            return std::tie(fmt, D, I, want3d) < std::tie(o.fmt, o.D, o.I, o.want3d);
        }
    };
    struct Val {
        TmapTemplates t;
        int box3d;
    };
    static std::mutex mu;
    static std::map<Key, Val> cache;
    const Key k{fmt, D, I, *box3d};
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(k);
    if (it == cache.end()) {
        Val v{};
        v.box3d = *box3d;
        if (int rc = make_templates(&v.t, fmt, D, I, pick_ks(D), pick_ks(I), placeholder,
                                    &v.box3d))
            return rc;
        it = cache.emplace(k, v).first;
    }
    *tpl = it->second.t;
    *box3d = it->second.box3d;
    return MVLLM_OK;
}

// The expert FFN over nb experts: plan, optional operand staging, phase 1,
// phase 2.  Leaves y [rows, D] (reference base order) in w.y.  When
// `x_staged` is set, x already is the staged operand (f16 in stage_pos order
// on the fast path, f32 on the generic path) indexed by xoff.  With `pre`, the
// plan and the decode tensor maps were already written (layer_prep_small_kernel
// and stage_maps_kernel) from that same plan.
int run_experts(cudaStream_t st, int sms, int nb, int D, int I, int fmt, const Tables &tb,
                const int *nr, const int *xoff, const void *x, int x_dtype, int x_rows,
                bool x_staged, int avg_rows, int act, float act_a, float act_b, RunWs &w,
                bool allow_tc = true, const ExpertPlan *pre = nullptr) {
    const ExpertPlan ep = pre ? *pre
                              : make_expert_plan(nb, D, I, fmt, tb, nr, xoff, x_rows, avg_rows, w,
                                                 allow_tc);
    const PlanArgs &pa = ep.pa;
    const bool fast = ep.fast, mx = ep.mx;
    w.y16 = fast; // the decode and tensor-core kernels write f16 rows of y
    const int tc_min = ep.tc_min, mode = ep.mode, nt = ep.nt;
    if (!pre)
        CUDA_TRY(launch_pdl(plan_kernel, dim3(1), dim3(1024), 0, st, pa));
    prof_mark(st, kPhPlan);

    const void *xop = x;
    if (!x_staged) {
        if (fast) {
            const int blocks = std::max(1, std::min(x_rows, 8 * sms));
            if (x_dtype == MVLLM_DTYPE_BF16)
                CUDA_TRY(launch_pdl(stage_rows_f16x8_kernel<__nv_bfloat16>, dim3(blocks), dim3(256),
                                    0, st, static_cast<const __nv_bfloat16 *>(x),
                                    static_cast<const int *>(nullptr),
                                    static_cast<const int *>(nullptr), x_rows, D, fmt,
                                    static_cast<__half *>(w.xs), w.err));
            else
                CUDA_TRY(launch_pdl(stage_rows_f16x8_kernel<float>, dim3(blocks), dim3(256), 0, st,
                                    static_cast<const float *>(x),
                                    static_cast<const int *>(nullptr),
                                    static_cast<const int *>(nullptr), x_rows, D, fmt,
                                    static_cast<__half *>(w.xs), w.err));
            CUDA_TRY(cudaGetLastError());
            xop = w.xs;
        } else if (x_dtype == MVLLM_DTYPE_BF16) {
            stage_rows_kernel<__nv_bfloat16, float><<<std::max(1, std::min(x_rows, 4 * sms)), 256, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(x), nullptr, nullptr, x_rows, D, fmt,
                static_cast<float *>(w.xs));
            CUDA_TRY(cudaGetLastError());
            xop = w.xs;
        }
    }

    if (fast) {
        // Per-expert tensor maps: host templates, device-side address swap.
        TmapTemplates tpl;
        int box3d = getenv("MVLLM_DECODE_2D_BOXES") ? 0 : 1;
        if (int rc = decode_templates(&tpl, fmt, D, I, w.y, &box3d))
            return rc;
        const int nmaps = nb * kTmapsPerExpert;
        // (the plan kernel cleared w.tmaps_dirty)
        if (!pre)
            CUDA_TRY(launch_pdl(build_tmaps_kernel<kTmapsPerExpert>, dim3((nmaps + 127) / 128),
                                dim3(128), 0, st, tpl,
                                TableSet<kTmapsPerExpert>{{tb.g, tb.u, tb.d, tb.gs, tb.us, tb.ds}},
                                nb, w.tmaps, w.tmaps_dirty));
        CUtensorMap tok1{}, tok2{}, tsc1{}, tsc2{};
        TcArgs t1{};
        const int kind = mode_kind(mode), nterm = mx ? mode_nterm(mode) : 0;
        if (tc_min && mx) {
            TmapSet<kMxMapCount> mtpl;
            if (int rc = make_mx_templates(&mtpl, kind, D, I, w.y))
                return rc;
            const int nmx = nb * kMxMapCount;
            build_tmaps_kernel<kMxMapCount><<<(nmx + 127) / 128, 128, 0, st>>>(
                mtpl, TableSet<kMxMapCount>{{tb.g, tb.u, tb.d, tb.gs, tb.us, tb.ds}}, nb,
                w.mx_tmaps, w.tmaps_dirty);
            CUDA_TRY(cudaGetLastError());
            // x as block-scaled terms, then the maps of both phases' operands.
            if (int rc = launch_terms(mode, xop, x_rows, D, w.xq, w.xc, st, sms))
                return rc;
            const uint64_t xb = kind == kMxF4 ? D / 2 : D, hb = kind == kMxF4 ? I / 2 : I;
            if (int rc = encode_planes(&tok1, w.xq, xb, x_rows, nterm, 128,
                                       CU_TENSOR_MAP_SWIZZLE_128B))
                return rc;
            if (int rc = encode_planes(&tsc1, w.xc, D / 32, x_rows, nterm, 16,
                                       CU_TENSOR_MAP_SWIZZLE_NONE))
                return rc;
            if (int rc = encode_planes(&tok2, w.hq, hb, w.h_rows, nterm, 128,
                                       CU_TENSOR_MAP_SWIZZLE_128B))
                return rc;
            if (int rc = encode_planes(&tsc2, w.hc, I / 32, w.h_rows, nterm, 16,
                                       CU_TENSOR_MAP_SWIZZLE_NONE))
                return rc;
        } else if (tc_min) {
            TmapSet<kTcMapCount> ttpl;
            if (int rc = make_tc_templates(&ttpl, fmt, D, I, w.y))
                return rc;
            const int ntc = nb * kTcMapCount;
            build_tmaps_kernel<kTcMapCount><<<(ntc + 127) / 128, 128, 0, st>>>(
                ttpl, TableSet<kTcMapCount>{{tb.g, tb.u, tb.d, tb.gs, tb.us, tb.ds}}, nb,
                w.tc_tmaps, w.tmaps_dirty);
            CUDA_TRY(cudaGetLastError());
            if (int rc = make_tok_map(&tok1, xop, D, x_rows))
                return rc;
            if (int rc = make_tok_map(&tok2, w.h, I, w.h_rows))
                return rc;
        }
        if (tc_min) {
            t1.tmaps = w.tc_tmaps;
            t1.tmaps_dirty = w.tmaps_dirty;
            t1.s0 = tb.gs, t1.s1 = tb.us;
            t1.xrow = xoff, t1.orow = w.base, t1.cnt = w.cnt, t1.item_off = w.toff1, t1.nb = nb;
            t1.small_max = pa.tc_small; // the plan's split of each expert's tiles
            t1.wide_max = pa.tc_wide;
            t1.tshift = pa.tc_shift;
            t1.K = D, t1.O = I, t1.out = w.h;
            t1.act = act, t1.act_a = act_a, t1.act_b = act_b, t1.err = w.err;
            t1.range = w.range;
        }
        DecodeArgs a{};
        a.tmaps = w.tmaps;
        a.tmaps_dirty = w.tmaps_dirty;
        a.xrow = xoff, a.orow = w.base, a.cnt = w.cnt, a.item_off = w.off1, a.nb = nb;
        a.x = static_cast<const __half *>(xop);
        a.K = D, a.O = I, a.out = w.h;
        a.act = act, a.act_a = act_a, a.act_b = act_b, a.err = w.err;
        a.wbox3d = box3d;
        int rc = (fmt == MVLLM_FMT_MXFP4)
                     ? launch_decode<MVLLM_FMT_MXFP4, 1>(a, pick_ks(D), nt, st, sms)
                     : launch_decode<MVLLM_FMT_INT4_G64, 1>(a, pick_ks(D), nt, st, sms);
        if (rc)
            return rc;
        if (tc_min) {
            TcArgs s1 = t1;
            s1.item_off = w.soff1;
            if (mx)
                rc = launch_mx<1>(mode, MxArgs{t1, w.mx_tmaps}, MxArgs{s1, w.mx_tmaps}, tok1, tsc1,
                                  st, sms);
            else {
                TcArgs w1 = t1;
                w1.item_off = w.woff1;
                rc = launch_tc<1>(fmt, t1, s1, pa.tc_wide > pa.tc_small ? &w1 : nullptr, tok1,
                                  st, sms);
            }
            if (rc)
                return rc;
            // Scale codes the tensor-core operands cannot represent: the
            // decode kernels recompute h of every tensor-core expert (a
            // launch that returns at once when nothing was raised).
            DecodeArgs r = a;
            r.item_off = w.roff1, r.enable = w.range;
            rc = (fmt == MVLLM_FMT_MXFP4)
                     ? launch_decode<MVLLM_FMT_MXFP4, 1>(r, pick_ks(D), nt, st, sms)
                     : launch_decode<MVLLM_FMT_INT4_G64, 1>(r, pick_ks(D), nt, st, sms);
            if (rc)
                return rc;
            // h (every phase-1 row, f16) as terms for the block-scaled phase 2.
            if (mx && (rc = launch_terms(mode, w.h, w.h_rows, I, w.hq, w.hc, st, sms)))
                return rc;
        }
        prof_mark(st, kPhExpert1);
        DecodeArgs b = a;
        b.xrow = w.base, b.item_off = w.off2;
        b.x = static_cast<const __half *>(w.h);
        b.K = I, b.O = D, b.out = w.y;
        rc = (fmt == MVLLM_FMT_MXFP4)
                 ? launch_decode<MVLLM_FMT_MXFP4, 2>(b, pick_ks(I), nt, st, sms)
                 : launch_decode<MVLLM_FMT_INT4_G64, 2>(b, pick_ks(I), nt, st, sms);
        if (rc)
            return rc;
        if (tc_min) {
            TcArgs t2 = t1;
            t2.s0 = tb.ds, t2.s1 = nullptr;
            t2.xrow = w.base, t2.item_off = w.toff2;
            t2.K = I, t2.O = D, t2.out = w.y;
            TcArgs s2 = t2;
            s2.item_off = w.soff2;
            if (mx)
                rc = launch_mx<2>(mode, MxArgs{t2, w.mx_tmaps}, MxArgs{s2, w.mx_tmaps}, tok2, tsc2,
                                  st, sms);
            else {
                TcArgs w2 = t2;
                w2.item_off = w.woff2;
                rc = launch_tc<2>(fmt, t2, s2, pa.tc_wide > pa.tc_small ? &w2 : nullptr, tok2,
                                  st, sms);
            }
            if (rc)
                return rc;
            DecodeArgs r = b;
            r.item_off = w.roff2, r.enable = w.range;
            rc = (fmt == MVLLM_FMT_MXFP4)
                     ? launch_decode<MVLLM_FMT_MXFP4, 2>(r, pick_ks(I), nt, st, sms)
                     : launch_decode<MVLLM_FMT_INT4_G64, 2>(r, pick_ks(I), nt, st, sms);
            if (rc)
                return rc;
        }
        prof_mark(st, kPhExpert2);
        return MVLLM_OK;
    }
    GenericArgs a{};
    a.w0 = tb.g, a.w1 = tb.u, a.s0 = (fmt == MVLLM_FMT_F32) ? nullptr : tb.gs;
    a.s1 = (fmt == MVLLM_FMT_F32) ? nullptr : tb.us;
    a.xrow = xoff, a.orow = w.base, a.cnt = w.cnt, a.item_off = w.off1, a.nb = nb, a.fmt = fmt;
    a.x = static_cast<const float *>(xop);
    a.K = D, a.O = I, a.out = static_cast<float *>(w.h);
    a.act = act, a.act_a = act_a, a.act_b = act_b;
    generic_ffn_kernel<1><<<sms * 8, 256, 0, st>>>(a);
    CUDA_TRY(cudaGetLastError());
    prof_mark(st, kPhExpert1);
    GenericArgs b = a;
    b.w0 = tb.d, b.w1 = nullptr, b.s0 = (fmt == MVLLM_FMT_F32) ? nullptr : tb.ds, b.s1 = nullptr;
    b.xrow = w.base, b.item_off = w.off2;
    b.x = static_cast<const float *>(w.h);
    b.K = I, b.O = D, b.out = w.y;
    generic_ffn_kernel<2><<<sms * 8, 256, 0, st>>>(b);
    CUDA_TRY(cudaGetLastError());
    prof_mark(st, kPhExpert2);
    return MVLLM_OK;
}

// [p, p + n) lies inside a buffer the caller page-locked with host_register.
bool host_registered(const Context &c, const void *p, size_t n) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    auto it = c.host_reg.upper_bound(a);
    if (it == c.host_reg.begin())
        return false;
    --it;
    return a >= it->first && a + n <= it->first + it->second;
}

int check_device_error(const int *err_dev, cudaStream_t st) {
    int err = 0;
    CUDA_TRY(cudaMemcpyAsync(&err, err_dev, sizeof(int), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (err)
        return fail(err, "device-side error code %d", err);
    return MVLLM_OK;
}

int init_locked(Context &c, int device) {
    if (c.inited && c.device == device)
        return MVLLM_OK;
    if (c.inited)
        return fail(MVLLM_ERR_INVALID, "already initialised on device %d", c.device);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return fail(MVLLM_ERR_CUDA, "no CUDA device");
    }
    if (device < 0 || device >= n)
        return fail(MVLLM_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop{};
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(MVLLM_ERR_UNSUPPORTED, "device %d is sm_%d%d, this build targets sm_100a",
                    device, prop.major, prop.minor);
    CUDA_TRY(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    CUDA_TRY(cudaStreamCreateWithFlags(&c.copy_stream, cudaStreamNonBlocking));
    CUDA_TRY(cudaEventCreateWithFlags(&c.copy_done, cudaEventDisableTiming));
    for (cudaEvent_t *e : {&c.call_start, &c.x_in, &c.out_in, &c.x_head})
        CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    for (auto &e : c.ev)
        CUDA_TRY(cudaEventCreate(&e));
    c.sms = prop.multiProcessorCount;
    c.device = device;
    c.inited = true;
    return MVLLM_OK;
}

int ensure_current(Context &c) {
    if (!c.inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    CUDA_TRY(cudaSetDevice(c.device));
    return MVLLM_OK;
}

// Device address for a host array of `len` bytes: the registered cache copy
// when one covers it, else a per-call upload into the transient arena.
struct Resolver {
    Context &c;
    std::unordered_map<const void *, void *> seen;
    std::vector<std::pair<const void *, size_t>> uploads; // host ptr, bytes
    std::vector<size_t> up_off;
    size_t transient_bytes = 0;

    explicit Resolver(Context &cc) : c(cc) {}

    // The range the last lookup resolved (a registered buffer or a tier
    // blob), checked before the maps: an expert's six arrays usually lie in
    // one ExpertStore slot, so five of six lookups stop here.
    uintptr_t memo_lo = 0, memo_hi = 0;
    uint8_t *memo_dev = nullptr;
    bool memo_late = false;

    // First pass: returns the cached device pointer or nullptr (to upload).
    void *cached(const void *host, size_t len) {
        if (!host)
            return nullptr;
        auto it = c.cache.upper_bound(reinterpret_cast<uintptr_t>(host));
        if (it == c.cache.begin())
            return nullptr;
        --it;
        const uintptr_t start = it->first, h = reinterpret_cast<uintptr_t>(host);
        if (h >= start && h + len <= start + it->second.bytes) {
            memo_lo = start, memo_hi = start + it->second.bytes;
            memo_dev = static_cast<uint8_t *>(it->second.dev), memo_late = false;
            return static_cast<uint8_t *>(it->second.dev) + (h - start);
        }
        return nullptr;
    }

    // Blobs of the device tier this call copies into their slots (issued on
    // the copy stream before the call's second batch of experts).
    std::vector<TierEntry *> stream_in;
    bool tier_miss = false; // the array lies in a blob being streamed in

    // Through the device tier: a resident blob's slot, or a slot the blob is
    // streamed into (noted in stream_in), or nullptr (not bound, or no slot).
    void *tiered(const void *host, size_t len) {
        tier_miss = false;
        if (!c.tier_arena)
            return nullptr;
        TierEntry *e = c.tier.find(reinterpret_cast<uintptr_t>(host), len);
        if (!e)
            return nullptr;
        bool copy = false;
        const int slot = c.tier.acquire(*e, &copy);
        if (slot < 0)
            return nullptr;
        if (copy)
            stream_in.push_back(e);
        for (TierEntry *s : stream_in)
            if (s == e)
                tier_miss = true;
        uint8_t *base = static_cast<uint8_t *>(c.tier_arena) + size_t(slot) * c.tier.slot_bytes();
        memo_lo = e->host, memo_hi = e->host + e->bytes, memo_dev = base, memo_late = tier_miss;
        return base + (reinterpret_cast<uintptr_t>(host) - e->host);
    }

    // Returns an index into uploads (or -1 when cached/null) and, through
    // *dev_or_null, the device pointer for cached arrays.  *late: the array
    // arrives with the stream-in copies (its expert runs in the second batch).
    long note(const void *host, size_t len, void **dev, bool *late = nullptr) {
        *dev = nullptr;
        if (late)
            *late = false;
        if (!host)
            return -1;
        const uintptr_t h = reinterpret_cast<uintptr_t>(host);
        if (memo_dev && h >= memo_lo && h + len <= memo_hi) {
            *dev = memo_dev + (h - memo_lo);
            if (late)
                *late = memo_late;
            return -1;
        }
        if (void *p = cached(host, len)) {
            *dev = p;
            return -1;
        }
        if (void *p = tiered(host, len)) {
            *dev = p;
            if (late)
                *late = tier_miss;
            return -1;
        }
        auto it = seen.find(host);
        if (it != seen.end())
            return reinterpret_cast<long>(it->second);
        const long idx = static_cast<long>(uploads.size());
        uploads.push_back({host, len});
        transient_bytes = (transient_bytes + 255) & ~size_t(255);
        up_off.push_back(transient_bytes);
        transient_bytes += len;
        seen[host] = reinterpret_cast<void *>(idx);
        return idx;
    }
};

} // namespace

// =================================================================== C ABI ==
namespace {
template <int KIND, bool PAIR> int mma_rate_t(int n, int iters, int sms, double *tflops) {
    auto kern = mma_rate_kernel<KIND, PAIR>;
    // 120 KB of (unused) dynamic shared memory keeps one CTA per SM.
    const int pad = 120 * 1024;
    CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pad));
    int *err = nullptr;
    CUDA_TRY(cudaMalloc(&err, sizeof(int)));
    CUDA_TRY(cudaMemset(err, 0, sizeof(int)));
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(128);
    cfg.gridDim = dim3(PAIR ? (sms & ~1) : sms);
    cfg.dynamicSmemBytes = pad;
    cudaLaunchAttribute at[1];
    if (PAIR) {
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    }
    cudaEvent_t e0, e1;
    CUDA_TRY(cudaEventCreate(&e0));
    CUDA_TRY(cudaEventCreate(&e1));
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, n, std::max(16, iters / 10), err)); // warm
    CUDA_TRY(cudaEventRecord(e0));
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, n, iters, err));
    CUDA_TRY(cudaEventRecord(e1));
    CUDA_TRY(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&ms, e0, e1));
    int herr = 0;
    CUDA_TRY(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost));
    cudaFree(err);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (herr)
        return fail(herr, "mma_rate: device error %d", herr);
    const double kstep = KIND == 0 ? 64 : KIND == 1 ? 32 : 16;
    const double units = PAIR ? (sms & ~1) / 2 : sms;
    *tflops = 2.0 * (PAIR ? 256 : 128) * n * kstep * iters * units / (ms * 1e-3) / 1e12;
    return MVLLM_OK;
}
} // namespace

extern "C" {

int mvllm_moe_init(int device) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    return init_locked(c, device);
}

void mvllm_moe_shutdown(void) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (!c.inited)
        return;
    cudaSetDevice(c.device);
    cudaStreamSynchronize(c.stream);
    cudaStreamSynchronize(c.copy_stream);
    for (auto &kv : c.cache)
        cudaFree(kv.second.dev);
    c.cache.clear();
    c.cache_bytes = 0;
    if (c.tier_arena)
        cudaFree(c.tier_arena);
    c.tier_arena = nullptr;
    c.tier.configure(0, 0);
    for (auto &kv : c.host_reg)
        cudaHostUnregister(reinterpret_cast<void *>(kv.first));
    c.host_reg.clear();
    if (c.ws.p)
        cudaFree(c.ws.p);
    if (c.transient.p)
        cudaFree(c.transient.p);
    if (c.pinned)
        cudaFreeHost(c.pinned);
    c.ws = DevBuf{};
    c.transient = DevBuf{};
    c.pinned = nullptr;
    c.pinned_bytes = 0;
    for (auto &e : c.ev)
        cudaEventDestroy(e);
    cudaEventDestroy(c.copy_done);
    for (cudaEvent_t e : {c.call_start, c.x_in, c.out_in, c.x_head})
        cudaEventDestroy(e);
    c.call_start = c.x_in = c.out_in = c.x_head = nullptr;
    cudaStreamDestroy(c.copy_stream);
    cudaStreamDestroy(c.stream);
    c.stream = nullptr;
    c.copy_stream = nullptr;
    c.copy_done = nullptr;
    c.inited = false;
    c.device = -1;
}

int mvllm_moe_available(void) { return ctx().inited ? 1 : 0; }

int mvllm_moe_set_prefill_mode(int mode) {
    if (mode < -1 || mode > MVLLM_PREFILL_MXF8_X2)
        return fail(MVLLM_ERR_INVALID, "set_prefill_mode: unknown mode %d", mode);
    g_prefill_mode.store(mode);
    return MVLLM_OK;
}

int mvllm_moe_get_prefill_mode(void) { return prefill_mode(); }

int mvllm_moe_set_exact(int on) {
    if (on < -1 || on > 1)
        return fail(MVLLM_ERR_INVALID, "set_exact: %d is not -1, 0 or 1", on);
    g_exact.store(on);
    return MVLLM_OK;
}

int mvllm_moe_get_exact(void) { return exact_mode() ? 1 : 0; }

int mvllm_moe_set_sm_limit(int sms) {
    if (sms < 0)
        return fail(MVLLM_ERR_INVALID, "set_sm_limit: negative SM count");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    c.sm_limit = sms;
    return MVLLM_OK;
}


int mvllm_moe_mma_rate(int kind, int n, int pair, int iters, double *tflops) {
    if (kind < 0 || kind > 2 || n < 16 || n > 256 || n % 16 || iters < 1 || !tflops ||
        (kind == 2 && pair))
        return fail(MVLLM_ERR_INVALID, "mma_rate: invalid arguments");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    if (kind == 0)
        return pair ? mma_rate_t<0, true>(n, iters, c.sms, tflops)
                    : mma_rate_t<0, false>(n, iters, c.sms, tflops);
    if (kind == 1)
        return pair ? mma_rate_t<1, true>(n, iters, c.sms, tflops)
                    : mma_rate_t<1, false>(n, iters, c.sms, tflops);
    return mma_rate_t<2, false>(n, iters, c.sms, tflops);
}

int mvllm_mx_terms_dev(void *stream, int mode, const void *src, int rows, int K, void *planes,
                       void *codes) {
    if (mode <= MVLLM_PREFILL_F16 || mode > MVLLM_PREFILL_MXF8_X2 || !src || !planes || !codes ||
        rows < 1 || K < 32 || K % 32 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) ||
        (reinterpret_cast<uintptr_t>(planes) & 7u))
        return fail(MVLLM_ERR_INVALID, "mx_terms_dev: invalid arguments");
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    return launch_terms(mode, src, rows, K, static_cast<uint8_t *>(planes),
                        static_cast<uint8_t *>(codes), static_cast<cudaStream_t>(stream), sms);
}

const char *mvllm_moe_backend_name(void) { return "cuda-sm100a"; }

const char *mvllm_moe_last_error(void) { return g_last_error.c_str(); }

void mvllm_moe_stats(uint64_t *calls, uint64_t *experts, uint64_t *rows, double *h2d_ms,
                     double *kernel_ms, double *d2h_ms) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (calls)
        *calls = c.calls;
    if (experts)
        *experts = c.experts;
    if (rows)
        *rows = c.rows;
    if (h2d_ms)
        *h2d_ms = c.h2d_ms;
    if (kernel_ms)
        *kernel_ms = c.kernel_ms;
    if (d2h_ms)
        *d2h_ms = c.d2h_ms;
}

// ----------------------------------------------------------- expert cache --
int mvllm_moe_cache_register(const void *host, size_t bytes, uint64_t generation) {
    if (!host || bytes == 0)
        return fail(MVLLM_ERR_INVALID, "cache_register: null pointer or zero size");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    const uintptr_t key = reinterpret_cast<uintptr_t>(host);
    auto it = c.cache.find(key);
    if (it != c.cache.end()) {
        if (it->second.bytes == bytes && it->second.generation == generation)
            return MVLLM_OK;
        cudaFree(it->second.dev);
        c.cache_bytes -= it->second.bytes;
        c.cache.erase(it);
    }
    // Ranges may not overlap: an overlapping older entry is dropped.
    for (auto jt = c.cache.begin(); jt != c.cache.end();) {
        const uintptr_t s = jt->first, e = s + jt->second.bytes;
        if (s < key + bytes && key < e) {
            cudaFree(jt->second.dev);
            c.cache_bytes -= jt->second.bytes;
            jt = c.cache.erase(jt);
        } else {
            ++jt;
        }
    }
    CacheEntry ce;
    if (cudaMalloc(&ce.dev, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(MVLLM_ERR_NOMEM, "cache_register: cudaMalloc(%zu) failed", bytes);
    }
    if (cudaMemcpy(ce.dev, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(ce.dev);
        return fail(MVLLM_ERR_CUDA, "cache_register: upload failed");
    }
    ce.bytes = bytes;
    ce.generation = generation;
    c.cache[key] = ce;
    c.cache_bytes += bytes;
    return MVLLM_OK;
}

int mvllm_moe_cache_unregister(const void *host) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    auto it = c.cache.find(reinterpret_cast<uintptr_t>(host));
    if (it == c.cache.end())
        return fail(MVLLM_ERR_INVALID, "cache_unregister: pointer not registered");
    if (c.inited)
        cudaSetDevice(c.device);
    cudaFree(it->second.dev);
    c.cache_bytes -= it->second.bytes;
    c.cache.erase(it);
    return MVLLM_OK;
}

void mvllm_moe_cache_clear(void) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (c.inited)
        cudaSetDevice(c.device);
    for (auto &kv : c.cache)
        cudaFree(kv.second.dev);
    c.cache.clear();
    c.cache_bytes = 0;
}

size_t mvllm_moe_cache_bytes(void) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    return c.cache_bytes;
}

// ------------------------------------------------ page-locked caller buffers --
int mvllm_moe_host_register(void *host, size_t bytes) {
    if (!host || bytes == 0)
        return fail(MVLLM_ERR_INVALID, "host_register: null pointer or zero size");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    const uintptr_t a = reinterpret_cast<uintptr_t>(host);
    auto it = c.host_reg.find(a);
    if (it != c.host_reg.end() && it->second == bytes)
        return MVLLM_OK;
    for (auto &kv : c.host_reg)
        if (kv.first < a + bytes && a < kv.first + kv.second)
            return fail(MVLLM_ERR_INVALID, "host_register: overlaps a registered buffer");
    if (cudaHostRegister(host, bytes, cudaHostRegisterDefault) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return fail(MVLLM_ERR_CUDA, "host_register: %s", cudaGetErrorString(e));
    }
    c.host_reg[a] = bytes;
    return MVLLM_OK;
}

int mvllm_moe_host_unregister(void *host) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    auto it = c.host_reg.find(reinterpret_cast<uintptr_t>(host));
    if (it == c.host_reg.end())
        return fail(MVLLM_ERR_INVALID, "host_unregister: buffer not registered");
    if (c.inited) {
        cudaSetDevice(c.device);
        cudaStreamSynchronize(c.stream);
    }
    cudaHostUnregister(host);
    c.host_reg.erase(it);
    return MVLLM_OK;
}

// ----------------------------------------------------- device expert tier --
int mvllm_moe_tier_configure(size_t budget_bytes, size_t slot_bytes) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    if (budget_bytes > 0 && slot_bytes == 0)
        return fail(MVLLM_ERR_INVALID, "tier_configure: zero slot size");
    cudaStreamSynchronize(c.copy_stream);
    if (c.tier_arena)
        cudaFree(c.tier_arena);
    c.tier_arena = nullptr;
    const size_t slot = (slot_bytes + 255) & ~size_t(255);
    const size_t n = slot ? budget_bytes / slot : 0;
    c.tier.configure(0, slot);
    if (n == 0)
        return MVLLM_OK; // tier off
    if (n > size_t(1) << 20)
        return fail(MVLLM_ERR_INVALID, "tier_configure: %zu slots", n);
    if (cudaMalloc(&c.tier_arena, n * slot) != cudaSuccess) {
        cudaGetLastError();
        c.tier_arena = nullptr;
        return fail(MVLLM_ERR_NOMEM, "tier_configure: cudaMalloc(%zu) failed", n * slot);
    }
    c.tier.configure(static_cast<int>(n), slot);
    return MVLLM_OK;
}

int mvllm_moe_expert_bind(const void *host_blob, size_t bytes, uint64_t generation) {
    if (!host_blob || bytes == 0)
        return fail(MVLLM_ERR_INVALID, "expert_bind: null pointer or zero size");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    c.tier.bind(reinterpret_cast<uintptr_t>(host_blob), bytes, generation);
    return MVLLM_OK;
}

int mvllm_moe_expert_unbind(const void *host_blob) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (!c.tier.unbind(reinterpret_cast<uintptr_t>(host_blob)))
        return fail(MVLLM_ERR_INVALID, "expert_unbind: blob not bound");
    return MVLLM_OK;
}

void mvllm_moe_tier_stats(uint64_t *hits, uint64_t *misses, uint64_t *evictions,
                          uint64_t *bytes_in, uint64_t *overflow, uint64_t *overflow_bytes,
                          size_t *resident_bytes) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    const TierStats &t = c.tier.stats();
    if (hits)
        *hits = t.hits;
    if (misses)
        *misses = t.misses;
    if (evictions)
        *evictions = t.evictions;
    if (bytes_in)
        *bytes_in = t.bytes_in;
    if (overflow)
        *overflow = t.overflow;
    if (overflow_bytes)
        *overflow_bytes = t.overflow_bytes;
    if (resident_bytes)
        *resident_bytes = c.tier.resident_bytes();
}

// ----------------------------------------------------- moe_block (host) --
static int moe_block_impl(int nb, int D, int Iinter, int fmt, const void *const *g,
                          const void *const *u, const void *const *d, const float *const *gs,
                          const float *const *us, const float *const *ds, const float *xg,
                          const int *xoff, const int *nr, const int *rows, const float *rw,
                          float *out, int S, int act, float act_a, float act_b, bool allow_tc);

int mvllm_moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
                    const void *const *u, const void *const *d, const float *const *gs,
                    const float *const *us, const float *const *ds, const float *xg,
                    const int *xoff, const int *nr, const int *rows, const float *rw, float *out,
                    int S, int act, float act_a, float act_b) {
    (void)qgs;
    int rc = moe_block_impl(nb, D, Iinter, fmt, g, u, d, gs, us, ds, xg, xoff, nr, rows, rw, out,
                            S, act, act_a, act_b, true);
    if (rc == MVLLM_ERR_RANGE) // scale codes the f16 tensor-core operands cannot hold
        rc = moe_block_impl(nb, D, Iinter, fmt, g, u, d, gs, us, ds, xg, xoff, nr, rows, rw, out,
                            S, act, act_a, act_b, false);
    return rc;
}

static int moe_block_impl(int nb, int D, int Iinter, int fmt, const void *const *g,
                          const void *const *u, const void *const *d, const float *const *gs,
                          const float *const *us, const float *const *ds, const float *xg,
                          const int *xoff, const int *nr, const int *rows, const float *rw,
                          float *out, int S, int act, float act_a, float act_b, bool allow_tc) {
    // Argument checks of metal_ops.cpp:452-457.
    if (nb < 1 || D < 1 || !out || !xg || (fmt != 0 && fmt != 4 && fmt != 7))
        return fail(MVLLM_ERR_INVALID, "moe_block: invalid nb/D/out/xg/fmt");
    if (!xoff || !nr)
        return fail(MVLLM_ERR_INVALID, "moe_block: xoff and nr are required");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;

    // Host pass over experts: cpu_moe_block's base/skip rules.
    const bool packed = fmt != MVLLM_FMT_F32;
    int R = 0, n_valid = 0;
    int64_t x_rows = 0;
    std::vector<int> base(nb), valid(nb);
    for (int e = 0; e < nb; ++e) {
        const int n = nr[e];
        base[e] = R;
        valid[e] = 0;
        if (n <= 0)
            continue;
        bool ok = Iinter >= 1 && g && u && d && g[e] && u[e] && d[e];
        if (packed)
            ok = ok && gs && us && ds && gs[e] && us[e] && ds[e];
        if (ok) {
            if (xoff[e] < 0)
                return fail(MVLLM_ERR_INVALID, "moe_block: negative xoff for expert %d", e);
            valid[e] = 1;
            ++n_valid;
            x_rows = std::max<int64_t>(x_rows, int64_t(xoff[e]) + n);
        }
        R += n;
    }
    // Nothing observable happens without rows+rw (the reference computes and
    // discards) or without an expert that runs.
    if (!rows || !rw || n_valid == 0)
        return MVLLM_OK;
    if (x_rows > (int64_t(1) << 31) / std::max(D, 1))
        return fail(MVLLM_ERR_INVALID, "moe_block: activation extent too large");

    // Destinations -> CSR (ascending row id within each destination).
    int S_ext = S;
    if (S <= 0) {
        S_ext = 0;
        for (int e = 0; e < nb; ++e)
            if (valid[e])
                for (int r = 0; r < nr[e]; ++r)
                    S_ext = std::max(S_ext, rows[base[e] + r] + 1);
    }
    std::vector<int> csr_off(size_t(S_ext) + 1, 0), csr_ids;
    for (int e = 0; e < nb; ++e)
        if (valid[e])
            for (int r = 0; r < nr[e]; ++r) {
                const int dest = rows[base[e] + r];
                if (dest >= 0 && dest < S_ext)
                    ++csr_off[size_t(dest) + 1];
            }
    for (int s = 0; s < S_ext; ++s)
        csr_off[size_t(s) + 1] += csr_off[size_t(s)];
    csr_ids.resize(size_t(csr_off[size_t(S_ext)]));
    {
        std::vector<int> cur(csr_off.begin(), csr_off.end() - 1);
        for (int e = 0; e < nb; ++e)
            if (valid[e])
                for (int r = 0; r < nr[e]; ++r) {
                    const int dest = rows[base[e] + r];
                    if (dest >= 0 && dest < S_ext)
                        csr_ids[size_t(cur[size_t(dest)]++)] = base[e] + r;
                }
    }
    if (csr_ids.empty())
        return MVLLM_OK; // every destination filtered out

    // Resolve weights: cached device copies or per-call uploads.
    const size_t gu_b = size_t(Iinter) * row_bytes_packed(fmt, D);
    const size_t d_b = size_t(D) * row_bytes_packed(fmt, Iinter);
    const size_t gus_b = size_t(Iinter) * scale_row_bytes(fmt, D);
    const size_t ds_b = size_t(D) * scale_row_bytes(fmt, Iinter);
    Resolver rs(c);
    if (c.tier_arena) {
        c.tier.begin_call();
        // Slots filled by an earlier call that returned early (an error after
        // its copies were issued) are complete before this call reads them.
        CUDA_TRY(cudaStreamWaitEvent(c.stream, c.copy_done, 0));
    }
    std::vector<void *> tdev(size_t(6) * nb, nullptr);
    std::vector<long> tidx(size_t(6) * nb, -1);
    std::vector<char> late(size_t(nb), 0); // weights arrive with the tier's stream-in copies
    for (int e = 0; e < nb; ++e) {
        if (!valid[e])
            continue;
        const void *hp[6] = {g[e], u[e], d[e], packed ? gs[e] : nullptr, packed ? us[e] : nullptr,
                             packed ? ds[e] : nullptr};
        const size_t len[6] = {gu_b, gu_b, d_b, gus_b, gus_b, ds_b};
        for (int k = 0; k < 6; ++k) {
            bool lt = false;
            tidx[size_t(6) * e + k] = rs.note(hp[k], len[k], &tdev[size_t(6) * e + k], &lt);
            if (lt)
                late[size_t(e)] = 1;
        }
    }
    // Cold tier blobs stream into their slots on the copy stream while the
    // experts whose weights are already on the device run (first batch).
    for (size_t i = 0; i < rs.stream_in.size(); ++i) {
        TierEntry *t = rs.stream_in[i];
        void *dst = static_cast<uint8_t *>(c.tier_arena) + size_t(t->slot) * c.tier.slot_bytes();
        if (cudaMemcpyAsync(dst, reinterpret_cast<const void *>(t->host), t->bytes,
                            cudaMemcpyHostToDevice, c.copy_stream) != cudaSuccess) {
            for (size_t j = i; j < rs.stream_in.size(); ++j)
                c.tier.abandon(*rs.stream_in[j]);
            cudaStreamSynchronize(c.copy_stream);
            return fail(MVLLM_ERR_CUDA, "moe_block: tier stream-in failed: %s",
                        cudaGetErrorString(cudaGetLastError()));
        }
    }
    if (!rs.stream_in.empty())
        CUDA_TRY(cudaEventRecord(c.copy_done, c.copy_stream));
    int n_late = 0;
    for (int e = 0; e < nb; ++e)
        n_late += late[size_t(e)];
    const bool two_batches = n_late > 0;
    if (rs.transient_bytes) {
        if (int rc = ensure_dev(c.transient, rs.transient_bytes))
            return rc;
        for (size_t i = 0; i < rs.uploads.size(); ++i)
            CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t *>(c.transient.p) + rs.up_off[i],
                                     rs.uploads[i].first, rs.uploads[i].second,
                                     cudaMemcpyHostToDevice, c.stream));
        for (size_t i = 0; i < tidx.size(); ++i)
            if (tidx[i] >= 0)
                tdev[i] = static_cast<uint8_t *>(c.transient.p) + rs.up_off[size_t(tidx[i])];
    }
    // Fast path needs 16-byte aligned weight and scale rows.
    bool fast = fast_path_ok(fmt, D, Iinter);
    for (size_t i = 0; i < tdev.size() && fast; ++i)
        if (reinterpret_cast<uintptr_t>(tdev[i]) & 15u)
            fast = false;
    const int fmt_run = fmt;

    // With tier stream-ins, two table sets: the first batch sees the late
    // experts' pointers as null (skipped, their row base still advancing --
    // the plan's rule), the second batch the reverse; both write their own y
    // rows and the combine runs once.
    // Without them, on the fast path, a call with at least kXgSplitBytes of
    // gathered rows uploads xg in two parts: the experts whose rows all lie in
    // the head part (below row x_split) run as a first batch once it has
    // arrived, while the tail copies; the others run after the tail.
    const size_t xb = size_t(x_rows) * D * 4, ob = size_t(S_ext) * D * 4;
    constexpr size_t kXgSplitBytes = size_t(1) << 20;
    int x_split = 0; // rows in the head part; 0: one upload, one batch
    if (!two_batches && fast && n_valid >= 2 && xb >= kXgSplitBytes) {
        const int half = int(x_rows / 2);
        int head = 0;
        for (int e = 0; e < nb; ++e)
            if (valid[e] && xoff[e] + nr[e] <= half)
                ++head;
        if (head > 0 && head < n_valid)
            x_split = half;
    }
    const int n_groups = (two_batches || x_split) ? 2 : 1;
    std::vector<int> grp(size_t(nb), 0);
    for (int e = 0; e < nb; ++e)
        grp[size_t(e)] = two_batches ? (late[size_t(e)] ? 1 : 0)
                         : x_split   ? (valid[e] && xoff[e] + nr[e] > x_split ? 1 : 0)
                                     : 0;
    std::vector<void *> tab(size_t(6) * n_groups * nb, nullptr);
    for (int e = 0; e < nb; ++e)
        for (int k = 0; k < 6; ++k)
            tab[(size_t(6) * grp[size_t(e)] + k) * nb + e] = tdev[size_t(6) * e + k];
    std::vector<int> nr_run(nb), xoff_run(nb);
    for (int e = 0; e < nb; ++e) {
        nr_run[e] = nr[e];
        xoff_run[e] = valid[e] ? xoff[e] : 0;
    }
    Carve hcv(nullptr, ~size_t(0));
    const size_t o_tab = (hcv.take<void *>(tab.size()), hcv.used - tab.size() * sizeof(void *));
    const size_t o_nr = (hcv.take<int>(nb), hcv.used - nb * 4);
    const size_t o_xoff = (hcv.take<int>(nb), hcv.used - nb * 4);
    const size_t o_coff = (hcv.take<int>(csr_off.size()), hcv.used - csr_off.size() * 4);
    const size_t o_cids = (hcv.take<int>(csr_ids.size()), hcv.used - csr_ids.size() * 4);
    const size_t o_rw = (hcv.take<float>(R), hcv.used - size_t(R) * 4);
    const size_t o_x = (hcv.take<uint8_t>(xb), hcv.used - xb);
    const size_t o_out = (hcv.take<uint8_t>(ob), hcv.used - ob);
    const size_t o_err = (hcv.take<int>(16), hcv.used - 64); // the error word, read back
    const size_t up_bytes = hcv.used;
    if (int rc = ensure_pinned(c, up_bytes))
        return rc;
    uint8_t *hp = static_cast<uint8_t *>(c.pinned);
    memcpy(hp + o_tab, tab.data(), tab.size() * sizeof(void *));
    memcpy(hp + o_nr, nr_run.data(), size_t(nb) * 4);
    memcpy(hp + o_xoff, xoff_run.data(), size_t(nb) * 4);
    memcpy(hp + o_coff, csr_off.data(), csr_off.size() * 4);
    memcpy(hp + o_cids, csr_ids.data(), csr_ids.size() * 4);
    memcpy(hp + o_rw, rw, size_t(R) * 4);
    // Caller rows page-locked with mvllm_moe_host_register go straight to
    // the device; the others through the pinned staging buffer.
    const bool x_reg = host_registered(c, xg, xb);
    const bool out_reg = S_ext > 0 && host_registered(c, out, ob);
    if (!x_reg)
        memcpy(hp + o_x, xg, xb);
    if (S_ext > 0 && !out_reg)
        memcpy(hp + o_out, out, ob);

    Carve dcv(nullptr, ~size_t(0));
    dcv.take<uint8_t>(up_bytes);
    RunWs w{};
    carve_run(dcv, w, nb, D, Iinter, fast, R, int(x_rows));
    dcv.take<uint8_t>(ob); // the caller's out rows as uploaded
    if (int rc = ensure_dev(c.ws, dcv.used))
        return rc;
    uint8_t *db = static_cast<uint8_t *>(c.ws.p);
    Carve dcv2(db, c.ws.bytes);
    dcv2.take<uint8_t>(up_bytes);
    carve_run(dcv2, w, nb, D, Iinter, fast, R, int(x_rows));
    uint8_t *d_out_in = dcv2.take<uint8_t>(ob);

    // Metadata on the launch stream; the caller's rows on the copy stream (x,
    // then out, which only the combine reads, so its copy overlaps the expert
    // kernels), except when the tier's stream-ins occupy the copy stream:
    // then on the launch stream ahead of the kernels.
    const void *x_src = x_reg ? static_cast<const void *>(xg) : hp + o_x;
    const void *o_src = out_reg ? static_cast<const void *>(out) : hp + o_out;
    cudaStream_t rows_st = two_batches ? c.stream : c.copy_stream;
    CUDA_TRY(cudaEventRecord(c.ev[0], c.stream));
    CUDA_TRY(cudaMemcpyAsync(db, hp, o_x, cudaMemcpyHostToDevice, c.stream));
    CUDA_TRY(cudaMemsetAsync(w.err, 0, sizeof(int), c.stream));
    if (!two_batches) {
        CUDA_TRY(cudaEventRecord(c.call_start, c.stream));
        CUDA_TRY(cudaStreamWaitEvent(c.copy_stream, c.call_start, 0));
    }
    if (x_split) {
        const size_t hb = size_t(x_split) * D * 4;
        CUDA_TRY(cudaMemcpyAsync(db + o_x, x_src, hb, cudaMemcpyHostToDevice, rows_st));
        CUDA_TRY(cudaEventRecord(c.x_head, rows_st));
        CUDA_TRY(cudaMemcpyAsync(db + o_x + hb, static_cast<const uint8_t *>(x_src) + hb, xb - hb,
                                 cudaMemcpyHostToDevice, rows_st));
    } else {
        CUDA_TRY(cudaMemcpyAsync(db + o_x, x_src, xb, cudaMemcpyHostToDevice, rows_st));
    }
    CUDA_TRY(cudaEventRecord(c.x_in, rows_st));
    if (S_ext > 0) {
        CUDA_TRY(cudaMemcpyAsync(db + o_out, o_src, ob, cudaMemcpyHostToDevice, rows_st));
        if (out_reg) // kept as uploaded: on a device error the caller's rows go back
            CUDA_TRY(cudaMemcpyAsync(d_out_in, db + o_out, ob, cudaMemcpyDeviceToDevice,
                                     rows_st));
    }
    CUDA_TRY(cudaEventRecord(c.out_in, rows_st));
    CUDA_TRY(cudaStreamWaitEvent(c.stream, x_split ? c.x_head : c.x_in, 0));
    CUDA_TRY(cudaEventRecord(c.ev[1], c.stream));
    prof_mark(c.stream, kPhStart);
    void *const *dt = reinterpret_cast<void *const *>(db + o_tab);
    const int *d_nr = reinterpret_cast<const int *>(db + o_nr);
    const int *d_xoff = reinterpret_cast<const int *>(db + o_xoff);
    float *d_out = reinterpret_cast<float *>(db + o_out);
    const float *d_x = reinterpret_cast<const float *>(db + o_x);
    auto run_batch = [&](void *const *t, int xr) -> int {
        Tables tb{t, t + nb, t + 2 * nb, t + 3 * nb, t + 4 * nb, t + 5 * nb};
        if (fast)
            return run_experts(c.stream, launch_sms(c), nb, D, Iinter, fmt_run, tb, d_nr, d_xoff, d_x,
                               MVLLM_DTYPE_F32, xr, false, R / n_valid, act, act_a, act_b, w,
                               allow_tc);
        // Generic path reads the uploaded f32 rows directly.
        RunWs w2 = w;
        w2.xs = const_cast<float *>(d_x);
        return run_experts(c.stream, launch_sms(c), nb, D, Iinter, fmt_run, tb, d_nr, d_xoff, d_x,
                           MVLLM_DTYPE_F32, xr, true, R / n_valid, act, act_a, act_b, w2);
    };
    int rc = MVLLM_OK;
    if (two_batches) {
        if (n_late < n_valid)
            rc = run_batch(dt, int(x_rows));
        if (!rc) {
            CUDA_TRY(cudaStreamWaitEvent(c.stream, c.copy_done, 0));
            rc = run_batch(dt + 6 * nb, int(x_rows));
        }
    } else if (x_split) {
        // The head batch stages only the head rows (the tail may still be
        // copying); the tail batch stages them all.
        rc = run_batch(dt, x_split);
        if (!rc) {
            CUDA_TRY(cudaStreamWaitEvent(c.stream, c.x_in, 0));
            rc = run_batch(dt + 6 * nb, int(x_rows));
        }
    } else {
        rc = run_batch(dt, int(x_rows));
    }
    if (rc) {
        cudaStreamSynchronize(c.copy_stream);
        cudaStreamSynchronize(c.stream);
        return rc;
    }
    CUDA_TRY(cudaStreamWaitEvent(c.stream, c.out_in, 0));
    {
        dim3 grid((D + 255) / 256, std::min(S_ext, 65535));
        const float *crw = reinterpret_cast<const float *>(db + o_rw);
        const int *coff = reinterpret_cast<const int *>(db + o_coff);
        const int *cids = reinterpret_cast<const int *>(db + o_cids);
        if (w.y16)
            combine_csr_kernel<__half><<<grid, 256, 0, c.stream>>>(
                d_out, reinterpret_cast<const __half *>(w.y), crw, coff, cids, S_ext, D);
        else
            combine_csr_kernel<float><<<grid, 256, 0, c.stream>>>(d_out, w.y, crw, coff, cids,
                                                                   S_ext, D);
        CUDA_TRY(cudaGetLastError());
        prof_mark(c.stream, kPhCombine);
    }
    if (out_reg) {
        // The error word and `out` in one round trip; on an error the rows the
        // caller passed in are copied back, so `out` is left as it was.
        int *herr = reinterpret_cast<int *>(hp + o_err);
        CUDA_TRY(cudaEventRecord(c.ev[2], c.stream));
        CUDA_TRY(cudaMemcpyAsync(herr, w.err, sizeof(int), cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaMemcpyAsync(out, d_out, ob, cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaEventRecord(c.ev[3], c.stream));
        CUDA_TRY(cudaStreamSynchronize(c.stream));
        if (*herr) {
            const int err = *herr;
            CUDA_TRY(cudaMemcpyAsync(out, d_out_in, ob, cudaMemcpyDeviceToHost, c.stream));
            CUDA_TRY(cudaStreamSynchronize(c.stream));
            return fail(err, "device-side error code %d", err);
        }
    } else {
        CUDA_TRY(cudaEventRecord(c.ev[2], c.stream));
        CUDA_TRY(cudaMemcpyAsync(hp + o_out, d_out, ob, cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaEventRecord(c.ev[3], c.stream));
        if (int rc2 = check_device_error(w.err, c.stream))
            return rc2; // `out` untouched: a rerun starts from the caller's rows
        memcpy(out, hp + o_out, ob);
    }
    float a = 0, b = 0, cc = 0;
    cudaEventElapsedTime(&a, c.ev[0], c.ev[1]);
    cudaEventElapsedTime(&b, c.ev[1], c.ev[2]);
    cudaEventElapsedTime(&cc, c.ev[2], c.ev[3]);
    c.h2d_ms += a;
    c.kernel_ms += b;
    c.d2h_ms += cc;
    c.calls += 1;
    c.experts += uint64_t(n_valid);
    c.rows += uint64_t(R);
    return MVLLM_OK;
}

// ------------------------------------------------------ moe_block (device) --
size_t mvllm_moe_block_dev_workspace(int nb, int D, int Iinter, int fmt, int rows_cap, int x_rows,
                                     int S) {
    if (nb < 1 || D < 1 || Iinter < 1 || rows_cap < 0 || x_rows < 0 || S < 1)
        return 0;
    const bool fast = fast_path_ok(fmt, D, Iinter);
    Carve cv(nullptr, ~size_t(0));
    RunWs w{};
    carve_run(cv, w, nb, D, Iinter, fast, rows_cap, x_rows);
    cv.take<int>(S);          // hist
    cv.take<int>(size_t(S) + 1); // off
    cv.take<int>(std::max(rows_cap, 1));
    return cv.used + 256;
}

int mvllm_moe_block_dev(void *stream, int nb, int D, int Iinter, int fmt, const void *const *g,
                        const void *const *u, const void *const *d, const void *const *gs,
                        const void *const *us, const void *const *ds, const void *x, int x_dtype,
                        int x_rows, const int *xoff, const int *nr, const int *rows,
                        const float *rw, float *out, int S, int act, float act_a, float act_b,
                        int rows_cap, void *workspace, size_t workspace_bytes) {
    if (nb < 1 || D < 1 || !out || !x || (fmt != 0 && fmt != 4 && fmt != 7) || !xoff || !nr)
        return fail(MVLLM_ERR_INVALID, "moe_block_dev: invalid arguments");
    if (!g || !u || !d || (fmt != MVLLM_FMT_F32 && (!gs || !us || !ds)) || S < 1 || Iinter < 1 ||
        rows_cap < 0 || x_rows < 0)
        return fail(MVLLM_ERR_INVALID, "moe_block_dev: invalid tables or sizes");
    if (x_dtype != MVLLM_DTYPE_F32 && x_dtype != MVLLM_DTYPE_BF16)
        return fail(MVLLM_ERR_INVALID, "moe_block_dev: unknown x dtype");
    if (!rows || !rw)
        return MVLLM_OK;
    const size_t need = mvllm_moe_block_dev_workspace(nb, D, Iinter, fmt, rows_cap, x_rows, S);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "moe_block_dev: workspace %zu < %zu", workspace_bytes,
                    need);
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool fast = fast_path_ok(fmt, D, Iinter);
    Carve cv(workspace, workspace_bytes);
    RunWs w{};
    carve_run(cv, w, nb, D, Iinter, fast, rows_cap, x_rows);
    int *hist = cv.take<int>(S);
    int *off = cv.take<int>(size_t(S) + 1);
    int *ids = cv.take<int>(std::max(rows_cap, 1));
    CUDA_TRY(cudaMemsetAsync(w.err, 0, sizeof(int), st));
    prof_mark(st, kPhStart);
    Tables tb{g, u, d, gs, us, ds};
    const bool staged = !fast && x_dtype == MVLLM_DTYPE_F32;
    int rc = run_experts(st, sms, nb, D, Iinter, fmt, tb, nr, xoff, x, x_dtype, x_rows, staged,
                         rows_cap / nb, act, act_a, act_b, w);
    if (rc)
        return rc;
    build_csr_kernel<<<1, 1024, 0, st>>>(rows, w.base, w.cnt, nb, w.total_rows, S, hist, off, ids);
    CUDA_TRY(cudaGetLastError());
    dim3 grid((D + 255) / 256, std::min(S, 65535));
    if (w.y16)
        combine_csr_kernel<__half><<<grid, 256, 0, st>>>(
            out, reinterpret_cast<const __half *>(w.y), rw, off, ids, S, D);
    else
        combine_csr_kernel<float><<<grid, 256, 0, st>>>(out, w.y, rw, off, ids, S, D);
    CUDA_TRY(cudaGetLastError());
    prof_mark(st, kPhCombine);
    return MVLLM_OK;
}

// --------------------------------------------------------------- permute --
namespace {
struct PermWs {
    uint32_t *bitmap;
    int *wpre;
    float *wsum;
    int words;
};
void carve_perm(Carve &cv, PermWs &p, int T, int K, int E, int n_shared) {
    p.words = (T + 31) / 32;
    p.bitmap = cv.take<uint32_t>(size_t(E + n_shared) * p.words);
    p.wpre = cv.take<int>(size_t(E + n_shared) * p.words);
    p.wsum = cv.take<float>(size_t(T) * (K + n_shared));
}
int run_permute(cudaStream_t st, int sms, const int *idx, const float *wt, int T, int K, int E,
                int n_shared, int *nr, int *xoff, int *rows, float *rw, int *tok_pos,
                int *n_rows, const PermWs &p) {
    if (T <= kPermSmallT && E + n_shared <= 4096) {
        permute_small_kernel<<<1, 1024, 0, st>>>(idx, wt, T, K, E, n_shared, p.words, p.bitmap,
                                                 p.wpre, p.wsum, nr, xoff, n_rows, rows, rw,
                                                 tok_pos);
        CUDA_TRY(cudaGetLastError());
        return MVLLM_OK;
    }
    CUDA_TRY(cudaMemsetAsync(p.bitmap, 0, size_t(E + n_shared) * p.words * 4, st));
    permute_member_kernel<<<std::max(1, std::min((T + 127) / 128, 4 * sms)), 128, 0, st>>>(
        idx, wt, T, K, E, n_shared, p.words, p.bitmap, p.wsum, tok_pos);
    CUDA_TRY(cudaGetLastError());
    permute_count_kernel<<<E + n_shared, 256, 0, st>>>(p.words, p.bitmap, p.wpre, nr);
    CUDA_TRY(cudaGetLastError());
    permute_offsets_kernel<<<1, 1024, 0, st>>>(E + n_shared, nr, xoff, n_rows);
    CUDA_TRY(cudaGetLastError());
    const size_t slots = size_t(T) * (K + n_shared);
    permute_place_kernel<<<static_cast<int>(std::min<size_t>((slots + 255) / 256, 16 * sms)), 256, 0,
                           st>>>(idx, T, K, E, n_shared, p.words, p.bitmap, p.wpre, xoff, p.wsum,
                                 rows, rw, tok_pos);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}
} // namespace

namespace {
// Bytes the permutation's scratch takes from a 256-byte-aligned base (the
// carve's own use, without the alignment slack a caller buffer needs).
size_t perm_scratch_bytes(int T, int K, int E, int n_shared) {
    Carve cv(nullptr, ~size_t(0));
    PermWs p{};
    carve_perm(cv, p, T, K, E, n_shared);
    return cv.used;
}
} // namespace

size_t mvllm_moe_permute_workspace(int T, int K, int E, int n_shared) {
    if (T < 1 || K < 1 || E < 1 || n_shared < 0 || n_shared > 1)
        return 0;
    return perm_scratch_bytes(T, K, E, n_shared) + 256;
}

int mvllm_moe_permute_dev(void *stream, const int *idx, const float *wt, int T, int K, int E,
                          int n_shared, int *nr, int *xoff, int *rows, float *rw, int *tok_pos,
                          int *n_rows, void *workspace, size_t workspace_bytes) {
    if (!idx || !wt || T < 1 || K < 1 || E < 1 || n_shared < 0 || n_shared > 1 || !nr || !xoff ||
        !rows || !rw || !tok_pos || !n_rows)
        return fail(MVLLM_ERR_INVALID, "permute_dev: invalid arguments");
    const size_t need = mvllm_moe_permute_workspace(T, K, E, n_shared);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "permute_dev: workspace too small");
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    Carve cv(workspace, workspace_bytes);
    PermWs p{};
    carve_perm(cv, p, T, K, E, n_shared);
    return run_permute(static_cast<cudaStream_t>(stream), sms, idx, wt, T, K, E, n_shared, nr,
                       xoff, rows, rw, tok_pos, n_rows, p);
}

// ------------------------------------------------ permutation, no allocation --
// Some callers cannot allocate device memory at the moment they need the
// permutation: engines that partition HBM once at start-up and forbid
// allocation in the serving loop, and plugins living inside a host process
// whose own allocator owns the GPU's memory.  For them
// mvllm_moe_permute_dev_noalloc keeps its scratch (membership bitmap and
// per-token weight sums) in this file-scope device array.  Every GPU that
// loads the library holds it until the process exits.
namespace {
constexpr size_t kPermuteStaticBytes = MVLLM_PERMUTE_STATIC_BYTES;
__device__ __align__(256) uint8_t g_permute_scratch[kPermuteStaticBytes];

struct StaticScratch {
    void *ptr = nullptr;
    int sms = 0;
};
std::mutex g_static_mu;
std::map<int, StaticScratch> g_static_by_device;

// Device address of g_permute_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
int static_scratch(StaticScratch *out) {
    int dev = -1;
    CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_static_mu);
    auto it = g_static_by_device.find(dev);
    if (it == g_static_by_device.end()) {
        StaticScratch s;
        const cudaError_t e = cudaGetSymbolAddress(&s.ptr, g_permute_scratch);
        if (e != cudaSuccess || !s.ptr)
            return fail(MVLLM_ERR_CUDA, "cudaGetSymbolAddress(g_permute_scratch) on device %d: %s",
                        dev, cudaGetErrorString(e));
        CUDA_TRY(cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev));
        it = g_static_by_device.emplace(dev, s).first;
    }
    *out = it->second;
    return MVLLM_OK;
}
} // namespace

int mvllm_moe_permute_dev_noalloc(void *stream, const int *idx, const float *wt, int T, int K,
                                  int E, int n_shared, int *nr, int *xoff, int *rows, float *rw,
                                  int *tok_pos, int *n_rows) {
    if (!idx || !wt || T < 1 || K < 1 || E < 1 || n_shared < 0 || n_shared > 1 || !nr || !xoff ||
        !rows || !rw || !tok_pos || !n_rows)
        return fail(MVLLM_ERR_INVALID, "permute_dev_noalloc: invalid arguments");
    // g_permute_scratch is 256-byte aligned, so the carve needs no slack.
    const size_t need = perm_scratch_bytes(T, K, E, n_shared);
    if (need > kPermuteStaticBytes)
        return fail(MVLLM_ERR_WORKSPACE,
                    "permute_dev_noalloc: T=%d K=%d E=%d n_shared=%d needs %zu bytes of scratch, "
                    "above the %zu-byte static maximum; use mvllm_moe_permute_dev",
                    T, K, E, n_shared, need, kPermuteStaticBytes);
    StaticScratch s;
    if (int rc = static_scratch(&s))
        return rc;
    Carve cv(s.ptr, kPermuteStaticBytes);
    PermWs p{};
    carve_perm(cv, p, T, K, E, n_shared);
    // run_permute clears the bitmap before use (the array keeps the previous
    // call's contents); the weight sums are written before they are read.
    return run_permute(static_cast<cudaStream_t>(stream), s.sms, idx, wt, T, K, E, n_shared, nr,
                       xoff, rows, rw, tok_pos, n_rows, p);
}

// ----------------------------------------------------------------- layer --
namespace {
struct LayerWs {
    PermWs perm;
    int *nr, *xoff, *rows, *tok_pos, *n_rows;
    float *rw;
    RunWs run;
};
void carve_layer(Carve &cv, LayerWs &l, int T, int K, int E, int n_shared, int D, int I,
                 bool fast) {
    const int EE = E + n_shared, R = T * (K + n_shared);
    int *err = cv.take<int>(64); // the call's error word at the workspace's first bytes
    carve_perm(cv, l.perm, T, K, E, n_shared);
    l.nr = cv.take<int>(EE);
    l.xoff = cv.take<int>(EE);
    l.rows = cv.take<int>(R);
    l.rw = cv.take<float>(R);
    l.tok_pos = cv.take<int>(R);
    l.n_rows = cv.take<int>(1);
    carve_run(cv, l.run, EE, D, I, fast, R, R);
    l.run.err = err;
}
} // namespace

size_t mvllm_moe_layer_workspace(int T, int K, int E, int n_shared, int D, int Iinter, int fmt) {
    if (T < 1 || K < 1 || E < 1 || n_shared < 0 || n_shared > 1 || D < 1 || Iinter < 1)
        return 0;
    Carve cv(nullptr, ~size_t(0));
    LayerWs l{};
    carve_layer(cv, l, T, K, E, n_shared, D, Iinter, fast_path_ok(fmt, D, Iinter));
    return cv.used + 256;
}

// Host work a caller can slot in before the stages that first read x
// (`before_gather`) and out (`before_combine`): the host-buffer entry stages
// those rows there, so their host copies overlap the device work queued
// ahead of them.
struct LayerHooks {
    std::function<int()> before_gather, before_combine;
    PeerRows peer{};  // partial rows into the owners' exchange windows
};

static int layer_combine(cudaStream_t st, int sms, int T, int KK, int D, float *out,
                         uint8_t *out16, const RunWs &w, const LayerWs &l,
                         const LayerHooks *hooks);

static int layer_dev_impl(cudaStream_t st, int sms, int T, int K, int E, int n_shared, int D,
                          int Iinter, int fmt, const int *idx, const float *wt, const void *x,
                          int x_dtype, const Tables &tb, float *out, int act, float act_a,
                          float act_b, const LayerWs &l, bool allow_tc = true,
                          const LayerHooks *hooks = nullptr, uint8_t *out16 = nullptr) {
    const bool fast = fast_path_ok(fmt, D, Iinter);
    const int EE = E + n_shared, KK = K + n_shared, R = T * KK;
    // Decode-sized calls on the fast path: error word, permutation and plan in
    // one launch, the gather-stage and the decode tensor maps in the next.
    const bool small = fast && T <= kPermSmallT && EE <= 4096;
    ExpertPlan ep{};
    if (small) {
        ep = make_expert_plan(EE, D, Iinter, fmt, tb, l.nr, l.xoff, R, R / EE, l.run, allow_tc);
        PermSmallArgs q{idx, wt, T, K, E, n_shared, l.perm.words, l.perm.bitmap, l.perm.wpre,
                        l.perm.wsum, l.nr, l.xoff, l.n_rows, l.rows, l.rw, l.tok_pos};
        prof_mark(st, kPhStart);
        const size_t psm = perm_smem_bytes(T, KK, EE, l.perm.words);
        const int smem = K <= kPermSmemMaxK && psm <= kPermSmemMaxBytes ? 1 : 0;
        // One thread per expert or slot, whichever is more (the steps loop
        // beyond 1024): fewer warps make each of the CTA's barriers and block
        // scans cheaper.
        const int pthreads = std::min(1024, (std::max({EE, T * KK, 32}) + 31) / 32 * 32);
        CUDA_TRY(launch_pdl(layer_prep_small_kernel, dim3(1), dim3(pthreads), smem ? psm : 0, st,
                            q, ep.pa, smem));
        prof_mark(st, kPhPermute);
        if (hooks && hooks->before_gather)
            if (int rc = hooks->before_gather())
                return rc;
        TmapTemplates tpl;
        int box3d = getenv("MVLLM_DECODE_2D_BOXES") ? 0 : 1;
        if (int rc = decode_templates(&tpl, fmt, D, Iinter, l.run.y, &box3d))
            return rc;
        const int sblocks = std::max(1, std::min(R, 8 * sms));
        const int mblocks = (EE * kTmapsPerExpert + 255) / 256;
        const TableSet<kTmapsPerExpert> tabs{{tb.g, tb.u, tb.d, tb.gs, tb.us, tb.ds}};
        if (x_dtype == MVLLM_DTYPE_BF16)
            CUDA_TRY(launch_pdl(stage_maps_kernel<__nv_bfloat16>, dim3(sblocks + mblocks),
                                dim3(256), 0, st, static_cast<const __nv_bfloat16 *>(x),
                                static_cast<const int *>(l.rows),
                                static_cast<const int *>(l.n_rows), D, fmt,
                                static_cast<__half *>(l.run.xs), l.run.err, sblocks, tpl, tabs,
                                EE, l.run.tmaps, l.run.tmaps_dirty));
        else
            CUDA_TRY(launch_pdl(stage_maps_kernel<float>, dim3(sblocks + mblocks), dim3(256), 0,
                                st, static_cast<const float *>(x),
                                static_cast<const int *>(l.rows),
                                static_cast<const int *>(l.n_rows), D, fmt,
                                static_cast<__half *>(l.run.xs), l.run.err, sblocks, tpl, tabs,
                                EE, l.run.tmaps, l.run.tmaps_dirty));
        prof_mark(st, kPhGather);
        RunWs w = l.run;
        if (int rc = run_experts(st, sms, EE, D, Iinter, fmt, tb, l.nr, l.xoff, l.run.xs,
                                 MVLLM_DTYPE_F32, R, true, R / EE, act, act_a, act_b, w, allow_tc,
                                 &ep))
            return rc;
        return layer_combine(st, sms, T, KK, D, out, out16, w, l, hooks);
    }
    CUDA_TRY(cudaMemsetAsync(l.run.err, 0, sizeof(int), st));
    prof_mark(st, kPhStart);
    if (int rc = run_permute(st, sms, idx, wt, T, K, E, n_shared, l.nr, l.xoff, l.rows, l.rw,
                             l.tok_pos, l.n_rows, l.perm))
        return rc;
    prof_mark(st, kPhPermute);
    if (hooks && hooks->before_gather)
        if (int rc = hooks->before_gather())
            return rc;
    // Gather + stage the token rows into expert-major order: token-major on
    // the fast path (each x row read once, stored at its slots' positions).
    const int gblocks = std::min(R, 8 * sms);
    if (fast) {
        const int tblocks = std::max(1, std::min(T, 8 * sms));
        if (x_dtype == MVLLM_DTYPE_BF16)
            CUDA_TRY(launch_pdl(stage_tokens_f16x8_kernel<__nv_bfloat16>, dim3(tblocks),
                                dim3(256), 0, st, static_cast<const __nv_bfloat16 *>(x),
                                static_cast<const int *>(l.tok_pos), T, KK, D, fmt,
                                static_cast<__half *>(l.run.xs), l.run.err));
        else
            CUDA_TRY(launch_pdl(stage_tokens_f16x8_kernel<float>, dim3(tblocks), dim3(256), 0, st,
                                static_cast<const float *>(x), static_cast<const int *>(l.tok_pos),
                                T, KK, D, fmt, static_cast<__half *>(l.run.xs), l.run.err));
    } else {
        if (x_dtype == MVLLM_DTYPE_BF16)
            stage_rows_kernel<__nv_bfloat16, float><<<gblocks, 256, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(x), l.rows, l.n_rows, 0, D, fmt,
                static_cast<float *>(l.run.xs));
        else
            stage_rows_kernel<float, float><<<gblocks, 256, 0, st>>>(
                static_cast<const float *>(x), l.rows, l.n_rows, 0, D, fmt,
                static_cast<float *>(l.run.xs));
    }
    CUDA_TRY(cudaGetLastError());
    prof_mark(st, kPhGather);
    RunWs w = l.run;
    if (int rc = run_experts(st, sms, EE, D, Iinter, fmt, tb, l.nr, l.xoff, l.run.xs,
                             MVLLM_DTYPE_F32, R, true, R / EE, act, act_a, act_b, w, allow_tc))
        return rc;
    return layer_combine(st, sms, T, KK, D, out, out16, w, l, hooks);
}

// The layer's ordered combine (f32 rows, or the partial-row form).
static int layer_combine(cudaStream_t st, int sms, int T, int KK, int D, float *out,
                         uint8_t *out16, const RunWs &w, const LayerWs &l,
                         const LayerHooks *hooks) {
    if (hooks && hooks->before_combine)
        if (int rc = hooks->before_combine())
            return rc;
    if (out16) {
        const PeerRows peer = hooks ? hooks->peer : PeerRows{};
        const size_t sm = size_t(D) * 4;
        const dim3 grid(std::min(T, 8 * sms));
        if (w.y16) {
            if (sm > 48 * 1024)
                CUDA_TRY(cudaFuncSetAttribute(combine_tokens_f16_kernel<__half>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              int(sm)));
            combine_tokens_f16_kernel<__half><<<grid, 256, sm, st>>>(
                out16, reinterpret_cast<const __half *>(w.y), l.rw, l.tok_pos, T, KK, D, w.err,
                peer);
        } else {
            if (sm > 48 * 1024)
                CUDA_TRY(cudaFuncSetAttribute(combine_tokens_f16_kernel<float>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              int(sm)));
            combine_tokens_f16_kernel<float><<<grid, 256, sm, st>>>(out16, w.y, l.rw, l.tok_pos,
                                                                    T, KK, D, w.err, peer);
        }
    } else {
        const bool cw8 = D % 8 == 0;
        const int cw = cw8 ? 8 : 4;
        dim3 grid(std::max(1, std::min((D / cw + 255) / 256, 8)), std::min(T, 65535));
        const float *rw = l.rw;
        const int *tp = l.tok_pos, *err = w.err;
        if (w.y16) {
            const __half *y = reinterpret_cast<const __half *>(w.y);
            CUDA_TRY(cw8 ? launch_pdl(combine_tokens_kernel<__half, 8>, grid, dim3(256), 0, st,
                                      out, y, rw, tp, T, KK, D, err)
                         : launch_pdl(combine_tokens_kernel<__half, 4>, grid, dim3(256), 0, st,
                                      out, y, rw, tp, T, KK, D, err));
        } else {
            const float *y = w.y;
            CUDA_TRY(cw8 ? launch_pdl(combine_tokens_kernel<float, 8>, grid, dim3(256), 0, st,
                                      out, y, rw, tp, T, KK, D, err)
                         : launch_pdl(combine_tokens_kernel<float, 4>, grid, dim3(256), 0, st,
                                      out, y, rw, tp, T, KK, D, err));
        }
    }
    CUDA_TRY(cudaGetLastError());
    prof_mark(st, kPhCombine);
    return MVLLM_OK;
}

int mvllm_moe_layer_dev(void *stream, int T, int K, int E, int n_shared, int D, int Iinter,
                        int fmt, const int *idx, const float *wt, const void *x, int x_dtype,
                        const void *const *g, const void *const *u, const void *const *d,
                        const void *const *gs, const void *const *us, const void *const *ds,
                        float *out, int act, float act_a, float act_b, void *workspace,
                        size_t workspace_bytes) {
    if (T < 1 || K < 1 || K > 16 || E < 1 || n_shared < 0 || n_shared > 1 || D < 1 ||
        Iinter < 1 || (fmt != 0 && fmt != 4 && fmt != 7) || !idx || !wt || !x || !g || !u || !d ||
        !out || (fmt != MVLLM_FMT_F32 && (!gs || !us || !ds)) || D % 4 != 0)
        return fail(MVLLM_ERR_INVALID, "layer_dev: invalid arguments");
    if (x_dtype != MVLLM_DTYPE_F32 && x_dtype != MVLLM_DTYPE_BF16)
        return fail(MVLLM_ERR_INVALID, "layer_dev: unknown x dtype");
    const size_t need = mvllm_moe_layer_workspace(T, K, E, n_shared, D, Iinter, fmt);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "layer_dev: workspace %zu < %zu", workspace_bytes, need);
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    Carve cv(workspace, workspace_bytes);
    LayerWs l{};
    carve_layer(cv, l, T, K, E, n_shared, D, Iinter, fast_path_ok(fmt, D, Iinter));
    Tables tb{g, u, d, gs, us, ds};
    return layer_dev_impl(static_cast<cudaStream_t>(stream), sms, T, K, E, n_shared, D, Iinter,
                          fmt, idx, wt, x, x_dtype, tb, out, act, act_a, act_b, l);
}

int mvllm_moe_layer_partial_dev(void *stream, int T, int K, int E, int n_shared, int D,
                                int Iinter, int fmt, const int *idx, const float *wt,
                                const void *x, int x_dtype, const void *const *g,
                                const void *const *u, const void *const *d,
                                const void *const *gs, const void *const *us,
                                const void *const *ds, void *out16, int act, float act_a,
                                float act_b, void *workspace, size_t workspace_bytes) {
    if (T < 1 || K < 1 || K > 16 || E < 1 || n_shared < 0 || n_shared > 1 || D < 8 ||
        Iinter < 1 || (fmt != 0 && fmt != 4 && fmt != 7) || !idx || !wt || !x || !g || !u || !d ||
        !out16 || (fmt != MVLLM_FMT_F32 && (!gs || !us || !ds)) || D % 8 != 0 ||
        D > 32768 || (reinterpret_cast<uintptr_t>(out16) & 15u))
        return fail(MVLLM_ERR_INVALID, "layer_partial_dev: invalid arguments");
    if (x_dtype != MVLLM_DTYPE_F32 && x_dtype != MVLLM_DTYPE_BF16)
        return fail(MVLLM_ERR_INVALID, "layer_partial_dev: unknown x dtype");
    const size_t need = mvllm_moe_layer_workspace(T, K, E, n_shared, D, Iinter, fmt);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "layer_partial_dev: workspace %zu < %zu",
                    workspace_bytes, need);
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    Carve cv(workspace, workspace_bytes);
    LayerWs l{};
    carve_layer(cv, l, T, K, E, n_shared, D, Iinter, fast_path_ok(fmt, D, Iinter));
    Tables tb{g, u, d, gs, us, ds};
    return layer_dev_impl(static_cast<cudaStream_t>(stream), sms, T, K, E, n_shared, D, Iinter,
                          fmt, idx, wt, x, x_dtype, tb, nullptr, act, act_a, act_b, l, true,
                          nullptr, static_cast<uint8_t *>(out16));
}

int mvllm_moe_layer_error(void *stream, const void *workspace) {
    if (!workspace)
        return fail(MVLLM_ERR_INVALID, "layer_error: no workspace");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CUDA_TRY(cudaStreamSynchronize(st));
    int code = 0;
    CUDA_TRY(cudaMemcpy(&code, workspace, sizeof(int), cudaMemcpyDeviceToHost));
    return code;
}

static int layer_host_impl(int T, int K, int E, int n_shared, int D, int Iinter, int fmt,
                           const int *idx, const float *wt, const float *x,
                           const void *const *g, const void *const *u, const void *const *d,
                           const void *const *gs, const void *const *us, const void *const *ds,
                           float *out, int act, float act_a, float act_b, bool allow_tc);

int mvllm_moe_layer_host(int T, int K, int E, int n_shared, int D, int Iinter, int fmt,
                         const int *idx, const float *wt, const float *x, const void *const *g,
                         const void *const *u, const void *const *d, const void *const *gs,
                         const void *const *us, const void *const *ds, float *out, int act,
                         float act_a, float act_b) {
    int rc = layer_host_impl(T, K, E, n_shared, D, Iinter, fmt, idx, wt, x, g, u, d, gs, us, ds,
                             out, act, act_a, act_b, true);
    if (rc == MVLLM_ERR_RANGE) // scale codes the f16 tensor-core operands cannot hold
        rc = layer_host_impl(T, K, E, n_shared, D, Iinter, fmt, idx, wt, x, g, u, d, gs, us, ds,
                             out, act, act_a, act_b, false);
    return rc;
}

static int layer_host_impl(int T, int K, int E, int n_shared, int D, int Iinter, int fmt,
                           const int *idx, const float *wt, const float *x,
                           const void *const *g, const void *const *u, const void *const *d,
                           const void *const *gs, const void *const *us, const void *const *ds,
                           float *out, int act, float act_a, float act_b, bool allow_tc) {
    if (T < 1 || K < 1 || K > 16 || E < 1 || n_shared < 0 || n_shared > 1 || D < 1 ||
        Iinter < 1 || (fmt != 0 && fmt != 4 && fmt != 7) || !idx || !wt || !x || !g || !u || !d ||
        !out || (fmt != MVLLM_FMT_F32 && (!gs || !us || !ds)) || D % 4 != 0)
        return fail(MVLLM_ERR_INVALID, "layer_host: invalid arguments");
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    const int EE = E + n_shared;
    const bool fast = fast_path_ok(fmt, D, Iinter);
    const size_t tab_b = size_t(6) * EE * sizeof(void *);
    const size_t idx_b = size_t(T) * K * 4, x_b = size_t(T) * D * 4;
    const size_t up = tab_b + 2 * idx_b + 2 * x_b + 1024 + 64;
    if (int rc = ensure_pinned(c, up))
        return rc;
    // Pinned staging, uploaded in three pieces: tables + routing (read by the
    // permutation), x (first read by the gather), out (read by the combine).
    Carve hcv(c.pinned, c.pinned_bytes);
    void **htab = hcv.take<void *>(size_t(6) * EE);
    int *hidx = hcv.take<int>(size_t(T) * K);
    float *hwt = hcv.take<float>(size_t(T) * K);
    float *hx = hcv.take<float>(size_t(T) * D);
    float *hout = hcv.take<float>(size_t(T) * D);
    int *herr = hcv.take<int>(16); // the error word, read back with `out`
    uint8_t *hbase = static_cast<uint8_t *>(c.pinned);
    const size_t x_off = reinterpret_cast<uint8_t *>(hx) - hbase;
    const size_t out_off = reinterpret_cast<uint8_t *>(hout) - hbase;
    const size_t up_bytes = out_off + x_b;
    for (int e = 0; e < EE; ++e) {
        htab[e] = const_cast<void *>(g[e]);
        htab[EE + e] = const_cast<void *>(u[e]);
        htab[2 * EE + e] = const_cast<void *>(d[e]);
        htab[3 * EE + e] = gs ? const_cast<void *>(gs[e]) : nullptr;
        htab[4 * EE + e] = us ? const_cast<void *>(us[e]) : nullptr;
        htab[5 * EE + e] = ds ? const_cast<void *>(ds[e]) : nullptr;
    }
    memcpy(hidx, idx, idx_b);
    memcpy(hwt, wt, idx_b);
    Carve dcv(nullptr, ~size_t(0));
    dcv.take<uint8_t>(up_bytes);
    LayerWs l{};
    carve_layer(dcv, l, T, K, E, n_shared, D, Iinter, fast);
    dcv.take<float>(size_t(T) * D); // the caller's out rows as uploaded
    if (int rc = ensure_dev(c.ws, dcv.used + 256))
        return rc;
    uint8_t *db = static_cast<uint8_t *>(c.ws.p);
    Carve dcv2(db, c.ws.bytes);
    dcv2.take<uint8_t>(up_bytes);
    carve_layer(dcv2, l, T, K, E, n_shared, D, Iinter, fast);
    float *dout_in = dcv2.take<float>(size_t(T) * D);
    auto dptr = [&](const void *hp) { return db + (static_cast<const uint8_t *>(hp) - hbase); };
    CUDA_TRY(cudaEventRecord(c.ev[0], c.stream));
    CUDA_TRY(cudaMemcpyAsync(db, c.pinned, x_off, cudaMemcpyHostToDevice, c.stream));
    CUDA_TRY(cudaEventRecord(c.ev[1], c.stream));
    void *const *dt = reinterpret_cast<void *const *>(dptr(htab));
    Tables tb{dt, dt + EE, dt + 2 * EE, dt + 3 * EE, dt + 4 * EE, dt + 5 * EE};
    float *dout = reinterpret_cast<float *>(dptr(hout));
    // Caller buffers page-locked with mvllm_moe_host_register are copied
    // straight to and from the device, on the copy stream from the start of the
    // call, so x lands while the permutation runs and out while the experts
    // run; the gather and the combine wait for them.  Other buffers go through
    // the pinned staging, copied in by the host while the kernels run.
    const bool x_reg = host_registered(c, x, x_b), out_reg = host_registered(c, out, x_b);
    if (x_reg || out_reg) {
        CUDA_TRY(cudaEventRecord(c.call_start, c.stream)); // earlier work on these buffers
        CUDA_TRY(cudaStreamWaitEvent(c.copy_stream, c.call_start, 0));
        if (x_reg) {
            CUDA_TRY(cudaMemcpyAsync(db + x_off, x, x_b, cudaMemcpyHostToDevice, c.copy_stream));
            CUDA_TRY(cudaEventRecord(c.x_in, c.copy_stream));
        }
        if (out_reg) {
            CUDA_TRY(cudaMemcpyAsync(dout, out, x_b, cudaMemcpyHostToDevice, c.copy_stream));
            // kept as uploaded: on a device error the caller's rows are put back
            CUDA_TRY(cudaMemcpyAsync(dout_in, dout, x_b, cudaMemcpyDeviceToDevice,
                                     c.copy_stream));
            CUDA_TRY(cudaEventRecord(c.out_in, c.copy_stream));
        }
    }
    LayerHooks hooks;
    hooks.before_gather = [&]() -> int {
        if (x_reg) {
            CUDA_TRY(cudaStreamWaitEvent(c.stream, c.x_in, 0));
            return MVLLM_OK;
        }
        memcpy(hx, x, x_b); // the permutation kernels run meanwhile
        CUDA_TRY(cudaMemcpyAsync(db + x_off, hx, x_b, cudaMemcpyHostToDevice, c.stream));
        return MVLLM_OK;
    };
    hooks.before_combine = [&]() -> int {
        if (out_reg) {
            CUDA_TRY(cudaStreamWaitEvent(c.stream, c.out_in, 0));
            return MVLLM_OK;
        }
        memcpy(hout, out, x_b); // the expert kernels run meanwhile
        CUDA_TRY(cudaMemcpyAsync(dout, hout, x_b, cudaMemcpyHostToDevice, c.stream));
        return MVLLM_OK;
    };
    if (int rc = layer_dev_impl(c.stream, launch_sms(c), T, K, E, n_shared, D, Iinter, fmt,
                                reinterpret_cast<const int *>(dptr(hidx)),
                                reinterpret_cast<const float *>(dptr(hwt)), dptr(hx),
                                MVLLM_DTYPE_F32, tb, dout, act, act_a, act_b, l, allow_tc, &hooks)) {
        cudaStreamSynchronize(c.stream); // no copy may still read the staging buffer
        cudaStreamSynchronize(c.copy_stream); // nor a caller buffer
        return rc;
    }
    if (out_reg) {
        // The error word and `out` in one round trip; on an error the rows the
        // caller passed in are copied back, so `out` is left as it was.
        CUDA_TRY(cudaEventRecord(c.ev[2], c.stream));
        CUDA_TRY(cudaMemcpyAsync(herr, l.run.err, sizeof(int), cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaMemcpyAsync(out, dout, x_b, cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaEventRecord(c.ev[3], c.stream));
        CUDA_TRY(cudaStreamSynchronize(c.stream));
        if (*herr) {
            const int err = *herr;
            CUDA_TRY(cudaMemcpyAsync(out, dout_in, x_b, cudaMemcpyDeviceToHost, c.stream));
            CUDA_TRY(cudaStreamSynchronize(c.stream));
            return fail(err, "device-side error code %d", err);
        }
    } else {
        CUDA_TRY(cudaEventRecord(c.ev[2], c.stream));
        CUDA_TRY(cudaMemcpyAsync(hout, dout, x_b, cudaMemcpyDeviceToHost, c.stream));
        CUDA_TRY(cudaEventRecord(c.ev[3], c.stream));
        if (int rc = check_device_error(l.run.err, c.stream))
            return rc; // `out` untouched: a rerun starts from the caller's rows
        memcpy(out, hout, x_b);
    }
    float a = 0, b = 0, cc = 0;
    cudaEventElapsedTime(&a, c.ev[0], c.ev[1]);
    cudaEventElapsedTime(&b, c.ev[1], c.ev[2]);
    cudaEventElapsedTime(&cc, c.ev[2], c.ev[3]);
    c.h2d_ms += a;
    c.kernel_ms += b;
    c.d2h_ms += cc;
    c.calls += 1;
    c.rows += uint64_t(T) * (K + n_shared);
    return MVLLM_OK;
}

// --------------------------------------------------------------- routing --
static int topk_launch(cudaStream_t st, const float *choice, const float *mix, int T, int E,
                       int K, float scale, int *idx, float *wt) {
    const int warps = 8;
    CUDA_TRY(launch_pdl(topk_kernel, dim3(std::min((T + warps - 1) / warps, 65535)),
                        dim3(32 * warps), 0, st, choice, mix, T, E, K, scale, idx, wt));
    return MVLLM_OK;
}

int mvllm_moe_topk_dev(void *stream, const float *choice, const float *mix, int T, int E, int K,
                       int *idx, float *wt) {
    if (!choice || !idx || !wt || T < 0 || E < 1 || E > 32 * kTopkMaxPerLane || K < 1 ||
        K > kTopkMaxK)
        return fail(MVLLM_ERR_INVALID, "topk_dev: invalid arguments");
    if (T == 0)
        return MVLLM_OK;
    return topk_launch(static_cast<cudaStream_t>(stream), choice, mix, T, E, K, 1.f, idx, wt);
}

int mvllm_moe_route_ex_dev(void *stream, const void *x, int x_dtype, int T, int H,
                           const float *router, const float *bias, int E, int K, int score_fn,
                           float routed_scale, int *idx, float *wt, float *scores,
                           float *choice) {
    if (!x || !router || !idx || !wt || !scores || !choice || T < 0 || H < 1 || E < 1 ||
        E > 32 * kTopkMaxPerLane || K < 1 || K > kTopkMaxK ||
        (x_dtype != MVLLM_DTYPE_F32 && x_dtype != MVLLM_DTYPE_BF16) ||
        (score_fn != MVLLM_SCORE_SIGMOID && score_fn != MVLLM_SCORE_SQRT_SOFTPLUS))
        return fail(MVLLM_ERR_INVALID, "route_dev: invalid arguments");
    if (T == 0)
        return MVLLM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((T + kSeqS - 1) / kSeqS > 65535)
        return fail(MVLLM_ERR_INVALID, "route_dev: T too large");
    // Tolerance mode: 32 experts per CTA (one wave of clusters at E = 256)
    // when the slices fit shared memory, else 16.
    const bool bf = x_dtype == MVLLM_DTYPE_BF16;
    const size_t sm32 = bf ? rf_smem_bytes<__nv_bfloat16, 32>(H) : rf_smem_bytes<float, 32>(H);
    const size_t sm16 = bf ? rf_smem_bytes<__nv_bfloat16, 16>(H) : rf_smem_bytes<float, 16>(H);
    const int exp_per_cta = sm32 <= 200 * 1024 ? 32 : sm16 <= 200 * 1024 ? 16 : 0;
    const bool fast = !exact_mode() && H % 8 == 0 && exp_per_cta > 0 &&
                      (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                      (reinterpret_cast<uintptr_t>(router) & 15u) == 0;
    if (fast) {
        const size_t rf_sm = exp_per_cta == 32 ? sm32 : sm16;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(kRfSplit * ((E + exp_per_cta - 1) / exp_per_cta), (T + 31) / 32);
        cfg.blockDim = dim3(16 * exp_per_cta);
        cfg.dynamicSmemBytes = rf_sm;
        cfg.stream = st;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kRfSplit, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 2;
#define MVB_RF(TXT, N)                                                                         \
    do {                                                                                       \
        CUDA_TRY(cudaFuncSetAttribute(route_scores_fast_kernel<TXT, N>,                        \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(rf_sm))); \
        CUDA_TRY(cudaLaunchKernelEx(&cfg, route_scores_fast_kernel<TXT, N>,                    \
                                    static_cast<const TXT *>(x), router, bias, T, H, E,        \
                                    score_fn, scores, choice));                                \
    } while (0)
        if (bf && exp_per_cta == 32)
            MVB_RF(__nv_bfloat16, 32);
        else if (bf)
            MVB_RF(__nv_bfloat16, 16);
        else if (exp_per_cta == 32)
            MVB_RF(float, 32);
        else
            MVB_RF(float, 16);
#undef MVB_RF
    } else if (x_dtype == MVLLM_DTYPE_BF16) {
        CUDA_TRY(route_scores_launch(st, static_cast<const __nv_bfloat16 *>(x), router, bias, T,
                                     H, E, score_fn, scores, choice));
    } else {
        CUDA_TRY(route_scores_launch(st, static_cast<const float *>(x), router, bias, T, H, E,
                                     score_fn, scores, choice));
    }
    return topk_launch(st, choice, scores, T, E, K, routed_scale, idx, wt);
}

int mvllm_moe_route_dev(void *stream, const void *x, int x_dtype, int T, int H,
                        const float *router, const float *bias, int E, int K, int *idx,
                        float *wt, float *scores, float *choice) {
    return mvllm_moe_route_ex_dev(stream, x, x_dtype, T, H, router, bias, E, K,
                                  MVLLM_SCORE_SIGMOID, 1.f, idx, wt, scores, choice);
}

// ------------------------------------------------------ expert parallelism --
int mvllm_moe_ep_local_ids_dev(void *stream, const int *idx, int T, int K, int E, int nranks,
                               const int *dest, const int *lid, int self_rank, int *local_idx) {
    if (!idx || !local_idx || T < 0 || K < 1 || E < 1 || nranks < 1 || self_rank < 0 ||
        self_rank >= nranks || (!dest) != (!lid))
        return fail(MVLLM_ERR_INVALID, "ep_local_ids_dev: invalid arguments");
    const size_t n = size_t(T) * K;
    if (n == 0)
        return MVLLM_OK;
    const int blocks = int(std::min<size_t>((n + 255) / 256, 4096));
    ep_local_ids_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        idx, int(n), E, nranks, dest, lid, self_rank, local_idx);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_ep_plan_dev(void *stream, const int *idx, int T, int K, int E, int nranks,
                          const int *dest, int self_rank, int *pos, int *send_cnt) {
    if (!idx || !pos || !send_cnt || T < 0 || K < 1 || E < 1 || nranks < 1 || nranks > 32 ||
        self_rank < 0 || self_rank >= nranks)
        return fail(MVLLM_ERR_INVALID, "ep_plan_dev: invalid arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ep_plan_kernel<<<1, 1024, 0, st>>>(idx, T, K, E, nranks, dest, self_rank, pos, send_cnt, 0);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_ep_plan_fixed_dev(void *stream, const int *idx, int T, int K, int E, int nranks,
                                const int *dest, int self_rank, int capacity, int *pos,
                                int *send_cnt) {
    if (!idx || !pos || !send_cnt || T < 0 || K < 1 || E < 1 || nranks < 1 || nranks > 32 ||
        self_rank < 0 || self_rank >= nranks || capacity < T)
        return fail(MVLLM_ERR_INVALID, "ep_plan_fixed_dev: invalid arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ep_plan_kernel<<<1, 1024, 0, st>>>(idx, T, K, E, nranks, dest, self_rank, pos, send_cnt,
                                       capacity);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_ep_pack_dev(void *stream, const void *x, int x_dtype, const int *idx,
                          const float *wt, int T, int K, int D, int E, int nranks, const int *dest,
                          const int *lid, int self_rank, const int *pos, void *send_x,
                          int *send_idx, float *send_wt) {
    if (!x || !idx || !wt || !pos || !send_x || !send_idx || !send_wt || T < 0 || K < 1 ||
        D < 8 || D % 8 != 0 || E < 1 || nranks < 1 || nranks > 32 || self_rank < 0 ||
        self_rank >= nranks || (!dest != !lid) ||
        (x_dtype != MVLLM_DTYPE_F32 && x_dtype != MVLLM_DTYPE_BF16) ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send_x)) & 15u))
        return fail(MVLLM_ERR_INVALID, "ep_pack_dev: invalid arguments");
    if (T == 0)
        return MVLLM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int blocks = std::min(T, 65535);
    if (x_dtype == MVLLM_DTYPE_BF16)
        ep_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(x), idx, wt, T, K, D, E, nranks, dest, lid,
            self_rank, pos, static_cast<__nv_bfloat16 *>(send_x), send_idx, send_wt);
    else
        ep_pack_kernel<float><<<blocks, 256, 0, st>>>(
            static_cast<const float *>(x), idx, wt, T, K, D, E, nranks, dest, lid, self_rank, pos,
            static_cast<float *>(send_x), send_idx, send_wt);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_ep_combine16_dev(void *stream, const void *back16, const int *pos, int T,
                               int nranks, int D, float *out) {
    if (!pos || !out || T < 0 || nranks < 1 || nranks > 32 || D < 8 || D % 8 != 0 ||
        (!back16 && T > 0) ||
        ((reinterpret_cast<uintptr_t>(back16) | reinterpret_cast<uintptr_t>(out)) & 15u))
        return fail(MVLLM_ERR_INVALID, "ep_combine16_dev: invalid arguments");
    if (T == 0)
        return MVLLM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dim3 grid(std::max(1, std::min((D / 4 + 255) / 256, 8)), std::min(T, 65535));
    ep_combine16_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t *>(back16), pos, T,
                                               nranks, D, out);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_ep_combine_dev(void *stream, const float *back, const int *pos, int T, int nranks,
                             int D, float *out) {
    if (!pos || !out || T < 0 || nranks < 1 || nranks > 32 || D < 4 || D % 4 != 0 ||
        (!back && T > 0) ||
        ((reinterpret_cast<uintptr_t>(back) | reinterpret_cast<uintptr_t>(out)) & 15u))
        return fail(MVLLM_ERR_INVALID, "ep_combine_dev: invalid arguments");
    if (T == 0)
        return MVLLM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dim3 grid(std::max(1, std::min((D / 4 + 255) / 256, 8)), std::min(T, 65535));
    ep_combine_kernel<<<grid, 256, 0, st>>>(back, pos, T, nranks, D, out);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

// ------------------------------------ expert-parallel exchange over NVLink --
int mvllm_moe_peer_alloc(size_t bytes, void **ptr, void *handle) {
    if (!bytes || !ptr || !handle)
        return fail(MVLLM_ERR_INVALID, "peer_alloc: invalid arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == MVLLM_PEER_HANDLE_BYTES, "IPC handle size");
    Context &c = ctx();
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
    }
    void *p = nullptr;
    CUDA_TRY(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        cudaFree(p);
        return fail(MVLLM_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return MVLLM_OK;
}

int mvllm_moe_peer_open(const void *handle, void **ptr) {
    if (!handle || !ptr)
        return fail(MVLLM_ERR_INVALID, "peer_open: invalid arguments");
    Context &c = ctx();
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = p;
    return MVLLM_OK;
}

int mvllm_moe_peer_close(void *ptr) {
    if (!ptr)
        return fail(MVLLM_ERR_INVALID, "peer_close: null pointer");
    CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return MVLLM_OK;
}

int mvllm_moe_peer_free(void *ptr) {
    if (!ptr)
        return fail(MVLLM_ERR_INVALID, "peer_free: null pointer");
    CUDA_TRY(cudaFree(ptr));
    return MVLLM_OK;
}

static size_t dtype_size(int x_dtype) {
    return x_dtype == MVLLM_DTYPE_BF16 ? 2 : x_dtype == MVLLM_DTYPE_F32 ? 4 : 0;
}

size_t mvllm_moe_ep_window_layout(int nranks, int seg, int K, int D, int x_dtype,
                                  size_t *offsets) {
    if (nranks < 1 || nranks > 32 || seg < 1 || K < 1 || K > 16 || D < 8 || D % 8 != 0 ||
        !dtype_size(x_dtype))
        return 0;
    const WindowLayout w = ep_window_layout(nranks, seg, K, D, dtype_size(x_dtype));
    if (offsets) {
        offsets[0] = w.x;
        offsets[1] = w.ids;
        offsets[2] = w.wt;
        offsets[3] = w.back;
    }
    return w.total;
}

int mvllm_moe_ep_dispatch_peer_dev(void *stream, const void *x, int x_dtype, const int *idx,
                                   const float *wt, int T, int K, int D, int E, int nranks,
                                   const int *dest, const int *lid, int self_rank, int seg,
                                   const int *pos, const int *send_cnt, void *const *windows) {
    if (!x || !idx || !wt || !pos || !send_cnt || !windows || T < 0 || T > seg || K < 1 ||
        K > 16 || D < 8 || D % 8 != 0 || E < 1 || nranks < 1 || nranks > 32 || self_rank < 0 ||
        self_rank >= nranks || (!dest != !lid) || !dtype_size(x_dtype) ||
        (reinterpret_cast<uintptr_t>(x) & 15u))
        return fail(MVLLM_ERR_INVALID, "ep_dispatch_peer_dev: invalid arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const WindowLayout lay = ep_window_layout(nranks, seg, K, D, dtype_size(x_dtype));
    const int blocks = std::max(1, std::min(std::max(T, (nranks * seg * K + 255) / 256), 65535));
    uint8_t *const *win = reinterpret_cast<uint8_t *const *>(windows);
    if (x_dtype == MVLLM_DTYPE_BF16)
        ep_dispatch_peer_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(x), idx, wt, T, K, D, E, nranks, dest, lid,
            self_rank, seg, pos, send_cnt, win, lay);
    else
        ep_dispatch_peer_kernel<float><<<blocks, 256, 0, st>>>(
            static_cast<const float *>(x), idx, wt, T, K, D, E, nranks, dest, lid, self_rank,
            seg, pos, send_cnt, win, lay);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_moe_layer_partial_peer_dev(void *stream, int nranks, int seg, int self_rank, int K,
                                     int E, int D, int Iinter, int fmt, int x_dtype,
                                     void *window, void *const *windows, const void *const *g,
                                     const void *const *u, const void *const *d,
                                     const void *const *gs, const void *const *us,
                                     const void *const *ds, int act, float act_a, float act_b,
                                     void *workspace, size_t workspace_bytes) {
    if (nranks < 1 || nranks > 32 || seg < 1 || self_rank < 0 || self_rank >= nranks || K < 1 ||
        K > 16 || E < 1 || D < 8 || D % 8 != 0 || D > 32768 || Iinter < 1 ||
        (fmt != 0 && fmt != 4 && fmt != 7) || !dtype_size(x_dtype) || !window || !windows ||
        !g || !u || !d || (fmt != MVLLM_FMT_F32 && (!gs || !us || !ds)) ||
        (reinterpret_cast<uintptr_t>(window) & 255u))
        return fail(MVLLM_ERR_INVALID, "layer_partial_peer_dev: invalid arguments");
    const int T = nranks * seg;
    const size_t need = mvllm_moe_layer_workspace(T, K, E, 0, D, Iinter, fmt);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "layer_partial_peer_dev: workspace %zu < %zu",
                    workspace_bytes, need);
    Context &c = ctx();
    int sms;
    {
        std::lock_guard<std::mutex> lk(c.mu);
        if (int rc = ensure_current(c))
            return rc;
        sms = launch_sms(c);
    }
    const WindowLayout lay = ep_window_layout(nranks, seg, K, D, dtype_size(x_dtype));
    uint8_t *base = static_cast<uint8_t *>(window);
    Carve cv(workspace, workspace_bytes);
    LayerWs l{};
    carve_layer(cv, l, T, K, E, 0, D, Iinter, fast_path_ok(fmt, D, Iinter));
    Tables tb{g, u, d, gs, us, ds};
    LayerHooks hooks;
    hooks.peer = PeerRows{reinterpret_cast<uint8_t *const *>(windows), lay.back, seg, self_rank};
    return layer_dev_impl(static_cast<cudaStream_t>(stream), sms, T, K, E, 0, D, Iinter, fmt,
                          reinterpret_cast<const int *>(base + lay.ids),
                          reinterpret_cast<const float *>(base + lay.wt), base + lay.x, x_dtype,
                          tb, nullptr, act, act_a, act_b, l, true, &hooks, base + lay.back);
}

// ------------------------------------------------------------ packers etc --
int mvllm_quantize_int4_g64_dev(void *stream, const float *w, int O, int I, uint8_t *packed,
                                float *scales) {
    if (!w || O < 1 || I < 1 || !packed || !scales)
        return fail(MVLLM_ERR_INVALID, "quantize_int4_g64_dev: invalid arguments");
    Context &c = ctx();
    if (!c.inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    const size_t groups = size_t(O) * ((I + 63) / 64);
    const int blocks = int(std::min<size_t>((groups + 255) / 256, size_t(c.sms) * 16));
    quantize_int4_g64_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, O, I,
                                                                                  packed, scales);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_pack_mxfp4_dev(void *stream, const float *w, int O, int I, uint8_t *packed,
                         uint8_t *scales) {
    if (!w || O < 1 || I < 1 || !packed || !scales)
        return fail(MVLLM_ERR_INVALID, "pack_mxfp4_dev: invalid arguments");
    Context &c = ctx();
    if (!c.inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    const size_t groups = size_t(O) * ((I + 31) / 32);
    const int blocks = int(std::min<size_t>((groups + 255) / 256, size_t(c.sms) * 16));
    pack_mxfp4_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(w, O, I, packed,
                                                                           scales);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

int mvllm_matmul_dev(void *stream, int fmt, float *y, const float *x, const void *w,
                     const void *scales, int S, int I, int O) {
    if ((fmt != 0 && fmt != 4 && fmt != 7 && fmt != MVLLM_FMT_INT8_ROW &&
         fmt != MVLLM_FMT_FP8_B128) ||
        !y || !x || !w || S < 1 || I < 1 || O < 1 || (fmt != 0 && !scales))
        return fail(MVLLM_ERR_INVALID, "matmul_dev: invalid arguments");
    if (!ctx().inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    CUDA_TRY(matmul_generic_launch(static_cast<cudaStream_t>(stream), fmt, y, x, w, scales, S, I,
                                   O));
    return MVLLM_OK;
}

// ------------------------------------------------------------- epilogue --
size_t mvllm_moe_epilogue_workspace(int T, int H, int L) {
    if (T < 1 || H < 1 || L < 1)
        return 0;
    return (size_t(T) * L + size_t(T) * H) * sizeof(float) + 256;
}

int mvllm_moe_epilogue_dev(void *stream, int T, int H, int L, const float *acc,
                           const float *lat_n, float eps, int up_fmt, const void *up_w,
                           const void *up_scales, float routed_scale, const float *shared,
                           float *h, void *workspace, size_t workspace_bytes) {
    if (T < 1 || H < 1 || L < 1 || !acc || !h || (!up_w && L != H) ||
        (up_w && up_fmt != 0 && up_fmt != MVLLM_FMT_INT4_G64 && up_fmt != MVLLM_FMT_INT8_ROW) ||
        (up_w && up_fmt != 0 && !up_scales) ||
        (up_w && up_fmt == MVLLM_FMT_INT4_G64 && L % 64 != 0))
        return fail(MVLLM_ERR_INVALID, "epilogue_dev: invalid arguments");
    const size_t need = mvllm_moe_epilogue_workspace(T, H, L);
    if ((lat_n || up_w) && (!workspace || workspace_bytes < need))
        return fail(MVLLM_ERR_WORKSPACE, "epilogue_dev: workspace %zu < %zu", workspace_bytes,
                    need);
    Context &c = ctx();
    if (!c.inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!exact_mode()) {
        // Tolerance mode: one fused kernel (epilogue.cuh).
        EpiArgs ea{acc, lat_n, eps, static_cast<const int8_t *>(up_w),
                   static_cast<const float *>(up_scales), routed_scale, shared, h, T, H, L};
        const bool a16 = (reinterpret_cast<uintptr_t>(up_w) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(acc) & 15u) == 0 &&
                         (!lat_n || (reinterpret_cast<uintptr_t>(lat_n) & 15u) == 0);
        if (up_w && up_fmt == MVLLM_FMT_INT8_ROW && a16 && L % 64 == 0 && H % 16 == 0 &&
            epi_ksl(L) <= kEpiWarps && epi_smem_bytes(L) <= 227 * 1024 &&
            epi_ws_bytes(T, L) <= workspace_bytes) {
            const int ksl = epi_ksl(L), rb = kEpiWarps / ksl;
            const dim3 grid((H / 16 + rb - 1) / rb), block(kEpiWarps * 32);
            const size_t sm = epi_smem_bytes(L);
            __half *rows = static_cast<__half *>(workspace);
            float *tinv = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) +
                                                    size_t(T) * L * 2);
            CUDA_TRY(launch_pdl(epilogue_stage_kernel, dim3(std::min(T, 8 * c.sms)), dim3(256),
                                0, st, ea, rows, tinv));
            switch (ksl) {
#define MVB_EPI(K)                                                                           \
    case K:                                                                                  \
        CUDA_TRY(cudaFuncSetAttribute(epilogue_up_kernel<K>,                                \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm))); \
        CUDA_TRY(launch_pdl(epilogue_up_kernel<K>, grid, block, sm, st, ea,                  \
                            static_cast<const __half *>(rows), static_cast<const float *>(tinv))); \
        return MVLLM_OK;
                MVB_EPI(1)
                MVB_EPI(2)
                MVB_EPI(4)
                MVB_EPI(8)
                MVB_EPI(16)
#undef MVB_EPI
            default:
                break;
            }
        }
        const bool h16 = (reinterpret_cast<uintptr_t>(h) & 15u) == 0 &&
                         (!shared || (reinterpret_cast<uintptr_t>(shared) & 15u) == 0);
        if (!up_w && lat_n && a16 && h16 && H % 4 == 0) {
            CUDA_TRY(launch_pdl(epilogue_norm_kernel, dim3(std::min(T, 8 * c.sms)), dim3(256), 0,
                                st, ea));
            return MVLLM_OK;
        }
    }
    const float *src = acc;
    float *norm = static_cast<float *>(workspace);
    float *up = norm ? norm + size_t(T) * L : nullptr;
    if (lat_n) {
        const size_t sm = size_t(L) * sizeof(float);
        if (sm > 227 * 1024)
            return fail(MVLLM_ERR_INVALID, "epilogue_dev: latent width %d too large", L);
        if (sm > 48 * 1024)
            CUDA_TRY(cudaFuncSetAttribute(rmsnorm_rows_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
        rmsnorm_rows_kernel<<<std::min(T, 8 * c.sms), 256, sm, st>>>(acc, lat_n, norm, T, L, eps);
        CUDA_TRY(cudaGetLastError());
        src = norm;
    }
    if (up_w) {
        CUDA_TRY(matmul_generic_launch(st, up_fmt, up, src, up_w, up_scales, T, L, H));
        src = up;
    }
    const size_t n = size_t(T) * H;
    epilogue_residual_kernel<<<int(std::min<size_t>((n + 255) / 256, size_t(c.sms) * 16)), 256, 0,
                               st>>>(h, src, shared, routed_scale, n);
    CUDA_TRY(cudaGetLastError());
    return MVLLM_OK;
}

// ---------------------------------------------------- bounded-wait check --
// The failure path every pipeline kernel takes when a copy or a peer never
// completes: a wait on an mbarrier that one thread completes (must succeed),
// then on one that nothing completes (must give up after kWaitNs and record
// MVLLM_ERR_TIMEOUT).  The kernel returns either way; nothing faults.
__global__ void wait_selftest_kernel(int *err, int *result) {
    __shared__ uint64_t bar[2];
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        mbar_arrive(&bar[0]);
    const bool completed = mbar_wait(&bar[0], 0, nullptr);
    const bool never = mbar_wait(&bar[1], 0, err); // nothing arrives
    if (threadIdx.x == 0)
        result[0] = (completed ? 1 : 0) | (never ? 2 : 0);
}

int mvllm_moe_wait_selftest(int *completed, int *timed_out) {
    Context &c = ctx();
    std::lock_guard<std::mutex> lk(c.mu);
    if (int rc = ensure_current(c))
        return rc;
    int *d = nullptr;
    CUDA_TRY(cudaMalloc(&d, 2 * sizeof(int)));
    int h[2] = {0, 0};
    cudaError_t e = cudaMemsetAsync(d, 0, 2 * sizeof(int), c.stream);
    if (e == cudaSuccess) {
        wait_selftest_kernel<<<1, 64, 0, c.stream>>>(d, d + 1);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(c.stream);
    cudaFree(d);
    if (e != cudaSuccess)
        return fail(MVLLM_ERR_CUDA, "wait_selftest: %s", cudaGetErrorString(e));
    if (completed)
        *completed = h[1] & 1;
    if (timed_out)
        *timed_out = h[0] == MVLLM_ERR_TIMEOUT && !(h[1] & 2);
    return MVLLM_OK;
}

// ------------------------------------------------------------- dense FFN --
size_t mvllm_moe_dense_ffn_workspace(int T, int H, int O) {
    if (T < 1 || H < 1 || O < 1)
        return 0;
    return (2 * size_t(T) * O + size_t(T) * H) * sizeof(float) + 256;
}

int mvllm_moe_dense_ffn_dev(void *stream, int fmt, int T, int H, int O, const void *gate_w,
                            const void *gate_s, const void *up_w, const void *up_s,
                            const void *down_w, const void *down_s, const float *x, int act,
                            float act_a, float act_b, float *y, int accumulate, void *workspace,
                            size_t workspace_bytes) {
    const bool scaled = fmt != MVLLM_FMT_F32;
    if (T < 1 || H < 1 || O < 1 || !x || !y || !gate_w || !up_w || !down_w ||
        (fmt != MVLLM_FMT_F32 && fmt != MVLLM_FMT_INT4_G64 && fmt != MVLLM_FMT_INT8_ROW &&
         fmt != MVLLM_FMT_FP8_B128) ||
        (scaled && (!gate_s || !up_s || !down_s)))
        return fail(MVLLM_ERR_INVALID, "dense_ffn_dev: invalid arguments");
    const size_t need = mvllm_moe_dense_ffn_workspace(T, H, O);
    if (!workspace || workspace_bytes < need)
        return fail(MVLLM_ERR_WORKSPACE, "dense_ffn_dev: workspace %zu < %zu", workspace_bytes,
                    need);
    Context &c = ctx();
    if (!c.inited)
        return fail(MVLLM_ERR_NOT_INIT, "mvllm_moe_init has not been called");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *g = static_cast<float *>(workspace);
    float *u = g + size_t(T) * O;
    float *d = u + size_t(T) * O;
    const MmOut gu{{g, u}, {gate_w, up_w}, {gate_s, up_s}};
    CUDA_TRY(matmul_generic_launch(st, fmt, gu, 2, x, T, H, O));
    const size_t nh = size_t(T) * O;
    dense_act_kernel<<<int(std::min<size_t>((nh + 255) / 256, size_t(c.sms) * 16)), 256, 0, st>>>(
        g, u, nh, act, act_a, act_b);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(matmul_generic_launch(st, fmt, accumulate ? d : y, g, down_w, down_s, T, O, H));
    if (accumulate) {
        const size_t ny = size_t(T) * H;
        add_rows_kernel<<<int(std::min<size_t>((ny + 255) / 256, size_t(c.sms) * 16)), 256, 0,
                          st>>>(y, d, ny);
        CUDA_TRY(cudaGetLastError());
    }
    return MVLLM_OK;
}

// ------------------------------------------------------------- profiling --
void mvllm_moe_profile_enable(int on) {
    Prof &p = prof();
    std::lock_guard<std::mutex> lk(p.mu);
    p.on = on != 0;
    p.marks.clear();
    p.used = 0;
}

int mvllm_moe_profile_read(double *ms, long long *launches, int n) {
    Prof &p = prof();
    std::lock_guard<std::mutex> lk(p.mu);
    for (int i = 0; i < n; ++i) {
        if (ms)
            ms[i] = 0.0;
        if (launches)
            launches[i] = 0;
    }
    if (!p.marks.empty())
        CUDA_TRY(cudaEventSynchronize(p.marks.back().first));
    for (size_t i = 1; i < p.marks.size(); ++i) {
        const int ph = p.marks[i].second;
        if (ph < 0 || ph >= n) // an interval ending at a call start spans host time
            continue;
        float t = 0.f;
        if (cudaEventElapsedTime(&t, p.marks[i - 1].first, p.marks[i].first) != cudaSuccess)
            continue;
        if (ms)
            ms[ph] += t;
        if (launches)
            launches[ph] += 1;
    }
    p.marks.clear();
    p.used = 0;
    return kPhCount;
}

} // extern "C"
