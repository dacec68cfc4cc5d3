/*
 * mvllm_moe.h -- C ABI of the B200 (sm_100a) routed-expert MoE block.
 *
 * Drop-in for micro-vllm's expert compute tier.  The reference reaches its
 * expert GEMMs through mvllm::metal_ops::moe_block (src/gpu/metal_ops.hpp:
 * 99-108) and, as a fallback, the coli_cuda tier (src/gpu/coli_cuda.hpp,
 * whose only device hook is extern "C" coli_cuda_gemm_f32_dev,
 * src/gpu/coli_cuda.cu:22-34).  This header replaces both with plain C entry
 * points: plain pointers and sizes, int status codes, no C++ or torch types.
 * include/mvllm_metal_ops.hpp puts the reference's exact C++ signature on
 * top of mvllm_moe_block so reference call sites link unchanged.
 *
 * Error convention (as the reference tiers: "returns false on bad args; never
 * throws", src/gpu/coli_cuda.hpp:13): every entry returns MVLLM_OK (0) or a
 * positive code and never aborts.  MVLLM_ERR_INVALID is exactly the set of
 * argument checks for which the reference moe_block returns false.
 *
 * Formats (src/quant/quant.hpp):
 *   fmt 0  f32 row-major [O, I]
 *   fmt 4  int4-g64: packed uint8 [O, ceil(I/2)] (low nibble = even column,
 *          value = nibble - 8), f32 scales [O, ceil(I/64)]
 *   fmt 7  MXFP4: packed e2m1 uint8 [O, ceil(I/2)] (bit 3 = sign), ue8m0
 *          scales uint8 [O, ceil(I/32)], passed through the float* slots
 *   fmt 8  int8 rows: int8 [O, I], one f32 scale per row (QuantMat 8-bit)
 *   fmt 9  FP8 tiles: e4m3fn uint8 [O, I], ue8m0 scales uint8
 *          [ceil(O/128), ceil(I/128)] (DeepSeek-V4)
 * moe_block and the layer entries take fmt 4 and 7 (and 0 on the generic
 * path); the dense entries (matmul, epilogue, dense FFN) also 8 and 9.
 * Gate/up weights are [Iinter, D]; down weights are [D, Iinter].
 */
#ifndef MVLLM_MOE_H
#define MVLLM_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MVLLM_API __attribute__((visibility("default")))
#else
#define MVLLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MVLLM_OK = 0,
    MVLLM_ERR_INVALID = 1,     /* argument rejected (reference: returns false) */
    MVLLM_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
    MVLLM_ERR_NOMEM = 3,       /* device or pinned allocation failed */
    MVLLM_ERR_UNSUPPORTED = 4, /* shape/format the requested entry cannot run */
    MVLLM_ERR_TIMEOUT = 5,     /* a bounded device-side wait ran out */
    MVLLM_ERR_NOT_INIT = 6,    /* mvllm_moe_init has not succeeded */
    MVLLM_ERR_DEVICE = 7,      /* a device-side bounds check rejected an index */
    MVLLM_ERR_WORKSPACE = 8,   /* caller workspace smaller than required */
    MVLLM_ERR_RANGE = 9,       /* an MXFP4 scale code the tensor-core operands cannot
                                  represent as the reference decodes it (f16 mode: 141..254;
                                  block-scaled modes: 255, which the MMA reads as NaN, not
                                  +inf).  Not returned by the layer and moe_block entries:
                                  their tensor-core kernels raise a redo word and the decode
                                  kernels recompute the call's tensor-core experts on the
                                  device, in the same call */
    MVLLM_ERR_ACT_RANGE = 10   /* a finite activation (a token row of x, h = act(gate, up),
                                  or an expert's output row y before its routing weight)
                                  beyond the f16 range (|v| >= 65520): the reference computes
                                  it in f32; this library refuses the call instead of
                                  returning inf */
};

/* How experts on the tensor-core path (prefill-sized calls) compute with
 * MXFP4 weights.  No counterpart in the reference (its matmul_mxfp4,
 * src/quant/quant.cpp:298-321, is f32 throughout).  Errors measured on B200
 * over all 4096 tokens of the config[3] layer against an f64 evaluation
 * (relative L2 / max-abs; the tolerance is 1e-2 / 2e-2):
 *   F16      weights dequantised to f16 in tensor memory, tokens f16
 *            (kind::f16): 2e-4 / 1.6e-3.
 *   MXF4_Xn  weights used as they are (e2m1 + ue8m0 per 32, kind::mxf4 with
 *            the block scales in tensor memory); tokens as n block-scaled
 *            e2m1 terms, each quantising the previous terms' residual:
 *            n = 1 2.2e-1 / 1.5, n = 2 2.8e-2 / 1.9e-1, n = 3 2.7e-3 /
 *            1.9e-2 (within tolerance, max-abs at 94% of the bar).
 *   MXF8_Xn  weights as they are (kind::mxf8f6f4, e2m1 x e4m3); tokens as n
 *            e4m3 terms: n = 1 4.7e-2 / 3.5e-1, n = 2 7e-4 / 5.7e-3.
 * The default is the fastest mode within tolerance on that measurement (F16);
 * MVLLM_PREFILL_MODE (f16, mxf4x1, mxf4x2, mxf4x3, mxf8x1, mxf8x2) or
 * mvllm_moe_set_prefill_mode selects another. */
enum {
    MVLLM_PREFILL_F16 = 0,
    MVLLM_PREFILL_MXF4_X1 = 1,
    MVLLM_PREFILL_MXF4_X2 = 2,
    MVLLM_PREFILL_MXF4_X3 = 3,
    MVLLM_PREFILL_MXF8_X1 = 4,
    MVLLM_PREFILL_MXF8_X2 = 5
};
#define MVLLM_PREFILL_DEFAULT MVLLM_PREFILL_F16

/* metal_ops::Act (src/gpu/metal_ops.hpp:44); any other value behaves as SILU. */
enum { MVLLM_ACT_SILU = 0, MVLLM_ACT_CLAMP_SWIGLU = 1, MVLLM_ACT_SITU = 2 };
enum { MVLLM_FMT_F32 = 0, MVLLM_FMT_INT4_G64 = 4, MVLLM_FMT_MXFP4 = 7 };
/* int8 with one f32 scale per row: QuantMat fmt 8 (src/quant/weight.cpp:37-40,
 * quant.cpp:230-268); accepted by mvllm_matmul_dev and the layer epilogue. */
enum { MVLLM_FMT_INT8_ROW = 8 };
/* e4m3fn bytes [O, I] with one ue8m0 scale byte per 128 x 128 tile, scales
 * [ceil(O/128), ceil(I/128)]: DeepSeek-V4's FP8 tensors (dsv4_cuda.hpp:45-46,
 * dequant dsv4_cuda.cpp:127-135).  Accepted by mvllm_matmul_dev and
 * mvllm_moe_dense_ffn_dev. */
enum { MVLLM_FMT_FP8_B128 = 9 };
enum { MVLLM_DTYPE_F32 = 0, MVLLM_DTYPE_BF16 = 1 };
/* Router score functions: sigmoid (GLM, Kimi K3: quant.hpp:22-29) and
 * sqrt(softplus) (DeepSeek-V4: dsv4_cuda.cpp:26-34). */
enum { MVLLM_SCORE_SIGMOID = 0, MVLLM_SCORE_SQRT_SOFTPLUS = 1 };

/* ---- lifecycle: metal_ops::init/shutdown/available/backend_name
 *      (src/gpu/metal_ops.hpp:15-18); coli_cuda::init (coli_cuda.hpp:25) ---- */
MVLLM_API int mvllm_moe_init(int device);
MVLLM_API void mvllm_moe_shutdown(void);
MVLLM_API int mvllm_moe_available(void);
MVLLM_API const char *mvllm_moe_backend_name(void); /* "cuda-sm100a" */
MVLLM_API const char *mvllm_moe_last_error(void);   /* text of the last failure in this process */
/* Process-wide prefill mode (MVLLM_PREFILL_*, or -1 for the default /
 * MVLLM_PREFILL_MODE); MVLLM_ERR_INVALID otherwise.  get returns the mode in
 * effect. */
MVLLM_API int mvllm_moe_set_prefill_mode(int mode);
MVLLM_API int mvllm_moe_get_prefill_mode(void);
/* Process-wide exact mode: 1 = the layer epilogue (mvllm_moe_epilogue_dev)
 * and the router scores (mvllm_moe_route_dev / _route_ex_dev) keep the
 * reference's summation order and roundings (bit-identical to its CPU
 * functions, serial sums); 0 = tolerance-mode kernels (fused multiply-adds,
 * tensor cores, reassociated sums: within 1e-2 relative L2 / 2e-2 max-abs of
 * the reference, run-to-run identical); -1 = the default, 0 unless the
 * environment sets MVLLM_EXACT=1.  get returns the mode in effect. */
MVLLM_API int mvllm_moe_set_exact(int on);
MVLLM_API int mvllm_moe_get_exact(void);
/* SMs the layer's persistent expert kernels fill (0: all, the default).  No
 * counterpart in the reference: a caller that overlaps an NCCL exchange on
 * another stream with the expert kernels (the chunked expert-parallel step)
 * leaves it SMs.  Process-wide; takes effect at the next launch. */
MVLLM_API int mvllm_moe_set_sm_limit(int sms);
/* The block-scaled modes' token operand, on its own (no counterpart in the
 * reference): f16 rows src [rows, K] (K % 32 == 0) as the mode's n terms,
 * planes [n][rows][K/2] packed e2m1 (low nibble = even element; MXF4 modes)
 * or [n][rows][K] e4m3 (MXF8 modes) and ue8m0 codes [n][rows][K/32].  Term t
 * holds round(r_t / 2^(c-127)) of the residual r_t the earlier terms left,
 * c the smallest code with 2^(c-127) >= max|r_t| / 6 (e2m1) or / 448 (e4m3)
 * over each 32 elements; a block of zeros gets code 0. */
/* The tensor pipe's own rate (no counterpart in the reference): `iters`
 * back-to-back MMAs of M = 128 (pair = 0) or 256 (pair = 1, CTA pairs) by n
 * tokens on every SM, kind 0 = mxf4 (K 64), 1 = mxf8f6f4 (K 32), 2 = f16
 * (K 16, single CTAs only); *tflops = dense TFLOP/s from CUDA events.  The
 * denominator of the prefill path's tensor fraction.  Synchronous. */
MVLLM_API int mvllm_moe_mma_rate(int kind, int n, int pair, int iters, double *tflops);
MVLLM_API int mvllm_mx_terms_dev(void *stream, int mode, const void *src, int rows, int K,
                                 void *planes, void *codes);

/* coli_cuda::group_stats (src/gpu/coli_cuda.hpp:35-36): calls, experts, rows
 * and host-timed h2d / kernel / d2h milliseconds of the host-pointer entries.
 * h2d counts the copies before the first expert kernel starts; copies that
 * overlap the kernels (mvllm_moe_block's tail of a two-part activation
 * upload) count as kernel time. */
MVLLM_API void mvllm_moe_stats(uint64_t *calls, uint64_t *experts, uint64_t *rows, double *h2d_ms,
                     double *kernel_ms, double *d2h_ms);

/* ---- the hot path, host pointers: metal_ops::moe_block
 *      (src/gpu/metal_ops.hpp:104-108, body src/gpu/metal_ops.cpp:278-342) --
 * For expert e in call order with nr[e] > 0: rows xg[xoff[e] .. +nr[e]) of D
 * floats; hh = down(act(gate, up)); out[rows[base+r]] += rw[base+r] * hh[r]
 * (skipped when the destination is < 0 or >= S with S > 0).  base advances by
 * nr[e] for every expert with nr[e] > 0, also ones skipped for null weights.
 * `out` is accumulated into.  qgs is ignored (group sizes are fixed by fmt).
 * All pointers are caller-owned host memory, borrowed for the call.  Weight
 * and scale arrays inside a range given to mvllm_moe_cache_register are read
 * from the device copy; any other array is uploaded for this call only.
 * Synchronous: returns after `out` holds the result. */
MVLLM_API int mvllm_moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
                    const void *const *u, const void *const *d, const float *const *gs,
                    const float *const *us, const float *const *ds, const float *xg,
                    const int *xoff, const int *nr, const int *rows, const float *rw, float *out,
                    int S, int act, float act_a, float act_b);

/* ---- device-resident expert cache (mirrors an ExpertStore slot,
 *      src/store/expert_store.hpp:71-175; the host pointer of a pinned slot
 *      is the key, `generation` must change whenever the slot is refilled,
 *      e.g. on the REPIN events of src/store/expert_store.cpp:306-316) ---- */
MVLLM_API int mvllm_moe_cache_register(const void *host, size_t bytes, uint64_t generation);
MVLLM_API int mvllm_moe_cache_unregister(const void *host);
MVLLM_API void mvllm_moe_cache_clear(void);
MVLLM_API size_t mvllm_moe_cache_bytes(void);

/* Page-locks a caller buffer (cudaHostRegister) for the host-pointer entries:
 * mvllm_moe_layer_host copies x and out that lie inside registered buffers
 * straight to and from the device instead of through its pinned staging
 * copy.  The buffer must stay allocated until mvllm_moe_host_unregister (or
 * mvllm_moe_shutdown).  Registered buffers may not overlap. */
MVLLM_API int mvllm_moe_host_register(void *host, size_t bytes);
MVLLM_API int mvllm_moe_host_unregister(void *host);

/* ---- device expert tier: the VRAM level above an ExpertStore
 *      (src/store/expert_store.hpp:59-175, expert_store.cpp:273-405).
 *      A budget of equal VRAM slots holds copies of bound host blobs, least
 *      recently used out first.  mvllm_moe_block finds its weight arrays in
 *      bound blobs: resident ones are read from their slot; cold ones are
 *      copied into a slot on a second stream while the call's resident
 *      experts compute, then run.  Explicit cache_register ranges take
 *      precedence; arrays in no bound blob are uploaded for the call. ---- */
/* budget_bytes / slot_bytes slots (slot_bytes rounded up to 256); a budget
 * below one slot turns the tier off.  Drops every residency (bindings stay). */
MVLLM_API int mvllm_moe_tier_configure(size_t budget_bytes, size_t slot_bytes);
/* Binds a host blob (an ExpertStore slot: start, bytes, generation).  A new
 * generation or size for the same start drops the stale device copy; a blob
 * overlapping an older binding replaces it.  No copy is made until a call
 * uses the blob.  Blobs larger than a slot stay per-call uploads. */
MVLLM_API int mvllm_moe_expert_bind(const void *host_blob, size_t bytes, uint64_t generation);
MVLLM_API int mvllm_moe_expert_unbind(const void *host_blob);
/* Counters since init: blob acquisitions that found the blob resident
 * (hits), that copied it in (misses), slots taken from another blob
 * (evictions), bytes copied in, acquisitions that found no slot (overflow:
 * every slot held by a blob the call uses, or the blob too large) and their
 * bytes (uploaded for the call only); and the bytes now resident. */
MVLLM_API void mvllm_moe_tier_stats(uint64_t *hits, uint64_t *misses, uint64_t *evictions,
                                    uint64_t *bytes_in, uint64_t *overflow,
                                    uint64_t *overflow_bytes, size_t *resident_bytes);

/* ---- device-pointer entries (stream-ordered, no host sync, no allocation:
 *      the caller passes a workspace of at least the *_workspace size) ---- */

/* moe_block on device memory.  g,u,d,gs,us,ds are DEVICE arrays of nb device
 * pointers; xoff, nr [nb], rows, rw [rows_cap] and x (rows of D elements,
 * dtype MVLLM_DTYPE_*) are device arrays; out is device f32 [S, D].  S must be
 * > 0.  rows_cap bounds sum(max(nr,0)); x_rows bounds max(xoff+nr) (the rows
 * of x that may be read).  Same semantics as mvllm_moe_block. */
MVLLM_API size_t mvllm_moe_block_dev_workspace(int nb, int D, int Iinter, int fmt, int rows_cap, int x_rows,
                                     int S);
MVLLM_API int mvllm_moe_block_dev(void *stream, int nb, int D, int Iinter, int fmt, const void *const *g,
                        const void *const *u, const void *const *d, const void *const *gs,
                        const void *const *us, const void *const *ds, const void *x, int x_dtype,
                        int x_rows, const int *xoff, const int *nr, const int *rows,
                        const float *rw, float *out, int S, int act, float act_a, float act_b,
                        int rows_cap, void *workspace, size_t workspace_bytes);

/* Token permutation of the callers (src/model/glm53.cpp:1958-1971,
 * src/model/kimi_k3.cpp:2036-2050): from top-k ids idx[T,K] and weights
 * wt[T,K] (device), for each expert in ascending id the tokens c ascending
 * whose wsum = sum_t wt[c,t]*[idx[c,t]==e] (t ascending, f32) is non-zero.
 * Writes nr[E+n_shared], xoff[E+n_shared] (segment starts), rows[R] (token
 * ids), rw[R] (wsums) and tok_pos[T, K+n_shared] (segment position of each
 * token's entry, -1 where none).  n_shared = 1 appends an always-on expert
 * (id E, weight 1 for every token) after the routed ones.  Ids outside
 * [0, E) are ignored (the reference union drops ids < 0).  *n_rows (device
 * int) receives R. */
MVLLM_API size_t mvllm_moe_permute_workspace(int T, int K, int E, int n_shared);
MVLLM_API int mvllm_moe_permute_dev(void *stream, const int *idx, const float *wt, int T, int K, int E,
                          int n_shared, int *nr, int *xoff, int *rows, float *rw, int *tok_pos,
                          int *n_rows, void *workspace, size_t workspace_bytes);

/* The permutation above with no workspace argument and no allocation at
 * all.  No counterpart in the reference: it exists for callers that cannot
 * allocate device memory when they need the permutation -- engines that fix
 * their HBM budget at start-up and forbid allocation in the serving loop, and
 * plugins living in a host process whose own allocator owns the GPU's memory
 * (a cudaMalloc behind its back would take memory it has promised
 * elsewhere).  The scratch (bitmap and per-token weight sums) is a
 * file-scope __device__ array of MVLLM_PERMUTE_STATIC_BYTES that every GPU
 * loading the library keeps until the process exits.  Sizes whose scratch
 * exceeds it are rejected with MVLLM_ERR_WORKSPACE before any launch: the
 * scratch is mvllm_moe_permute_workspace() minus its 256 bytes of alignment
 * slack, so T=8192, K=8, E=384, n_shared=0 (exactly 1 MiB) fits and T=8193
 * does not.  The first call on a device looks up the array's device address
 * (once per device, with that device current); make that first call before
 * any stream capture.  All calls share the one array, which keeps the last
 * call's contents (each call clears what must start at zero): calls whose
 * executions overlap on the GPU race.  Outputs, ordering and error codes are
 * those of mvllm_moe_permute_dev; does not require mvllm_moe_init. */
#define MVLLM_PERMUTE_STATIC_BYTES (1u << 20)
MVLLM_API int mvllm_moe_permute_dev_noalloc(void *stream, const int *idx, const float *wt, int T,
                                            int K, int E, int n_shared, int *nr, int *xoff,
                                            int *rows, float *rw, int *tok_pos, int *n_rows);

/* A whole routed MoE layer on device, as moe_layer_n's routed part
 * (src/model/glm53.cpp:1936-1994, src/model/kimi_k3.cpp:2024-2075) plus an
 * optional always-on shared expert: permute -> expert FFN -> ordered combine
 * out[c] += sum over the token's experts in ascending id of wsum * hh.
 * x is device [T, D] (dtype MVLLM_DTYPE_*); g..ds are device arrays of
 * E + n_shared device pointers (the shared expert last); out is device f32
 * [T, D], accumulated. */
MVLLM_API size_t mvllm_moe_layer_workspace(int T, int K, int E, int n_shared, int D, int Iinter, int fmt);
MVLLM_API int mvllm_moe_layer_dev(void *stream, int T, int K, int E, int n_shared, int D, int Iinter,
                        int fmt, const int *idx, const float *wt, const void *x, int x_dtype,
                        const void *const *g, const void *const *u, const void *const *d,
                        const void *const *gs, const void *const *us, const void *const *ds,
                        float *out, int act, float act_a, float act_b, void *workspace,
                        size_t workspace_bytes);
/* Device-side errors of mvllm_moe_layer_dev / _layer_partial_dev (an
 * activation beyond the f16 range, a skipped misaligned or out-of-range
 * expert, a bounded wait that ran out) are recorded in the call's workspace
 * instead of being returned (the call does not synchronise): `out` is then
 * left as the caller passed it (partial rows: zero rows).  This synchronises
 * `stream` and returns the code of the last call that used `workspace`
 * (MVLLM_OK when none). */
MVLLM_API int mvllm_moe_layer_error(void *stream, const void *workspace);

/* The same layer with HOST buffers (x f32 [T,D], idx/wt [T,K], out f32
 * [T,D] accumulated) and weights already resident on the device: the
 * end-to-end entry.  Copies in, runs, copies out, synchronises. */
MVLLM_API int mvllm_moe_layer_host(int T, int K, int E, int n_shared, int D, int Iinter, int fmt,
                         const int *idx, const float *wt, const float *x, const void *const *g,
                         const void *const *u, const void *const *d, const void *const *gs,
                         const void *const *us, const void *const *ds, float *out, int act,
                         float act_a, float act_b);

/* ---- weight preparation on the device, bit-identical to
 *      quant::quantize_int4_g64 (src/quant/quant.cpp:170-201) and
 *      quant::pack_mxfp4 (src/quant/quant.cpp:270-296).  w is device f32
 *      [O, I]; outputs as the formats above. ---- */
MVLLM_API int mvllm_quantize_int4_g64_dev(void *stream, const float *w, int O, int I, uint8_t *packed,
                                float *scales);
MVLLM_API int mvllm_pack_mxfp4_dev(void *stream, const float *w, int O, int I, uint8_t *packed,
                         uint8_t *scales);

/* Dequantised GEMM y[S,O] = x[S,I] . W[O,I]^T on device (f32 in/out): the
 * role of coli_cuda::matmul / matmul_mxfp4 (src/gpu/coli_cuda.hpp:58-61) and
 * quant::matmul_* (src/quant/quant.hpp:53-70).  fmt 0, 4, 7 or 8 (int8 rows:
 * y = (sum x.q) x scale[o], quant.cpp:255-268), or 9 (FP8 tiles: the sum of
 * x[i] * (e4m3fn(q) * 2^(s-127)), dsv4_cuda.cpp:618-623).  Each weight row is
 * read once for up to 32 rows of x. */
MVLLM_API int mvllm_matmul_dev(void *stream, int fmt, float *y, const float *x, const void *w,
                     const void *scales, int S, int I, int O);

/* ---- routing on the device (glm53.cpp:1921-1931, kimi_k3.cpp:1986-1998). ----
 * moe_topk for T rows of choice [T, E] (device): the K largest choices, equal
 * values to the lower expert id, in that order; w = mix[id] (or choice[id] when
 * mix is null) clamped at 0, divided by their sum in selection order, or 1/K
 * each when the sum is 0 (ops.cpp:860-890).  K > E fills the tail with -1 / 0.
 * E <= 1024, K <= 32.  Bit-identical to the reference's moe_topk. */
MVLLM_API int mvllm_moe_topk_dev(void *stream, const float *choice, const float *mix, int T, int E,
                                 int K, int *idx, float *wt);
/* The router in front of it: scores[t, e] = sigmoid(x[t] . router[e]) with the
 * dot product in the reference's order (sequential f32 over H, product and sum
 * rounded separately, quant.cpp:156-168), choice = scores + bias (bias may be
 * null), then mvllm_moe_topk_dev(choice, mix = scores).  x: x_dtype [T, H];
 * router f32 [E, H]; scores, choice: f32 [T, E] outputs. */
MVLLM_API int mvllm_moe_route_dev(void *stream, const void *x, int x_dtype, int T, int H,
                                  const float *router, const float *bias, int E, int K, int *idx,
                                  float *wt, float *scores, float *choice);
/* The same with the score function chosen (MVLLM_SCORE_*) and every weight
 * multiplied by routed_scale at the end.  score_fn MVLLM_SCORE_SQRT_SOFTPLUS,
 * K 6 is DeepSeek-V4's dsv4_cuda::route (dsv4_cuda.cpp:1541-1587, without
 * fixed ids): choice = sqrt(softplus(logit)) + bias, the top min(6, E),
 * w = score / sum * routed_scale.  mvllm_moe_route_dev is score_fn
 * MVLLM_SCORE_SIGMOID with routed_scale 1. */
MVLLM_API int mvllm_moe_route_ex_dev(void *stream, const void *x, int x_dtype, int T, int H,
                                     const float *router, const float *bias, int E, int K,
                                     int score_fn, float routed_scale, int *idx, float *wt,
                                     float *scores, float *choice);

/* ---- expert parallelism (one rank per GPU).  No single counterpart in the
 *      reference, which runs every expert on one host; these are the
 *      device steps of the sharded layer around the NCCL exchanges.
 *      Placement: dest, lid (device int32 [E], both given or both NULL).
 *      dest[e] = the rank that serves expert e, or -1 for a replicated
 *      expert that every rank holds and serves for its own tokens;
 *      lid[e] = e's local id on the rank that serves it.  NULL: strided,
 *      expert e on rank e % nranks as local expert e / nranks.  dest
 *      entries must lie in [-1, nranks). ---- */
/* Dispatch plan for the T tokens of rank self_rank (idx [T,K] device, global
 * ids; ids outside [0, E) ignored): pos[T, nranks] = row of token c in the
 * destination-major send buffer for rank d (tokens ascending within a rank),
 * or -1 when rank d serves none of c's experts; send_cnt[nranks] = rows per
 * destination.  nranks <= 32. */
MVLLM_API int mvllm_moe_ep_plan_dev(void *stream, const int *idx, int T, int K, int E, int nranks,
                                    const int *dest, int self_rank, int *pos, int *send_cnt);
/* The plan with fixed-size send segments (no counterpart in the reference):
 * destination d's rows start at d * capacity (capacity >= T: a token goes to
 * a rank at most once), so every rank sends and receives nranks * capacity
 * rows and the exchange needs no counts on the host.  Rows of a segment past
 * send_cnt[d] carry no token: the caller sets their send_idx to -1. */
MVLLM_API int mvllm_moe_ep_plan_fixed_dev(void *stream, const int *idx, int T, int K, int E,
                                          int nranks, const int *dest, int self_rank,
                                          int capacity, int *pos, int *send_cnt);
/* Fills the send buffer from the plan: send_x[p] = x[c] (x_dtype rows of D,
 * D a multiple of 8), send_idx[p, k] = local id of idx[c, k] when rank d
 * serves it else -1, send_wt[p, k] = wt[c, k]. */
MVLLM_API int mvllm_moe_ep_pack_dev(void *stream, const void *x, int x_dtype, const int *idx,
                                    const float *wt, int T, int K, int D, int E, int nranks,
                                    const int *dest, const int *lid, int self_rank,
                                    const int *pos, void *send_x, int *send_idx, float *send_wt);
/* Expert parallelism without a token exchange, DeepSeek-V4's EP2
 * (route_moe_ep2, dsv4_cuda.cpp:1841-1906; map_ep_expert :1356-1369): every
 * rank sees all T tokens, serves its own experts and the ranks' partial
 * outputs are summed (allreduce_pair, :1195-1204; NCCL all-reduce here).
 * local_idx[T, K] = the local id of idx[t, k] when rank self_rank serves it,
 * else -1.  Placement as above, except that each expert has exactly one
 * serving rank (every rank holds all tokens, so a replicated expert would
 * count once per rank; dest entries of -1 serve no rank).  Strided with
 * nranks 2 is the reference's parity split, expert e on rank e % 2 as e / 2.
 * The result feeds mvllm_moe_layer_dev with the rank's expert tables. */
MVLLM_API int mvllm_moe_ep_local_ids_dev(void *stream, const int *idx, int T, int K, int E,
                                         int nranks, const int *dest, const int *lid,
                                         int self_rank, int *local_idx);
/* out[c] += back[pos[c, d]] for d = 0, 1, ... (f32 rows of D, D a multiple of 4):
 * the partial sums each rank returned, added in ascending rank order. */
MVLLM_API int mvllm_moe_ep_combine_dev(void *stream, const float *back, const int *pos, int T,
                                       int nranks, int D, float *out);
/* The same from partial rows in the form mvllm_moe_layer_partial_dev writes
 * (pitch 2*D + 16 bytes: D f16 values, then the row's f32 power-of-two scale):
 * out[c] += f16 value x scale, ranks ascending.  D a multiple of 8. */
MVLLM_API int mvllm_moe_ep_combine16_dev(void *stream, const void *back16, const int *pos,
                                         int T, int nranks, int D, float *out);
/* ---- the exchange over peer memory (no counterpart in the reference, whose
 *      experts all run on one host): each rank owns one exchange window that
 *      the other ranks map through CUDA IPC and write over NVLink, so the
 *      dispatch and the return are stores inside the producing kernels and
 *      no NCCL transfer carries rows.  Window of rank r, nranks * seg rows
 *      (seg = tokens per rank per step; rank s's rows for r are rows
 *      s*seg .. s*seg + seg - 1), regions at the offsets of
 *      mvllm_moe_ep_window_layout:
 *        [0] x    [nranks*seg, D] token rows received (x_dtype)
 *        [1] ids  [nranks*seg, K] int32 local expert ids, -1 = no slot here
 *        [2] wt   [nranks*seg, K] f32 routing weights
 *        [3] back [nranks*seg, 2*D + 16] partial rows returned to rank r:
 *            row d*seg + j = rank d's partial sum of r's token that the
 *            fixed plan put at row d*seg + j (pos[c, d]), so
 *            mvllm_moe_ep_combine16_dev(back, pos, ...) adds them.
 *      A step: ep_plan_fixed_dev (capacity = seg), ep_dispatch_peer_dev,
 *      a barrier over the ranks, layer_partial_peer_dev, a barrier,
 *      ep_combine16_dev.  The barriers must order every rank's preceding
 *      kernels before every rank's following ones (a stream-ordered
 *      collective such as an NCCL all-reduce of one word does).  One
 *      window serves every step: a rank writes into a peer's window only
 *      after a barrier that the peer enters once it has finished reading. */
#define MVLLM_PEER_HANDLE_BYTES 64
/* cudaMalloc'd window of `bytes` (zeroed) and its IPC handle (64 bytes) for
 * the other processes' mvllm_moe_peer_open. */
MVLLM_API int mvllm_moe_peer_alloc(size_t bytes, void **ptr, void *handle);
/* Maps another process's window (peer access enabled on first use). */
MVLLM_API int mvllm_moe_peer_open(const void *handle, void **ptr);
MVLLM_API int mvllm_moe_peer_close(void *ptr);
MVLLM_API int mvllm_moe_peer_free(void *ptr);
/* Window bytes (0 for invalid arguments) and, if offsets is not NULL, the
 * byte offsets of its four regions (x, ids, wt, back), each 256-aligned.
 * nranks <= 32, K <= 16, D a multiple of 8, x_dtype F32 or BF16. */
MVLLM_API size_t mvllm_moe_ep_window_layout(int nranks, int seg, int K, int D, int x_dtype,
                                            size_t *offsets);
/* The dispatch as stores into the ranks' windows (replaces ep_pack_dev and
 * the dispatch exchanges): with pos / send_cnt from ep_plan_fixed_dev
 * (capacity = seg, T <= seg), token c planned at row d*seg + j for rank d
 * goes to row self_rank*seg + j of d's window (x row, local ids or -1,
 * weights); rows j >= send_cnt[d] of that segment get ids -1.
 * windows: device array [nranks] of the window bases (own at self_rank). */
MVLLM_API int mvllm_moe_ep_dispatch_peer_dev(void *stream, const void *x, int x_dtype,
                                             const int *idx, const float *wt, int T, int K,
                                             int D, int E, int nranks, const int *dest,
                                             const int *lid, int self_rank, int seg,
                                             const int *pos, const int *send_cnt,
                                             void *const *windows);
/* The rank's experts over the nranks*seg rows of its own window (`window`,
 * the host value of windows[self_rank]), the routed layer of
 * mvllm_moe_layer_partial_dev with each token's partial row stored into its
 * owner's window instead of a local buffer: received row o*seg + j goes to
 * row self_rank*seg + j of the back region of rank o's window.  Rows with no
 * slot on this rank are not written.  Workspace: mvllm_moe_layer_workspace(
 * nranks*seg, K, E, 0, D, Iinter, fmt).  Errors as layer_partial_dev. */
MVLLM_API int mvllm_moe_layer_partial_peer_dev(void *stream, int nranks, int seg, int self_rank,
                                               int K, int E, int D, int Iinter, int fmt,
                                               int x_dtype, void *window, void *const *windows,
                                               const void *const *g, const void *const *u,
                                               const void *const *d, const void *const *gs,
                                               const void *const *us, const void *const *ds,
                                               int act, float act_a, float act_b,
                                               void *workspace, size_t workspace_bytes);
/* mvllm_moe_layer_dev whose per-token result goes to a partial row for the
 * expert-parallel return instead of being added into f32 `out`: row c of
 * out16 (pitch 2*D + 16 bytes, 16-byte aligned) holds the D values of the
 * token's ordered sum (from zero) as f16 of v / 2^s and, in its 16-byte tail,
 * the f32 2^s, chosen per row so that the largest |v| / 2^s lies in
 * [2^14, 2^15).  Relative error at most 2^-11 per element; half the bytes of
 * f32 rows.  D a multiple of 8, at most 32768; same workspace as layer_dev. */
MVLLM_API int mvllm_moe_layer_partial_dev(void *stream, int T, int K, int E, int n_shared, int D,
                                          int Iinter, int fmt, const int *idx, const float *wt,
                                          const void *x, int x_dtype, const void *const *g,
                                          const void *const *u, const void *const *d,
                                          const void *const *gs, const void *const *us,
                                          const void *const *ds, void *out16, int act,
                                          float act_a, float act_b, void *workspace,
                                          size_t workspace_bytes);

/* ---- layer epilogue after the routed combine: the step both
 *      callers take after moe_block, kimi_k3.cpp:2074-2108 and
 *      glm53.cpp:1993-2027 ---- */
/* For each token c: a = acc[c] (L floats, the routed sum); if lat_n:
 * a = rmsnorm(a, lat_n, eps) (quant.cpp:384-398); if up_w: u = a . W_up^T
 * (QuantMat::gemm, fmt 0/4/8, W_up [H, L]) else u = a (then L == H);
 * h[c][i] += u[i] * routed_scale; if shared: h[c][i] += shared[c][i] (the
 * shared expert's output, not scaled).  All device pointers; h accumulated. */
MVLLM_API size_t mvllm_moe_epilogue_workspace(int T, int H, int L);
MVLLM_API int mvllm_moe_epilogue_dev(void *stream, int T, int H, int L, const float *acc,
                                     const float *lat_n, float eps, int up_fmt, const void *up_w,
                                     const void *up_scales, float routed_scale,
                                     const float *shared, float *h, void *workspace,
                                     size_t workspace_bytes);

/* A dense gated FFN for T rows, in the reference's arithmetic:
 * g = x . gate^T, u = x . up^T (each [T, O], as mvllm_matmul_dev), the
 * activation per element (act, act_a, act_b as in moe_block), then
 * d = h . down^T ([T, H]); y = d, or y += d when accumulate.  All three
 * weights in format fmt (0, 4, 8 or 9) with their scales.  This is
 * DeepSeek-V4's shared expert (dsv4_cuda::expert_fp8 + moe,
 * dsv4_cuda.cpp:169-189, 826-848) and its dense/shared MLP
 * (dsv4.cpp:2849-2860, 2999-3008).  Workspace:
 * mvllm_moe_dense_ffn_workspace(T, H, O) bytes. */
MVLLM_API size_t mvllm_moe_dense_ffn_workspace(int T, int H, int O);
MVLLM_API int mvllm_moe_dense_ffn_dev(void *stream, int fmt, int T, int H, int O,
                                      const void *gate_w, const void *gate_s, const void *up_w,
                                      const void *up_s, const void *down_w, const void *down_s,
                                      const float *x, int act, float act_a, float act_b,
                                      float *y, int accumulate, void *workspace,
                                      size_t workspace_bytes);

/* Health check of the bounded device waits that every pipeline kernel uses:
 * runs one small kernel that waits on an mbarrier one thread completes and
 * then on one that nothing completes.  *completed = 1 when the first wait
 * succeeded; *timed_out = 1 when the second gave up after its time limit
 * (2 s) and recorded MVLLM_ERR_TIMEOUT.  The context stays usable. */
MVLLM_API int mvllm_moe_wait_selftest(int *completed, int *timed_out);

/* Per-phase device time of the device-pointer entries, from CUDA events
 * recorded on the launch stream after each phase while enabled (the role of
 * the reference's AccTimer accumulators, src/model/glm53.cpp:39-46, on the
 * device).  Phases: 0 permute, 1 gather, 2 plan, 3 expert phase 1 (gate/up
 * + activation), 4 expert phase 2 (down), 5 combine.  enable(1) starts a new
 * window; read() synchronises, fills ms[]/launches[] (n entries) and returns
 * the number of phases. */
MVLLM_API void mvllm_moe_profile_enable(int on);
MVLLM_API int mvllm_moe_profile_read(double *ms, long long *launches, int n);

#ifdef __cplusplus
}
#endif

#endif /* MVLLM_MOE_H */
