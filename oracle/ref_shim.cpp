// ref_shim.cpp -- C entry points over the UNMODIFIED reference sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the reference's own src/quant/quant.cpp, src/gpu/metal_ops.cpp,
// src/model/ops.cpp and src/model/moe_pick.cpp (read in place, never copied)
// into oracle/_ref/libmvllm_ref.so.  Tests use it to pin the C restatement in
// moe_oracle.c, tests/golden/gen_golden.py uses it to produce the fixtures,
// and bench.py's reference arm times ref_moe_block as the reference CPU path.
//
// Each wrapper forwards to the reference function named beside it; nothing
// here computes anything itself.
#include "src/gpu/metal_ops.hpp"
#include "src/model/moe_pick.hpp"
#include "src/quant/quant.hpp"

#include <cstdint>

namespace mvllm {
// Declared in src/model/family.hpp:402 and :458, defined in src/model/ops.cpp.
int moe_topk(const float *choice, int n, int k, int *idx, float *w, const float *mix);
int moe_union_ids(const int *idx, int n_tok, int topk, int *out, int out_cap);
} // namespace mvllm

#define REF_API extern "C" __attribute__((visibility("default")))

// metal_ops::moe_block (src/gpu/metal_ops.hpp:104-108); bool -> int.
REF_API int ref_moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
                          const void *const *u, const void *const *d, const float *const *gs,
                          const float *const *us, const float *const *ds, const float *xg,
                          const int *xoff, const int *nr, const int *rows, const float *rw,
                          float *out, int S, int act, float act_a, float act_b) {
    return mvllm::metal_ops::moe_block(nb, D, Iinter, fmt, qgs, g, u, d, gs, us, ds, xg, xoff, nr,
                                       rows, rw, out, S,
                                       static_cast<mvllm::metal_ops::Act>(act), act_a, act_b)
               ? 1
               : 0;
}

REF_API int ref_init() { return mvllm::metal_ops::init() ? 1 : 0; }

// quant:: codecs and matmuls (src/quant/quant.hpp:53-70).
REF_API void ref_quantize_int4_g64(const float *w, int O, int I, uint8_t *p, float *s) {
    mvllm::quant::quantize_int4_g64(w, O, I, p, s);
}
REF_API void ref_pack_mxfp4(const float *w, int O, int I, uint8_t *p, uint8_t *s) {
    mvllm::quant::pack_mxfp4(w, O, I, p, s);
}
REF_API void ref_matmul_f32(float *y, const float *x, const float *w, int S, int I, int O) {
    mvllm::quant::matmul_f32(y, x, w, S, I, O);
}
REF_API void ref_matmul_int4_g64(float *y, const float *x, const uint8_t *p, const float *s, int S,
                                 int I, int O) {
    mvllm::quant::matmul_int4_g64(y, x, p, s, S, I, O);
}
REF_API void ref_matmul_mxfp4(float *y, const float *x, const uint8_t *p, const uint8_t *s, int S,
                              int I, int O) {
    mvllm::quant::matmul_mxfp4(y, x, p, s, S, I, O);
}
REF_API void ref_quantize_int8_row(const float *w, int O, int I, int8_t *q, float *s) {
    mvllm::quant::quantize_int8_row(w, O, I, q, s);
}
REF_API void ref_matmul_int8_row(float *y, const float *x, const int8_t *q, const float *s, int S,
                                 int I, int O) {
    mvllm::quant::matmul_int8_row(y, x, q, s, S, I, O);
}
REF_API void ref_rmsnorm(const float *x, const float *w, float *y, int n, float eps) {
    mvllm::quant::rmsnorm(x, w, y, n, eps);
}
REF_API float ref_situ_glu(float g, float u, float b1, float b2) {
    return mvllm::quant::situ_glu(g, u, b1, b2);
}
REF_API float ref_clamped_swiglu(float g, float u, float limit) {
    return mvllm::quant::clamped_swiglu(g, u, limit);
}
REF_API void ref_softmax_inplace(float *x, int n) { mvllm::quant::softmax_inplace(x, n); }
REF_API float ref_sigmoid(float x) { return mvllm::quant::sigmoid(x); }
REF_API float ref_mx4_scale(uint8_t s) { return mvllm::quant::mx4_scale(s); }

// Routing (src/model/ops.cpp:860-890, :1082-1099; src/model/moe_pick.cpp:40-83).
REF_API int ref_moe_topk(const float *choice, int n, int k, int *idx, float *w, const float *mix) {
    return mvllm::moe_topk(choice, n, k, idx, w, mix);
}
REF_API int ref_moe_union_ids(const int *idx, int n_tok, int topk, int *out, int out_cap) {
    return mvllm::moe_union_ids(idx, n_tok, topk, out, out_cap);
}
REF_API int ref_moe_topk_pick(const float *scores, int n, int k, int *idx, float *w) {
    return mvllm::moe_topk_pick(scores, n, k, idx, w);
}
