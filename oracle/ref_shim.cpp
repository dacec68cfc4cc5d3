// ref_shim.cpp -- C entry points over the UNMODIFIED reference sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the reference's own src/quant/quant.cpp, src/gpu/metal_ops.cpp,
// src/model/ops.cpp, src/model/moe_pick.cpp and, for DeepSeek-V4, the CPU
// tier src/gpu/dsv4_cuda.cpp with src/quant/native_act.cpp and
// src/quant/bf16.cpp (read in place, never copied)
// into oracle/_ref/libmvllm_ref.so.  Tests use it to pin the C restatement in
// moe_oracle.c, tests/golden/gen_golden.py uses it to produce the fixtures,
// and bench.py's reference arm times ref_moe_block as the reference CPU path.
//
// Each wrapper forwards to the reference function named beside it; nothing
// here computes anything itself.
#include "src/gpu/dsv4_cuda.hpp"
#include "src/gpu/metal_ops.hpp"
#include "src/model/moe_pick.hpp"
#include "src/quant/native_act.hpp"
#include "src/quant/quant.hpp"

#include <cstdint>
#include <vector>

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

// ---- DeepSeek-V4 CPU tier (src/gpu/dsv4_cuda.hpp; src/quant/native_act.hpp) ----
// Each wrapper builds the reference's own Tensor / Activation / ExpertSet
// objects through its public upload calls and frees them afterwards.
namespace dsv4 = mvllm::dsv4_cuda;

REF_API float ref_e8m0_decode(uint8_t v) { return mvllm::e8m0_decode(v); }
REF_API float ref_e4m3fn_decode(uint8_t v) { return mvllm::e4m3fn_decode(v); }

// dsv4_cuda::matvec over FP8 tiles (dsv4_cuda.cpp:571-623), row by row.
REF_API void ref_matmul_fp8_b128(float *y, const float *x, const uint8_t *w, const uint8_t *sc,
                                 int S, int I, int O) {
    dsv4::Tensor *t = nullptr;
    if (!dsv4::upload_fp8(&t, w, sc, O, I, 0))
        return;
    for (int s = 0; s < S; ++s)
        dsv4::matvec(t, y + static_cast<size_t>(s) * O, x + static_cast<size_t>(s) * I);
    dsv4::tensor_free(t);
}

namespace {
dsv4::Activation *act_from(const float *x, int n) {
    dsv4::Activation *a = dsv4::activation_create(0, n);
    if (a)
        dsv4::activation_upload(a, x, n);
    return a;
}
struct Experts { // one FP4 tensor triple per expert, nullptr where absent
    std::vector<dsv4::Tensor *> g, u, d;
    Experts(int n, int H, int O, const void *const *gp, const void *const *up,
            const void *const *dp, const void *const *gs, const void *const *us,
            const void *const *ds)
        : g(n, nullptr), u(n, nullptr), d(n, nullptr) {
        for (int e = 0; e < n; ++e) {
            if (!gp[e] || !up[e] || !dp[e])
                continue;
            auto b = [](const void *p) { return static_cast<const uint8_t *>(p); };
            dsv4::upload_fp4(&g[e], b(gp[e]), b(gs[e]), O, H, 0);
            dsv4::upload_fp4(&u[e], b(up[e]), b(us[e]), O, H, 0);
            dsv4::upload_fp4(&d[e], b(dp[e]), b(ds[e]), H, O, 0);
        }
    }
    ~Experts() {
        for (size_t e = 0; e < g.size(); ++e) {
            dsv4::tensor_free(g[e]);
            dsv4::tensor_free(u[e]);
            dsv4::tensor_free(d[e]);
        }
    }
};
struct Shared { // FP8 shared expert: gate, gate scales, up, up scales, down, down scales
    dsv4::Tensor *g = nullptr, *u = nullptr, *d = nullptr;
    Shared(int H, int O, const void *const *sh) {
        if (!sh)
            return;
        auto b = [](const void *p) { return static_cast<const uint8_t *>(p); };
        dsv4::upload_fp8(&g, b(sh[0]), b(sh[1]), O, H, 0);
        dsv4::upload_fp8(&u, b(sh[2]), b(sh[3]), O, H, 0);
        dsv4::upload_fp8(&d, b(sh[4]), b(sh[5]), H, O, 0);
    }
    ~Shared() {
        dsv4::tensor_free(g);
        dsv4::tensor_free(u);
        dsv4::tensor_free(d);
    }
};
} // namespace

// dsv4_cuda::route (dsv4_cuda.cpp:1541-1587) for one token.
REF_API int ref_dsv4_route(const float *x, int H, const float *router, const float *bias, int E,
                           const int *fixed, float routed_scale, int *ids, float *w) {
    dsv4::Tensor *tg = nullptr, *tb = nullptr;
    dsv4::upload_f32(&tg, router, E, H, 0);
    if (bias)
        dsv4::upload_f32(&tb, bias, E, 1, 0);
    dsv4::Activation *a = act_from(x, H);
    const bool ok = dsv4::route(a, tg, tb, fixed, routed_scale, ids, w);
    dsv4::activation_free(a);
    dsv4::tensor_free(tg);
    dsv4::tensor_free(tb);
    return ok ? 1 : 0;
}

// dsv4_cuda::moe (dsv4_cuda.cpp:834-848) for one token.
REF_API int ref_dsv4_moe(const float *x, int H, int O, int n, const void *const *g,
                         const void *const *u, const void *const *d, const void *const *gs,
                         const void *const *us, const void *const *ds, const float *weights,
                         const void *const *sh, float limit, float *y) {
    Experts ex(n, H, O, g, u, d, gs, us, ds);
    Shared s(H, O, sh);
    return dsv4::moe(ex.g.data(), ex.u.data(), ex.d.data(), weights, n, s.g, s.u, s.d, limit, y,
                     x)
               ? 1
               : 0;
}

// dsv4_cuda::route_moe_ep2 (dsv4_cuda.cpp:1841-1906) for one token, one bank
// of E experts (plus the shared expert, if given) serving both ranks.
REF_API int ref_dsv4_route_moe_ep2(const float *x, int H, const float *router, const float *bias,
                                   int E, float routed_scale, int O, const void *const *g,
                                   const void *const *u, const void *const *d,
                                   const void *const *gs, const void *const *us,
                                   const void *const *ds, const void *const *sh, float limit,
                                   float *out, float *peer_out) {
    Experts ex(E, H, O, g, u, d, gs, us, ds);
    Shared s(H, O, sh);
    dsv4::ExpertSet *set =
        dsv4::expert_set_create(ex.g.data(), ex.u.data(), ex.d.data(), E, s.g, s.u, s.d);
    dsv4::Tensor *tg = nullptr, *tb = nullptr;
    dsv4::upload_f32(&tg, router, E, H, 0);
    if (bias)
        dsv4::upload_f32(&tb, bias, E, 1, 0);
    dsv4::Activation *a = act_from(x, H);
    dsv4::Activation *ao = dsv4::activation_create(0, H);
    dsv4::Activation *po = dsv4::activation_create(0, H);
    const bool ok = dsv4::route_moe_ep2(a, tg, tb, nullptr, nullptr, nullptr, 0, routed_scale,
                                        set, set, limit, ao, po);
    if (ok) {
        dsv4::activation_download(out, ao, H);
        dsv4::activation_download(peer_out, po, H);
    }
    for (dsv4::Activation *p : {a, ao, po})
        dsv4::activation_free(p);
    dsv4::tensor_free(tg);
    dsv4::tensor_free(tb);
    dsv4::expert_set_free(set);
    return ok ? 1 : 0;
}
