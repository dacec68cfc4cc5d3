/*
 * moe_oracle.c -- CPU restatement of micro-vllm's routed-expert MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path in micro-vllm_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product library never links
 * or calls it.
 *
 * Every function restates the reference algorithm with the same arithmetic
 * (f32, same loop nesting and accumulation order) so that, compiled with
 * -O2 -ffp-contract=off like the reference's Release build on x86-64, its
 * outputs are bit-identical to the reference.  That identity is pinned by
 * tests/test_oracle.py against oracle/_ref (the reference's own sources built
 * by oracle/Makefile) and against the committed fixtures in tests/golden/.
 *
 * Reference files (paths inside the micro-vllm project):
 *   src/quant/quant.hpp, src/quant/quant.cpp   -- codecs, matmuls, activations
 *   src/gpu/metal_ops.cpp                      -- moe_block / cpu_moe_block
 *   src/model/ops.cpp                          -- moe_topk, moe_union_ids
 *   src/model/moe_pick.cpp                     -- moe_topk_pick
 *   src/model/glm53.cpp, src/model/kimi_k3.cpp -- gather order, blob geometry
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* e2m1 magnitudes, bit 3 = sign.  quant.cpp:16-17 */
EXPORT const float orc_mx4_lut[16] = {0.f,  0.5f,  1.f,  1.5f,  2.f,  3.f,  4.f,  6.f,
                                      -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

/* ue8m0 -> 2^(s-127) by placing s in the f32 exponent field; s=0 gives +0,
 * s=255 gives +inf.  quant.hpp:12-20 */
EXPORT float orc_mx4_scale(uint8_t s) {
    union {
        uint32_t u;
        float f;
    } b;
    b.u = (uint32_t)s << 23;
    return b.f;
}

/* Two-branch logistic.  quant.hpp:22-29 */
EXPORT float orc_sigmoid(float x) {
    if (x >= 0.f)
        return 1.f / (1.f + expf(-x));
    float z = expf(x);
    return z / (1.f + z);
}

/* SiTU-GLU: b1*tanh(g/b1)*sigmoid(g) * b2*tanh(u/b2).  quant.hpp:32-34 */
EXPORT float orc_situ_glu(float g, float u, float b1, float b2) {
    return b1 * tanhf(g / b1) * orc_sigmoid(g) * b2 * tanhf(u / b2);
}

/* silu(min(g, L)) * clamp(u, -L, L); L <= 0 disables clamping.  quant.hpp:37-50 */
EXPORT float orc_clamped_swiglu(float gate, float up, float limit) {
    float g = gate;
    if (limit > 0.f && g > limit)
        g = limit;
    float s = g * orc_sigmoid(g);
    float u = up;
    if (limit > 0.f) {
        if (u > limit)
            u = limit;
        if (u < -limit)
            u = -limit;
    }
    return s * u;
}

static int packed_stride(int I) { return (I + 1) / 2; }
static int ceil_div(int a, int b) { return (a + b - 1) / b; }
static uint8_t nibble_at(const uint8_t *row, int i) {
    uint8_t b = row[i >> 1];
    return (i & 1) ? (uint8_t)(b >> 4) : (uint8_t)(b & 0x0f);
}
static void pack_nibble(uint8_t *row, int i, uint8_t n) {
    int b = i >> 1;
    if ((i & 1) == 0)
        row[b] = (uint8_t)((row[b] & 0xf0) | (n & 0x0f));
    else
        row[b] = (uint8_t)((row[b] & 0x0f) | ((n & 0x0f) << 4));
}

/* y[S,O] = x[S,I] . W[O,I]^T, sequential accumulation in i.  quant.cpp:143-156 */
EXPORT void orc_matmul_f32(float *y, const float *x, const float *w, int S, int I, int O) {
    for (int s = 0; s < S; ++s) {
        const float *xs = x + (size_t)s * I;
        float *ys = y + (size_t)s * O;
        for (int o = 0; o < O; ++o) {
            const float *wo = w + (size_t)o * I;
            float acc = 0.f;
            for (int i = 0; i < I; ++i)
                acc += xs[i] * wo[i];
            ys[o] = acc;
        }
    }
}

/* int8 per-row quantiser: scale = absmax/127, q = clamp(round(w * (1/scale)),
 * -127, 127), all zero for a zero row.  quant.cpp:230-253 */
EXPORT void orc_quantize_int8_row(const float *w, int O, int I, int8_t *q, float *scales) {
    for (int o = 0; o < O; ++o) {
        const float *row = w + (size_t)o * I;
        int8_t *qrow = q + (size_t)o * I;
        float amax = 0.f;
        for (int i = 0; i < I; ++i) {
            const float a = fabsf(row[i]);
            if (a > amax)
                amax = a;
        }
        const float scale = amax / 127.f;
        scales[o] = scale;
        if (scale == 0.f) {
            memset(qrow, 0, (size_t)I);
            continue;
        }
        const float inv = 1.f / scale;
        for (int i = 0; i < I; ++i) {
            int qi = (int)roundf(row[i] * inv);
            qi = qi < -127 ? -127 : (qi > 127 ? 127 : qi);
            qrow[i] = (int8_t)qi;
        }
    }
}

/* y[s,o] = (sum_i x[s,i] * q[o,i]) * scale[o], sequential in i.  quant.cpp:255-268 */
EXPORT void orc_matmul_int8_row(float *y, const float *x, const int8_t *q, const float *scales,
                                int S, int I, int O) {
    for (int s = 0; s < S; ++s) {
        const float *xs = x + (size_t)s * I;
        float *ys = y + (size_t)s * O;
        for (int o = 0; o < O; ++o) {
            const int8_t *qrow = q + (size_t)o * I;
            float acc = 0.f;
            for (int i = 0; i < I; ++i)
                acc += xs[i] * (float)qrow[i];
            ys[o] = acc * scales[o];
        }
    }
}

/* y = x * (1 / sqrt(sum(x^2)/n + eps)) * w (w may be null).  quant.cpp:384-398 */
EXPORT void orc_rmsnorm(const float *x, const float *w, float *y, int n, float eps) {
    if (n <= 0)
        return;
    float ss = 0.f;
    for (int i = 0; i < n; ++i)
        ss += x[i] * x[i];
    const float inv = 1.f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; ++i)
        y[i] = w ? x[i] * inv * w[i] : x[i] * inv;
}

/* int4-g64 quantiser: scale = absmax/7 floored at 1e-8, q = clamp(round(w/scale),-8,7),
 * nibble q+8, low nibble = even column.  quant.cpp:170-201 */
EXPORT void orc_quantize_int4_g64(const float *w, int O, int I, uint8_t *packed, float *scales) {
    const int stride = packed_stride(I);
    const int ng = ceil_div(I, 64);
    for (int o = 0; o < O; ++o) {
        const float *row = w + (size_t)o * I;
        uint8_t *prow = packed + (size_t)o * stride;
        memset(prow, 0, (size_t)stride);
        for (int g = 0; g < ng; ++g) {
            int i0 = g * 64, i1 = i0 + 64;
            if (i1 > I)
                i1 = I;
            float amax = 0.f;
            for (int i = i0; i < i1; ++i) {
                float a = fabsf(row[i]);
                if (a > amax)
                    amax = a;
            }
            float scale = amax / 7.f;
            if (scale < 1e-8f)
                scale = 1e-8f;
            scales[(size_t)o * ng + g] = scale;
            float inv = 1.f / scale;
            for (int i = i0; i < i1; ++i) {
                int q = (int)roundf(row[i] * inv);
                if (q < -8)
                    q = -8;
                if (q > 7)
                    q = 7;
                pack_nibble(prow, i, (uint8_t)(q + 8));
            }
        }
    }
}

/* y = x . dequant(W)^T, element = (nib-8)*scale[group], sequential f32 sum.
 * quant.cpp:203-228 */
EXPORT void orc_matmul_int4_g64(float *y, const float *x, const uint8_t *packed,
                                const float *scales, int S, int I, int O) {
    const int stride = packed_stride(I);
    const int ng = ceil_div(I, 64);
    for (int s = 0; s < S; ++s) {
        const float *xs = x + (size_t)s * I;
        float *ys = y + (size_t)s * O;
        for (int o = 0; o < O; ++o) {
            const uint8_t *prow = packed + (size_t)o * stride;
            const float *srow = scales + (size_t)o * ng;
            float acc = 0.f;
            for (int g = 0; g < ng; ++g) {
                int i0 = g * 64, i1 = i0 + 64;
                if (i1 > I)
                    i1 = I;
                float scale = srow[g];
                for (int i = i0; i < i1; ++i) {
                    int q = (int)nibble_at(prow, i) - 8;
                    acc += xs[i] * ((float)q * scale);
                }
            }
            ys[o] = acc;
        }
    }
}

/* Smallest ue8m0 code e with 2^(e-127) >= need (0 only for need == 0).  quant.cpp:47-77 */
static uint8_t ue8m0_cover(float need) {
    if (!(need > 0.f))
        return 0;
    if (!isfinite(need))
        return 255;
    union {
        uint32_t u;
        float f;
    } b;
    b.f = need;
    int exp_field = (int)((b.u >> 23) & 0xffu);
    uint32_t frac = b.u & 0x7fffffu;
    int e;
    if (exp_field == 0)
        e = 1;
    else if (exp_field == 255)
        e = 255;
    else
        e = (frac == 0) ? exp_field : exp_field + 1;
    if (e < 0)
        e = 0;
    if (e > 255)
        e = 255;
    while (e < 255 && orc_mx4_scale((uint8_t)e) < need)
        ++e;
    while (e > 0 && orc_mx4_scale((uint8_t)(e - 1)) >= need)
        --e;
    return (uint8_t)e;
}

/* Nearest e2m1 magnitude to |w/scale|, ties to the lower code; sign from signbit(w).
 * quant.cpp:79-96 */
static uint8_t closest_mx4(float w, float scale) {
    float target = 0.f;
    if (scale > 0.f && isfinite(scale))
        target = w / scale;
    float a = fabsf(target);
    int best = 0;
    float best_d = fabsf(orc_mx4_lut[0] - a);
    for (int k = 1; k < 8; ++k) {
        float d = fabsf(orc_mx4_lut[k] - a);
        if (d < best_d) {
            best_d = d;
            best = k;
        }
    }
    if (signbit(w))
        best |= 8;
    return (uint8_t)best;
}

EXPORT uint8_t orc_ue8m0_cover(float need) { return ue8m0_cover(need); }
EXPORT uint8_t orc_closest_mx4(float w, float scale) { return closest_mx4(w, scale); }

/* MXFP4 packer: per 32 columns e = ue8m0_cover(absmax/6).  quant.cpp:270-296 */
EXPORT void orc_pack_mxfp4(const float *w, int O, int I, uint8_t *packed, uint8_t *scales) {
    const int stride = packed_stride(I);
    const int ng = ceil_div(I, 32);
    for (int o = 0; o < O; ++o) {
        const float *row = w + (size_t)o * I;
        uint8_t *prow = packed + (size_t)o * stride;
        memset(prow, 0, (size_t)stride);
        for (int g = 0; g < ng; ++g) {
            int i0 = g * 32, i1 = i0 + 32;
            if (i1 > I)
                i1 = I;
            float amax = 0.f;
            for (int i = i0; i < i1; ++i) {
                float a = fabsf(row[i]);
                if (a > amax)
                    amax = a;
            }
            uint8_t e = ue8m0_cover(amax / 6.f);
            scales[(size_t)o * ng + g] = e;
            float scale = orc_mx4_scale(e);
            for (int i = i0; i < i1; ++i)
                pack_nibble(prow, i, closest_mx4(row[i], scale));
        }
    }
}

/* y = x . dequant(W)^T with element lut[nib]*2^(e-127).  quant.cpp:298-321 */
EXPORT void orc_matmul_mxfp4(float *y, const float *x, const uint8_t *packed,
                             const uint8_t *scales, int S, int I, int O) {
    const int stride = packed_stride(I);
    const int ng = ceil_div(I, 32);
    for (int s = 0; s < S; ++s) {
        const float *xs = x + (size_t)s * I;
        float *ys = y + (size_t)s * O;
        for (int o = 0; o < O; ++o) {
            const uint8_t *prow = packed + (size_t)o * stride;
            const uint8_t *srow = scales + (size_t)o * ng;
            float acc = 0.f;
            for (int g = 0; g < ng; ++g) {
                int i0 = g * 32, i1 = i0 + 32;
                if (i1 > I)
                    i1 = I;
                float scale = orc_mx4_scale(srow[g]);
                for (int i = i0; i < i1; ++i)
                    acc += xs[i] * (orc_mx4_lut[nibble_at(prow, i)] * scale);
            }
            ys[o] = acc;
        }
    }
}

/* In-place softmax: max-subtracted expf, sum, multiply by 1/sum (0 if the
 * sum is 0).  quant.cpp:412-429 */
EXPORT void orc_softmax_inplace(float *x, int n) {
    if (n <= 0)
        return;
    float m = x[0];
    for (int i = 1; i < n; ++i)
        if (x[i] > m)
            m = x[i];
    float sum = 0.f;
    for (int i = 0; i < n; ++i) {
        x[i] = expf(x[i] - m);
        sum += x[i];
    }
    float inv = (sum == 0.f) ? 0.f : 1.f / sum;
    for (int i = 0; i < n; ++i)
        x[i] *= inv;
}

/* act 1 = ClampSwiGLU(a), 2 = SiTU(a, b), anything else = silu(g)*u.
 * metal_ops.cpp:197-211, quant.cpp:400-403 */
EXPORT void orc_apply_act(float *g, const float *u, int n, int act, float a, float b) {
    if (!g || !u || n < 1)
        return;
    if (act == 1) {
        for (int i = 0; i < n; ++i)
            g[i] = orc_clamped_swiglu(g[i], u[i], a);
        return;
    }
    if (act == 2) {
        for (int i = 0; i < n; ++i)
            g[i] = orc_situ_glu(g[i], u[i], a, b);
        return;
    }
    for (int i = 0; i < n; ++i)
        g[i] = g[i] * orc_sigmoid(g[i]) * u[i];
}

/*
 * moe_block: validation as metal_ops.cpp:448-460 (returns 0 = reference
 * "false", 1 = "true"), body as cpu_moe_block metal_ops.cpp:278-342:
 * experts in call order; nr<=0 skipped without advancing base; experts with
 * missing weights (or scales for fmt 4/7) skipped but base advanced; gate, up,
 * act, down; then out[rows[base+r]] += rw[base+r]*hh[r] unless dest<0 or
 * (S>0 && dest>=S).
 */
EXPORT int orc_moe_block(int nb, int D, int Iinter, int fmt, int qgs, const void *const *g,
                         const void *const *u, const void *const *d, const float *const *gs,
                         const float *const *us, const float *const *ds, const float *xg,
                         const int *xoff, const int *nr, const int *rows, const float *rw,
                         float *out, int S, int act, float act_a, float act_b) {
    (void)qgs;
    if (nb < 1 || D < 1 || !out || !xg || (fmt != 0 && fmt != 4 && fmt != 7))
        return 0;
    if (!xoff || !nr)
        return 0;
    int base = 0;
    for (int e = 0; e < nb; ++e) {
        const int nre = nr[e];
        if (nre <= 0)
            continue;
        if (Iinter < 1 || !g || !u || !d || !g[e] || !u[e] || !d[e]) {
            base += nre;
            continue;
        }
        if ((fmt == 4 || fmt == 7) && (!gs || !us || !ds || !gs[e] || !us[e] || !ds[e])) {
            base += nre;
            continue;
        }
        const float *xe = xg + (size_t)xoff[e] * (size_t)D;
        float *gate = (float *)calloc((size_t)nre * Iinter, sizeof(float));
        float *up = (float *)calloc((size_t)nre * Iinter, sizeof(float));
        float *hh = (float *)calloc((size_t)nre * D, sizeof(float));
        if (fmt == 0) {
            orc_matmul_f32(gate, xe, (const float *)g[e], nre, D, Iinter);
            orc_matmul_f32(up, xe, (const float *)u[e], nre, D, Iinter);
            orc_apply_act(gate, up, nre * Iinter, act, act_a, act_b);
            orc_matmul_f32(hh, gate, (const float *)d[e], nre, Iinter, D);
        } else if (fmt == 7) {
            orc_matmul_mxfp4(gate, xe, (const uint8_t *)g[e], (const uint8_t *)gs[e], nre, D,
                             Iinter);
            orc_matmul_mxfp4(up, xe, (const uint8_t *)u[e], (const uint8_t *)us[e], nre, D,
                             Iinter);
            orc_apply_act(gate, up, nre * Iinter, act, act_a, act_b);
            orc_matmul_mxfp4(hh, gate, (const uint8_t *)d[e], (const uint8_t *)ds[e], nre,
                             Iinter, D);
        } else {
            orc_matmul_int4_g64(gate, xe, (const uint8_t *)g[e], gs[e], nre, D, Iinter);
            orc_matmul_int4_g64(up, xe, (const uint8_t *)u[e], us[e], nre, D, Iinter);
            orc_apply_act(gate, up, nre * Iinter, act, act_a, act_b);
            orc_matmul_int4_g64(hh, gate, (const uint8_t *)d[e], ds[e], nre, Iinter, D);
        }
        if (rows && rw) {
            for (int r = 0; r < nre; ++r) {
                const int dest = rows[base + r];
                if (dest < 0 || (S > 0 && dest >= S))
                    continue;
                const float wr = rw[base + r];
                const float *hr = hh + (size_t)r * D;
                float *orow = out + (size_t)dest * D;
                for (int i = 0; i < D; ++i)
                    orow[i] += wr * hr[i];
            }
        }
        free(gate);
        free(up);
        free(hh);
        base += nre;
    }
    return 1;
}

/*
 * moe_topk: the k largest `choice` entries, descending, ties to the lower
 * index (ops.cpp:860-890 uses partial_sort with that total order, so the
 * result is fully determined for non-NaN input).  Weights come from mix (or
 * choice), are clipped at 0 and L1-normalised; a non-positive sum gives 1/k.
 */
EXPORT int orc_moe_topk(const float *choice, int n, int k, int *idx, float *w, const float *mix) {
    if (k > n)
        k = n;
    char *taken = (char *)calloc((size_t)(n > 0 ? n : 1), 1);
    for (int j = 0; j < k; ++j) {
        int best = -1;
        for (int i = 0; i < n; ++i) {
            if (taken[i])
                continue;
            if (best < 0 || choice[i] > choice[best])
                best = i; /* strict > keeps the lower index on ties */
        }
        taken[best] = 1;
        idx[j] = best;
    }
    free(taken);
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
        w[i] = mix ? mix[idx[i]] : choice[idx[i]];
        if (w[i] < 0.f)
            w[i] = 0.f;
        sum += w[i];
    }
    if (sum > 0.f) {
        for (int i = 0; i < k; ++i)
            w[i] /= sum;
    } else {
        for (int i = 0; i < k; ++i)
            w[i] = 1.f / (float)k;
    }
    return k;
}

static int cmp_int(const void *a, const void *b) {
    int x = *(const int *)a, y = *(const int *)b;
    return (x > y) - (x < y);
}

/* Sorted unique non-negative ids, capped at out_cap.  ops.cpp:1082-1099 */
EXPORT int orc_moe_union_ids(const int *idx, int n_tok, int topk, int *out, int out_cap) {
    if (!idx || !out || n_tok <= 0 || topk <= 0 || out_cap <= 0)
        return 0;
    int *all = (int *)malloc(sizeof(int) * (size_t)n_tok * (size_t)topk);
    int n = 0;
    for (int i = 0; i < n_tok * topk; ++i)
        if (idx[i] >= 0)
            all[n++] = idx[i];
    if (n <= 0) {
        free(all);
        return 0;
    }
    qsort(all, (size_t)n, sizeof(int), cmp_int);
    int u = 0;
    for (int i = 0; i < n && u < out_cap; ++i)
        if (u == 0 || all[i] != out[u - 1])
            out[u++] = all[i];
    free(all);
    return u;
}

/* NaN-safe greedy pick: strict > over finite scores, fallback pick kk (or 0),
 * non-finite / negative weights -> 0, L1-normalise or uniform.
 * moe_pick.cpp:9-21 (moe_router_pick), :40-83 */
EXPORT int orc_moe_topk_pick(const float *scores, int n_experts, int k, int *idx, float *w) {
    if (!scores || !idx || !w || n_experts < 0)
        return 0;
    if (k > n_experts)
        k = n_experts;
    if (k < 0)
        k = 0;
    if (k == 0)
        return 0;
    char *taken = (char *)calloc((size_t)n_experts, 1);
    for (int kk = 0; kk < k; ++kk) {
        int best = -1;
        float bv = -1e30f;
        for (int e = 0; e < n_experts; ++e) {
            if (!taken[e] && scores[e] > bv) {
                bv = scores[e];
                best = e;
            }
        }
        int pick = best >= 0 ? best : (kk < n_experts ? kk : 0);
        idx[kk] = pick;
        if (pick >= 0 && pick < n_experts)
            taken[pick] = 1;
    }
    free(taken);
    float sum = 0.f;
    for (int kk = 0; kk < k; ++kk) {
        const int e = idx[kk];
        float v = (e >= 0 && e < n_experts) ? scores[e] : 0.f;
        if (!isfinite(v) || v < 0.f)
            v = 0.f;
        w[kk] = v;
        sum += v;
    }
    if (sum > 0.f) {
        for (int kk = 0; kk < k; ++kk)
            w[kk] /= sum;
    } else {
        const float uu = 1.f / (float)k;
        for (int kk = 0; kk < k; ++kk)
            w[kk] = uu;
    }
    return k;
}

/*
 * Caller-side permutation (glm53.cpp:1958-1971, kimi_k3.cpp:2036-2050): for
 * each union expert in ascending id, tokens c ascending whose
 * wsum = sum_t wt[c,t]*[idx[c,t]==e] (t ascending, from 0.f) is non-zero.
 * Emits nr[U], xoff[U] (segment starts), rows[R] (token ids) and rw[R]
 * (wsums) in expert-major order.  Returns R, the total routed rows.
 */
EXPORT int orc_moe_permute(const int *idx, const float *wt, int C, int K, const int *uniq, int nu,
                           int *nr, int *xoff, int *rows, float *rw) {
    int n_all = 0;
    for (int ui = 0; ui < nu; ++ui) {
        const int eid = uniq[ui];
        int n = 0;
        xoff[ui] = n_all;
        for (int c = 0; c < C; ++c) {
            float wsum = 0.f;
            for (int t = 0; t < K; ++t)
                if (idx[(size_t)c * K + t] == eid)
                    wsum += wt[(size_t)c * K + t];
            if (wsum == 0.f)
                continue;
            rows[n_all + n] = c;
            rw[n_all + n] = wsum;
            ++n;
        }
        nr[ui] = n;
        n_all += n;
    }
    return n_all;
}

/* Expert-blob byte offsets.  GLM int4-g64 (glm53.cpp:56-78): gate, gate
 * scales, up, up scales, down, down scales.  K3 MXFP4 (kimi_k3.cpp:83-102):
 * w1 (gate), w1 scales, w2 (down), w2 scales, w3 (up), w3 scales.
 * off[0..5] = byte offsets of g, gs, u, us, d, ds; returns the slot size. */
/* Layer epilogue after the routed combine, per token c (kimi_k3.cpp:2074-2108;
 * glm53.cpp:1993-2027 is the L == H case without norm or projection):
 *   a = acc[c] (L floats); if lat_n: a = rmsnorm(a, lat_n, eps);
 *   u = up_w ? QuantMat::gemm(up, a) (weight.cpp:47-64: fmt 4 int4-g64 when
 *       L % 64 == 0, fmt 8 int8 rows, else f32) : a;
 *   h[c][i] += u[i] * routed_scale;  if shared: h[c][i] += shared[c][i]. */
EXPORT void orc_moe_epilogue(int T, int H, int L, const float *acc, const float *lat_n, float eps,
                             int up_fmt, const void *up_w, const void *up_scales,
                             float routed_scale, const float *shared, float *h) {
    float *a = (float *)malloc(sizeof(float) * (size_t)L);
    float *u = (float *)malloc(sizeof(float) * (size_t)H);
    for (int c = 0; c < T; ++c) {
        const float *ac = acc + (size_t)c * L;
        if (lat_n)
            orc_rmsnorm(ac, lat_n, a, L, eps);
        else
            memcpy(a, ac, sizeof(float) * (size_t)L);
        if (up_w) {
            if (up_fmt == 4 && L % 64 == 0)
                orc_matmul_int4_g64(u, a, (const uint8_t *)up_w, (const float *)up_scales, 1, L,
                                    H);
            else if (up_fmt == 8)
                orc_matmul_int8_row(u, a, (const int8_t *)up_w, (const float *)up_scales, 1, L,
                                    H);
            else
                orc_matmul_f32(u, a, (const float *)up_w, 1, L, H);
        } else {
            memcpy(u, a, sizeof(float) * (size_t)H);
        }
        float *hc = h + (size_t)c * H;
        for (int i = 0; i < H; ++i)
            hc[i] += u[i] * routed_scale;
        if (shared)
            for (int i = 0; i < H; ++i)
                hc[i] += shared[(size_t)c * H + i];
    }
    free(a);
    free(u);
}

EXPORT int64_t orc_glm_geom(int hidden, int inter, int64_t *off) {
    int64_t pack_go, sc_go, pack_d, sc_d, slot;
    if (hidden > 0 && inter > 0 && hidden % 64 == 0 && inter % 64 == 0) {
        pack_go = (int64_t)inter * hidden / 2;
        sc_go = (int64_t)inter * hidden / 64 * 4;
        pack_d = pack_go;
        sc_d = sc_go;
        slot = 3 * (pack_go + sc_go);
    } else {
        pack_go = (int64_t)inter * ((hidden + 1) / 2);
        sc_go = (int64_t)inter * ((hidden + 63) / 64) * 4;
        pack_d = (int64_t)hidden * ((inter + 1) / 2);
        sc_d = (int64_t)hidden * ((inter + 63) / 64) * 4;
        slot = 2 * (pack_go + sc_go) + pack_d + sc_d;
    }
    off[0] = 0;
    off[1] = pack_go;
    off[2] = pack_go + sc_go;
    off[3] = off[2] + pack_go;
    off[4] = off[3] + sc_go;
    off[5] = off[4] + pack_d;
    (void)sc_d;
    return slot;
}

EXPORT int64_t orc_k3_geom(int latent, int inter, int64_t *off) {
    int64_t w1p, w1s, w2p, w2s;
    if (latent >= 32 && inter >= 32 && latent % 32 == 0 && inter % 32 == 0) {
        w1p = (int64_t)inter * (latent / 2);
        w1s = (int64_t)inter * (latent / 32);
        w2p = (int64_t)latent * (inter / 2);
        w2s = (int64_t)latent * (inter / 32);
    } else {
        w1p = (int64_t)inter * ((latent + 1) / 2);
        w1s = (int64_t)inter * ((latent + 31) / 32);
        w2p = (int64_t)latent * ((inter + 1) / 2);
        w2s = (int64_t)latent * ((inter + 31) / 32);
    }
    /* order in the blob: w1p w1s w2p w2s w3p w3s (kimi_k3.cpp:138-143) */
    off[0] = 0;                    /* gate = w1 */
    off[1] = w1p;                  /* gate scales */
    off[4] = w1p + w1s;            /* down = w2 */
    off[5] = off[4] + w2p;         /* down scales */
    off[2] = off[5] + w2s;         /* up = w3 */
    off[3] = off[2] + w1p;         /* up scales */
    return 2 * (w1p + w1s) + w2p + w2s;
}

/* ======================================================================
 * DeepSeek-V4 routed experts (src/gpu/dsv4_cuda.cpp, CPU tier; decoders in
 * src/quant/native_act.cpp).  Routing by sqrt(softplus), MXFP4 experts
 * through quant::matmul_mxfp4 with clamped SwiGLU, an optional FP8 shared
 * expert, and the two-rank expert split (EP2) whose partial outputs are
 * summed.  Per token, as the reference.
 * ====================================================================== */

/* ue8m0 -> 2^(v-127); 255 is NaN.  native_act.cpp:65-69 */
EXPORT float orc_e8m0_decode(uint8_t v) {
    if (v == 0xff)
        return NAN;
    return ldexpf(1.f, (int)v - 127);
}

/* e4m3fn: 0x7f / 0xff NaN, exponent 0 subnormal.  native_act.cpp:90-100 */
EXPORT float orc_e4m3fn_decode(uint8_t v) {
    const int sign = v >> 7, ex = (v >> 3) & 15, man = v & 7;
    if (ex == 15 && man == 7)
        return NAN;
    const float mag = ex == 0 ? ldexpf((float)man, -9) : ldexpf(1.f + (float)man / 8.f, ex - 7);
    return sign ? -mag : mag;
}

/* softplus with its +-20 cut-offs, then sqrt(max(., 0)).  dsv4_cuda.cpp:26-34 */
EXPORT float orc_sqrt_softplus(float z) {
    float sp;
    if (z > 20.f)
        sp = z;
    else if (z < -20.f)
        sp = expf(z);
    else
        sp = log1pf(expf(z));
    return sqrtf(sp < 0.f ? 0.f : sp);
}

/* y = x . dequant(W)^T for FP8 tensors: s += x[i] * (e4m3fn(q) * e8m0(tile)),
 * tile (o/128, i/128) of max(ceil(I/128), 1) per tile row.
 * dsv4_cuda.cpp:127-135 (dequant), :618-623 (matvec loop) */
EXPORT void orc_matmul_fp8_b128(float *y, const float *x, const uint8_t *w, const uint8_t *scales,
                                int S, int I, int O) {
    const int si = ceil_div(I, 128) > 1 ? ceil_div(I, 128) : 1;
    for (int s = 0; s < S; ++s) {
        const float *xs = x + (size_t)s * I;
        float *ys = y + (size_t)s * O;
        for (int o = 0; o < O; ++o) {
            float acc = 0.f;
            for (int i = 0; i < I; ++i) {
                const float sc = orc_e8m0_decode(scales[(size_t)(o / 128) * si + i / 128]);
                const float q = orc_e4m3fn_decode(w[(size_t)o * I + i]) * sc;
                acc += xs[i] * q;
            }
            ys[o] = acc;
        }
    }
}

/* dsv4_cuda::route (dsv4_cuda.cpp:1541-1587): logits = router . x
 * (quant::matmul_f32), score = sqrt_softplus, choice = score + bias; the top
 * k = min(6, E) choices by moe_topk (or `fixed` ids), then each weight is the
 * chosen score clipped at 0, divided by their sum over the 6 slots (1/k when
 * the sum is 0), times routed_scale.  ids / w: 6 slots, -1 / 0 past k. */
EXPORT int orc_dsv4_route(const float *x, int H, const float *router, const float *bias, int E,
                          const int *fixed, float routed_scale, int *ids, float *w) {
    if (!x || !router || !ids || !w || E <= 0 || H <= 0)
        return 0;
    float *logits = (float *)calloc((size_t)E * 3, sizeof(float));
    float *score = logits + E, *choice = score + E;
    orc_matmul_f32(logits, x, router, 1, H, E);
    for (int e = 0; e < E; ++e) {
        score[e] = orc_sqrt_softplus(logits[e]);
        choice[e] = score[e] + (bias ? bias[e] : 0.f);
    }
    const int k = E < 6 ? E : 6;
    if (fixed) {
        for (int i = 0; i < 6; ++i)
            ids[i] = i < k ? fixed[i] : -1;
    } else {
        orc_moe_topk(choice, E, k, ids, w, score);
        for (int i = k; i < 6; ++i)
            ids[i] = -1;
    }
    float sum = 0.f;
    for (int i = 0; i < 6; ++i) {
        const int e = ids[i];
        float v = (e >= 0 && e < E) ? score[e] : 0.f;
        if (v < 0.f)
            v = 0.f;
        w[i] = v;
        sum += v;
    }
    for (int i = 0; i < 6; ++i) {
        if (i >= k) {
            w[i] = 0.f;
            continue;
        }
        w[i] = (sum > 0.f ? w[i] / sum : 1.f / (float)k) * routed_scale;
    }
    free(logits);
    return 1;
}

/* One expert, dsv4_cuda::one_expert (dsv4_cuda.cpp:169-189):
 * g = gate . x, u = up . x ([O]), h = clamped_swiglu(g, u, limit),
 * d = down . h ([H]), y[i] += weight * d[i].  fp8 = 0: MXFP4 tensors
 * (quant::matmul_mxfp4); 1: FP8 tiles. */
static void dsv4_one_expert(int fp8, int H, int O, const void *gw, const void *gs, const void *uw,
                            const void *us, const void *dw, const void *ds, float weight,
                            float limit, float *y, const float *x) {
    float *g = (float *)malloc(sizeof(float) * ((size_t)O * 2 + (size_t)H));
    float *u = g + O, *d = u + O;
    if (fp8) {
        orc_matmul_fp8_b128(g, x, gw, gs, 1, H, O);
        orc_matmul_fp8_b128(u, x, uw, us, 1, H, O);
    } else {
        orc_matmul_mxfp4(g, x, gw, gs, 1, H, O);
        orc_matmul_mxfp4(u, x, uw, us, 1, H, O);
    }
    for (int i = 0; i < O; ++i)
        g[i] = orc_clamped_swiglu(g[i], u[i], limit);
    if (fp8)
        orc_matmul_fp8_b128(d, g, dw, ds, 1, O, H);
    else
        orc_matmul_mxfp4(d, g, dw, ds, 1, O, H);
    for (int i = 0; i < H; ++i)
        y[i] += weight * d[i];
    free(g);
}

/* dsv4_cuda::moe (dsv4_cuda.cpp:812-848): y = 0; the n MXFP4 experts in order
 * (expert_group; n <= 0 is the reference's false), then, when all six shared
 * pointers are given (gate, gate scales, up, up scales, down, down scales;
 * FP8 tiles), y[i] += sh[i] with sh = expert_fp8(x) (one_expert with weight 1
 * from zero, :826-832). */
EXPORT int orc_dsv4_moe(const float *x, int H, int O, int n, const void *const *g,
                        const void *const *u, const void *const *d, const void *const *gs,
                        const void *const *us, const void *const *ds, const float *weights,
                        const void *const *sh, float limit, float *y) {
    if (!x || !y || !weights || n <= 0 || H <= 0 || O <= 0)
        return 0;
    for (int i = 0; i < H; ++i)
        y[i] = 0.f;
    for (int e = 0; e < n; ++e)
        dsv4_one_expert(0, H, O, g[e], gs[e], u[e], us[e], d[e], ds[e], weights[e], limit, y, x);
    if (sh) {
        float *s = (float *)calloc((size_t)H, sizeof(float));
        dsv4_one_expert(1, H, O, sh[0], sh[1], sh[2], sh[3], sh[4], sh[5], 1.f, limit, s, x);
        for (int i = 0; i < H; ++i)
            y[i] += s[i];
        free(s);
    }
    return 1;
}

/* map_ep_expert (dsv4_cuda.cpp:1356-1369): the bank slot serving global id e
 * on the rank of parity r, or -1: e itself when present, else e / 2 (a bank
 * packed per rank). */
static int dsv4_map_ep(const void *const *g, int E, int e, int r) {
    if (e < 0 || e % 2 != r)
        return -1;
    if (e < E && g[e])
        return e;
    if (e / 2 < E && g[e / 2])
        return e / 2;
    return -1;
}

/* dsv4_cuda::route_moe_ep2 (dsv4_cuda.cpp:1841-1906) for one token with one
 * expert bank serving both ranks (local == peer, peer_input == input): route
 * once per rank, rank r runs the routed slots whose expert id has parity r
 * (map_ep_expert, :1356-1369) through moe_routed_parity (:1371-1404), the
 * shared expert (if given) on rank 0 only, then allreduce_pair
 * (:1195-1204): out = peer_out = rank0 + rank1.  Experts with a NULL gate
 * pointer are absent from the bank and skipped. */
EXPORT int orc_dsv4_route_moe_ep2(const float *x, int H, const float *router, const float *bias,
                                  int E, float routed_scale, int O, const void *const *g,
                                  const void *const *u, const void *const *d,
                                  const void *const *gs, const void *const *us,
                                  const void *const *ds, const void *const *sh, float limit,
                                  float *out, float *peer_out) {
    int ids[6];
    float w[6];
    if (!orc_dsv4_route(x, H, router, bias, E, NULL, routed_scale, ids, w))
        return 0;
    float *part[2] = {out, peer_out};
    for (int r = 0; r < 2; ++r) {
        const void *pg[6], *pu[6], *pd[6], *pgs[6], *pus[6], *pds[6];
        float pw[6];
        int n = 0;
        for (int k = 0; k < 6; ++k) {
            const int l = dsv4_map_ep(g, E, ids[k], r);
            if (l < 0 || !u[l] || !d[l])
                continue;
            pg[n] = g[l];
            pu[n] = u[l];
            pd[n] = d[l];
            pgs[n] = gs[l];
            pus[n] = us[l];
            pds[n] = ds[l];
            pw[n] = w[k];
            ++n;
        }
        const void *const *rsh = r == 0 ? sh : NULL;
        if (n > 0) {
            orc_dsv4_moe(x, H, O, n, pg, pu, pd, pgs, pus, pds, pw, rsh, limit, part[r]);
        } else {
            for (int i = 0; i < H; ++i)
                part[r][i] = 0.f;
            if (rsh) /* the shared expert's output copied in */
                dsv4_one_expert(1, H, O, rsh[0], rsh[1], rsh[2], rsh[3], rsh[4], rsh[5], 1.f,
                                limit, part[r], x);
        }
    }
    for (int i = 0; i < H; ++i) {
        const float s = out[i] + peer_out[i];
        out[i] = s;
        peer_out[i] = s;
    }
    return 1;
}
