// Layer epilogue after the routed combine, tolerance mode: the step both
// callers take after moe_block (kimi_k3.cpp:2074-2108, glm53.cpp:1993-2027):
//
//   a = acc[c]; if lat_n: a = rmsnorm(a, lat_n, eps) (quant.cpp:384-398)
//   u = a . W_up^T (QuantMat int8-row: (sum a.q) * scale[o], quant.cpp:255-268)
//   h[c] += u * routed_scale; if shared: h[c] += shared[c]
//
// in two kernels.  The exact path (aux_kernels.cuh: serial rmsnorm, the
// reference's sequential dot products) stays for the bit-exact mode; this one
// is held to the library's tolerance (<= 1e-2 relative L2, <= 2e-2 max-abs)
// and is bound by the W_up stream (H x L int8 bytes + H scales).
//
// epilogue_stage_kernel: a CTA per token row: rmsnorm, the row scaled by a
// power of two (below), f16 rows [T][L] plus 1/sigma per row in the workspace.
//
// epilogue_up_kernel: each CTA owns RB blocks of 16 W_up rows; its 16 warps
// are RB row blocks x KSL slices of L (at most 8 chunks of 64 = 512 latent
// columns each).  A warp requests its first four W_up chunks (2 x 16 bytes
// per lane per chunk, the HBM stream of the kernel) before waiting for the
// staging kernel (programmatic dependent launch); the staged rows of a token
// group (32 rows, 4 n-tiles) then arrive in shared memory by bulk copies, and
// the warp runs mma.m16n8k16 (f16 x f16 -> f32) over its slice with four
// chunks in flight: int8 codes are exact in f16.  Later token groups re-read
// W_up from L2.
//
// K order inside a 64-column chunk: lane (g, c) holds bytes 16c..16c+15 of
// rows g and g+8 (one 16-byte load each); MMA step j of the chunk reads the
// 4 bytes 16c+4j..16c+4j+3 as its k slots {2c, 2c+1, 2c+8, 2c+9}.  The token
// operand uses the same order (an 8-byte shared load per step), so the dot
// product covers every column once.
//
// Range: each token row is scaled by a power of two sigma_t so that its
// largest |value| lies in [2^13, 2^14) before the f16 rounding (no overflow,
// no f16 subnormals), and the sums are multiplied by 1/sigma_t (exact).
// Slices are summed in ascending order from shared memory: run-to-run
// identical.
#pragma once

#include "common.cuh"

namespace mvb {

constexpr int kEpiWarps = 16;
constexpr int kEpiTok = 32;   // tokens per group
constexpr int kEpiCpw = 8;    // 64-column chunks per warp slice
constexpr int kEpiRedPitch = 40; // floats per (row, group) partial line

struct EpiArgs {
    const float *acc;    // [T, L] routed sums
    const float *lat_n;  // [L] rmsnorm weight, or null (no norm)
    float eps;
    const int8_t *q;     // W_up int8 codes [H, L]
    const float *qs;     // [H] row scales
    float routed_scale;
    const float *shared; // [T, H] or null
    float *h;            // [T, H] accumulated
    int T, H, L;
};

// Slices of L per row block: the power of two covering L / 512.
__host__ __device__ inline int epi_ksl(int L) {
    const int need = (L + kEpiCpw * 64 - 1) / (kEpiCpw * 64);
    int k = 1;
    while (k < need)
        k <<= 1;
    return k;
}

__host__ __device__ inline size_t epi_smem_bytes(int L) {
    return size_t(kEpiTok) * (2 * L + 16) + size_t(kEpiWarps) * 16 * kEpiRedPitch * 4 +
           kEpiTok * 4 + 16;
}

// Workspace of the two kernels: f16 rows [T][L] then 1/sigma per row.
__host__ __device__ inline size_t epi_ws_bytes(int T, int L) {
    return size_t(T) * L * 2 + size_t(T) * 4;
}

// Signed int8 x4 -> two f16x2 (bytes 0,1 and bytes 2,3), exact: byte ^ 0x80
// in the low mantissa bits of 1024.0 gives 1024 + (b + 128); 1152 is taken off.
__device__ __forceinline__ void s8x4_to_f16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t x = w ^ 0x80808080u;
    const uint32_t t0 = __byte_perm(x, 0x64646464u, 0x5140u);
    const uint32_t t1 = __byte_perm(x, 0x64646464u, 0x7362u);
    const uint32_t bias = 0x64806480u; // 1152, 1152
    asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(t0), "r"(bias));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(t1), "r"(bias));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Power of two that puts vmax into [2^13, 2^14); 1 for 0 or a non-finite max.
__device__ __forceinline__ float epi_sigma(float vmax) {
    if (!(vmax > 0.f) || !isfinite(vmax))
        return 1.f;
    int e;
    frexpf(vmax, &e); // vmax = m * 2^e, m in [0.5, 1)
    return ldexpf(1.f, max(-126, min(126, 14 - e)));
}

// A CTA per token row (256 threads): sum of squares and the largest
// |a * lat_n| as block reductions, then the row as f16 of a * inv * lat_n *
// sigma_t, and 1 / sigma_t.
__global__ void __launch_bounds__(256) epilogue_stage_kernel(EpiArgs p, __half *rows,
                                                             float *tinv) {
    __shared__ float part[2][8];
    pdl_wait(); // acc comes from the kernels before this one
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n4 = p.L / 4;
    for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
        const float4 *a4 = reinterpret_cast<const float4 *>(p.acc + size_t(t) * p.L);
        const float4 *w4 = reinterpret_cast<const float4 *>(p.lat_n);
        float ss = 0.f, amax = 0.f;
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 a = a4[i];
            ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
            float4 w = make_float4(1.f, 1.f, 1.f, 1.f);
            if (w4)
                w = w4[i];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x * w.x), fabsf(a.y * w.y)),
                                     fmaxf(fabsf(a.z * w.z), fabsf(a.w * w.w))));
        }
        ss = warp_sum(ss);
        amax = warp_max(amax);
        if (lane == 0)
            part[0][warp] = ss, part[1][warp] = amax;
        __syncthreads();
        float tot = 0.f, mx = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            tot += part[0][k], mx = fmaxf(mx, part[1][k]);
        __syncthreads(); // part[] is rewritten for the next row
        const float inv = p.lat_n ? 1.f / sqrtf(tot / static_cast<float>(p.L) + p.eps) : 1.f;
        const float sigma = epi_sigma(mx * inv);
        const float f = inv * sigma;
        uint2 *dst = reinterpret_cast<uint2 *>(rows + size_t(t) * p.L);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 a = a4[i];
            float4 w = make_float4(1.f, 1.f, 1.f, 1.f);
            if (w4)
                w = w4[i];
            const __half2 lo = __floats2half2_rn(a.x * f * w.x, a.y * f * w.y);
            const __half2 hi = __floats2half2_rn(a.z * f * w.z, a.w * f * w.w);
            uint2 v;
            v.x = *reinterpret_cast<const uint32_t *>(&lo);
            v.y = *reinterpret_cast<const uint32_t *>(&hi);
            dst[i] = v;
        }
        if (threadIdx.x == 0)
            tinv[t] = 1.f / sigma;
    }
}

template <int KSL>
__global__ void __launch_bounds__(kEpiWarps * 32, 1)
    epilogue_up_kernel(EpiArgs p, const __half *rows, const float *tinv_g) {
    constexpr int RB = kEpiWarps / KSL;
    extern __shared__ __align__(16) uint8_t epi_sm[];
    const int pitch = 2 * p.L + 16; // bytes per staged token row
    uint8_t *act = epi_sm;
    float *red = reinterpret_cast<float *>(epi_sm + size_t(kEpiTok) * pitch);
    float *tinv = red + kEpiWarps * 16 * kEpiRedPitch;
    uint64_t *rows_bar = reinterpret_cast<uint64_t *>(tinv + kEpiTok);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int rb = warp / KSL, ks = warp % KSL;
    const int row0 = (blockIdx.x * RB + rb) * 16;
    const bool row_ok = row0 < p.H;
    const int nch = p.L / 64, ch0 = ks * kEpiCpw;

    // W_up chunks stream through a window of five (the chunk in use and four
    // in flight); the first four are requested before waiting for the
    // staging kernel, which they do not depend on.
    auto load_chunk = [&](int i, uint4 (&w)[2]) {
        w[0] = w[1] = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok && i < kEpiCpw && ch0 + i < nch) {
            const int8_t *b = p.q + size_t(row0 + g) * p.L + (ch0 + i) * 64 + 16 * c;
            w[0] = ldg_stream128(b);
            w[1] = ldg_stream128(b + size_t(8) * p.L);
        }
    };
    uint4 w0[2], w1[2], w2[2], w3[2];
    load_chunk(0, w0);
    load_chunk(1, w1);
    load_chunk(2, w2);
    load_chunk(3, w3);
    if (threadIdx.x == 0) {
        mbar_init(rows_bar, 1);
        fence_barrier_init();
    }
    pdl_wait(); // the staged rows, h and shared come from the kernels before this one

    uint32_t rows_phase = 0;
    for (int g0 = 0; g0 < p.T; g0 += kEpiTok) {
        const int ntok = min(kEpiTok, p.T - g0);
        __syncthreads(); // the previous group's shared-memory readers are done
        if (threadIdx.x == 0) {
            // the rows' async-proxy writes follow the generic reads of the
            // previous group
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(rows_bar, uint32_t(ntok) * 2u * uint32_t(p.L));
            for (int tk = 0; tk < ntok; ++tk)
                bulk_g2s(act + size_t(tk) * pitch, rows + size_t(g0 + tk) * p.L,
                         2u * uint32_t(p.L), rows_bar, policy_evict_last());
        }
        for (int tk = ntok + warp; tk < kEpiTok; tk += kEpiWarps) // padding tokens: zeros
            for (int i = lane; i < p.L / 8; i += 32)
                reinterpret_cast<uint4 *>(act + size_t(tk) * pitch)[i] =
                    make_uint4(0u, 0u, 0u, 0u);
        if (threadIdx.x < kEpiTok)
            tinv[threadIdx.x] = threadIdx.x < ntok ? tinv_g[g0 + threadIdx.x] : 0.f;
        const bool landed = mbar_wait(rows_bar, rows_phase, nullptr);
        rows_phase ^= 1u;
        if (!__syncthreads_and(landed ? 1 : 0))
            return; // a bounded wait that gave up: nothing is written
        const int ntv = (ntok + 7) / 8;
        float accv[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r)
                accv[nt][r] = 0.f;
        const uint32_t act_s = smem_u32(act);
        if (g0 > 0) { // the window restarts for every token group (W_up from L2)
            load_chunk(0, w0);
            load_chunk(1, w1);
            load_chunk(2, w2);
            load_chunk(3, w3);
        }
#pragma unroll 1
        for (int i = 0; i < kEpiCpw && ch0 + i < nch; ++i) {
            const uint4 cur0 = w0[0], cur1 = w0[1];
            w0[0] = w1[0], w0[1] = w1[1];
            w1[0] = w2[0], w1[1] = w2[1];
            w2[0] = w3[0], w2[1] = w3[1];
            load_chunk(i + 4, w3);
            const uint32_t q0[4] = {cur0.x, cur0.y, cur0.z, cur0.w};
            const uint32_t q1[4] = {cur1.x, cur1.y, cur1.z, cur1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t a0, a1, a2, a3;
                s8x4_to_f16x4(q0[j], a0, a2);
                s8x4_to_f16x4(q1[j], a1, a3);
                const uint32_t kb = 2u * ((ch0 + i) * 64 + 16 * c + 4 * j);
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    if (nt < ntv) {
                        const uint2 b = lds64(act_s + uint32_t(nt * 8 + g) * pitch + kb);
                        mma_f16_16816(accv[nt], a0, a1, a2, a3, b.x, b.y, accv[nt]);
                    }
                }
            }
        }
        // Partials: red[warp][row][token].
        float *rw = red + warp * 16 * kEpiRedPitch;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const int tk = nt * 8 + 2 * c;
            *reinterpret_cast<float2 *>(rw + g * kEpiRedPitch + tk) =
                make_float2(accv[nt][0], accv[nt][1]);
            *reinterpret_cast<float2 *>(rw + (g + 8) * kEpiRedPitch + tk) =
                make_float2(accv[nt][2], accv[nt][3]);
        }
        __syncthreads();
#pragma unroll 1
        for (int idx = threadIdx.x; idx < RB * 16 * kEpiTok; idx += blockDim.x) {
            const int r16 = idx & 15, rest = idx >> 4;
            const int rbl = rest % RB, tk = rest / RB;
            const int row = (blockIdx.x * RB + rbl) * 16 + r16, t = g0 + tk;
            if (tk >= ntok || row >= p.H)
                continue;
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < KSL; ++k)
                s += red[((rbl * KSL + k) * 16 + r16) * kEpiRedPitch + tk];
            const float u = s * tinv[tk] * p.qs[row];
            const size_t o = size_t(t) * p.H + row;
            float v = p.h[o] + u * p.routed_scale;
            if (p.shared)
                v += p.shared[o];
            p.h[o] = v;
        }
    }
}

// No up-projection (L == H): rmsnorm (when lat_n) and the residual update,
// one CTA per token row, the row's sum of squares as a block reduction.
__global__ void __launch_bounds__(256) epilogue_norm_kernel(EpiArgs p) {
    __shared__ float part[8];
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n4 = p.H / 4;
    for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
        const float4 *a4 = reinterpret_cast<const float4 *>(p.acc + size_t(t) * p.H);
        float inv = 1.f;
        if (p.lat_n) {
            float ss = 0.f;
            for (int i = threadIdx.x; i < n4; i += blockDim.x) {
                const float4 a = a4[i];
                ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
            }
            ss = warp_sum(ss);
            if (lane == 0)
                part[warp] = ss;
            __syncthreads();
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w)
                tot += part[w];
            inv = 1.f / sqrtf(tot / static_cast<float>(p.H) + p.eps);
            __syncthreads(); // part[] is rewritten by the next row
        }
        float4 *h4 = reinterpret_cast<float4 *>(p.h + size_t(t) * p.H);
        const float4 *s4 = p.shared ? reinterpret_cast<const float4 *>(p.shared + size_t(t) * p.H)
                                    : nullptr;
        const float4 *w4 = reinterpret_cast<const float4 *>(p.lat_n);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 a = a4[i];
            float4 w = make_float4(inv, inv, inv, inv);
            if (w4) {
                const float4 ln = w4[i];
                w = make_float4(ln.x * inv, ln.y * inv, ln.z * inv, ln.w * inv);
            }
            float4 v = h4[i];
            v.x += a.x * w.x * p.routed_scale;
            v.y += a.y * w.y * p.routed_scale;
            v.z += a.z * w.z * p.routed_scale;
            v.w += a.w * w.w * p.routed_scale;
            if (s4) {
                const float4 s = s4[i];
                v.x += s.x, v.y += s.y, v.z += s.z, v.w += s.w;
            }
            h4[i] = v;
        }
    }
}

} // namespace mvb
