// common.cuh -- device helpers shared by the sm_100a kernels of the MoE block.
//
// Everything here is a thin wrapper over one PTX instruction (mbarrier, bulk
// copy, conversion, mma) or a bounded wait built from them.  Every wait in
// this library is bounded: after kWaitNs of %globaltimer (or an iteration
// cap) it records MVLLM_ERR_TIMEOUT in the launch's error word and returns
// false, so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h> // CUtensorMap (header only; the driver entry point is fetched at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mvllm_moe.h"

namespace mvb {

constexpr uint64_t kWaitNs = 2000000000ull; // 2 s: far above any legitimate stall
constexpr uint32_t kWaitIters = 1u << 28;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream serialization attribute may start while the kernel before it on the
// stream is still finishing; it waits here, before reading anything that
// kernel wrote, until the earlier grid has completed and its writes are
// visible.  Without the attribute this returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream (launched with programmatic stream
// serialisation) start its prologue once every CTA of this grid issued it;
// that kernel's griddepcontrol.wait still waits for this grid to complete.
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Records the first error code of a launch (later codes do not overwrite it).
__device__ __forceinline__ void set_error(int *err, int code) {
    if (err)
        atomicCAS(err, 0, code);
}

__device__ __forceinline__ int load_volatile(const int *p) {
    return *reinterpret_cast<const volatile int *>(p);
}

// A finite value the f16 operands cannot hold (it would round to inf).
__device__ __forceinline__ bool beyond_f16(float v) {
    const float a = fabsf(v);
    return a >= 65520.f && a <= 3.402823466e38f;
}

// Token tiles of an expert with c rows: full tiles of 2^tshift rows (256
// for tc_ffn's pairs, 128 for the block-scaled kernel's) and the rest; the
// rest runs on single CTAs when it has at most kTcSoloMax rows (small_max),
// else as one more (narrower) pair tile.
__host__ __device__ __forceinline__ void tc_tiles(int c, int small_max, int tshift, int &npair,
                                                  int &nsolo) {
    const int f = c >> tshift, r = c & ((1 << tshift) - 1);
    npair = f + (r > small_max ? 1 : 0);
    nsolo = (r > 0 && r <= small_max) ? 1 : 0;
}

// The same split with a third form: a rest of more than small_max and at
// most wide_max rows runs as one wide single-CTA tile (tc_ffn's one-CTA-per-SM
// form); wide_max <= small_max leaves it out.
__host__ __device__ __forceinline__ void tc_tiles3(int c, int small_max, int wide_max, int tshift,
                                                   int &npair, int &nsolo, int &nwide) {
    const int f = c >> tshift, r = c & ((1 << tshift) - 1);
    const int top = wide_max > small_max ? wide_max : small_max;
    npair = f + (r > top ? 1 : 0);
    nsolo = (r > 0 && r <= small_max) ? 1 : 0;
    nwide = (r > small_max && r <= top) ? 1 : 0;
}

// Largest e with off[e] <= i, for off non-decreasing and off[nb] > i.
__device__ __forceinline__ int find_owner(const int *off, int nb, int i) {
    int lo = 0, hi = nb;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(off + mid) <= i)
            lo = mid;
        else
            hi = mid;
    }
    return lo;
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up (and
// records a timeout) after kWaitNs, or at once when another thread of the
// launch has already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1; it < kWaitIters; ++it) {
        if (mbar_try_wait(bar, parity))
            return true;
        if ((it & 31u) == 0) {
            if (err && load_volatile(err) != 0)
                return false;
            if (globaltimer_ns() - t0 > kWaitNs)
                break;
        }
    }
    set_error(err, MVLLM_ERR_TIMEOUT);
    return false;
}

// ---- bulk copy (TMA engine, non-tensor form; never multicast) ---------------
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
                 "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
                 : "memory");
}

// 16-byte Ampere-style async copy global -> shared (L2 only, bypassing L1).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}

// One arrival on `bar` once every cp.async this thread issued before has
// landed (the barrier's expected count must include this arrival).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// ---- tensor TMA (2-D tiles, never multicast) -------------------------------
// Box load described by a tensor map in global or param space; x is the
// innermost coordinate (its byte offset must be a multiple of 16).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
                 ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
                 "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
                 : "memory");
}

// 3-D box, coordinates innermost first.
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes"
                 ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
                 "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
                 : "memory");
}

// Writer side of a device-built tensor map: swap the global address of a
// 128-byte map in global memory, then release it to the tensormap proxy.
__device__ __forceinline__ void tmap_replace_address(void *tmap, const void *addr) {
    asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(tmap),
                 "l"(addr)
                 : "memory");
}
__device__ __forceinline__ void tmap_release() {
    asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
}
// Reader side: acquire a map written through the generic proxy before use.
__device__ __forceinline__ void tmap_acquire(const void *tmap) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier over `count` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- shared / global loads ---------------------------------------------------
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

// Streaming 16-byte read-only load that does not pollute L1.
__device__ __forceinline__ uint4 ldg_stream128(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---- conversions ---------------------------------------------------------------
// Four bytes of packed e2m1 pairs -> four f16x2 (low nibble -> low half).
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t &h0, uint32_t &h1,
                                                uint32_t &h2, uint32_t &h3) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}\n"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
        : "r"(w));
}

// Eight offset-8 int4 codes -> four f16x2 holding (code - 8), exact.
// Output pairs are (k0,k4), (k1,k5), (k2,k6), (k3,k7) for nibbles k0..k7 of w
// (k0 = bits 0..3): 0x6400 | n is the f16 1024 + n, and 1032 is subtracted.
__device__ __forceinline__ void int4x8_to_f16x8(uint32_t w, uint32_t &h0, uint32_t &h1,
                                                uint32_t &h2, uint32_t &h3) {
    const uint32_t magic = 0x64006400u, mask = 0x000F000Fu, bias = 0x64086408u; // 1032
    uint32_t t0, t1, t2, t3;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(t0) : "r"(w), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(t1) : "r"(w >> 4), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(t2) : "r"(w >> 8), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(t3) : "r"(w >> 12), "r"(mask), "r"(magic));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(h0) : "r"(t0), "r"(bias));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(h1) : "r"(t1), "r"(bias));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(h2) : "r"(t2), "r"(bias));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(h3) : "r"(t3), "r"(bias));
}

// ue8m0 code -> 2^(s-127) as the reference decodes it: s in the f32 exponent
// field, so 0 -> +0 and 255 -> +inf.
__device__ __forceinline__ float ue8m0_to_f32(uint32_t s) { return __uint_as_float(s << 23); }

// ---- warp-level MMA (m16n8k16, f16 in, f32 accumulate) ------------------------
// Not volatile: a pure function of its operands, so the compiler may
// interleave it with the next group's loads and conversions.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1, const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
                   "f"(c[2]), "f"(c[3]));
}

// d0,d1 += a0,a1 * s with one packed f32x2 FMA (sm_100).
__device__ __forceinline__ void ffma2(float &d0, float &d1, float a0, float a1, float s) {
    asm("{\n\t.reg .b64 acc, av, sv;\n\t"
        "mov.b64 acc, {%0, %1};\n\t"
        "mov.b64 av, {%2, %3};\n\t"
        "mov.b64 sv, {%4, %4};\n\t"
        "fma.rn.f32x2 acc, av, sv, acc;\n\t"
        "mov.b64 {%0, %1}, acc;\n\t}\n"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(s));
}

// Byte k of w as a ue8m0 scale (2^(b-127), the reference's decoding).
__device__ __forceinline__ float ue8m0_byte(uint32_t w, int k) {
    return __uint_as_float(__byte_perm(w, 0u, 0x4440u | static_cast<uint32_t>(k)) << 23);
}

// ---- activations (metal_ops.cpp:197-211, quant.hpp:22-50) ---------------------
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.f)
        return 1.f / (1.f + expf(-x));
    const float z = expf(x);
    return z / (1.f + z);
}

__device__ __forceinline__ float apply_act(float g, float u, int act, float a, float b) {
    if (act == MVLLM_ACT_CLAMP_SWIGLU) {
        if (a > 0.f && g > a)
            g = a;
        const float s = g * sigmoid_ref(g);
        if (a > 0.f) {
            if (u > a)
                u = a;
            if (u < -a)
                u = -a;
        }
        return s * u;
    }
    if (act == MVLLM_ACT_SITU)
        return a * tanhf(g / a) * sigmoid_ref(g) * b * tanhf(u / b);
    return g * sigmoid_ref(g) * u;
}

// The same activations from the SFU's approximate tanh and exp2 (PTX
// tanh.approx.f32 and ex2.approx.f32, relative errors near 2^-11 and 2^-22)
// and an approximate reciprocal.  The result is rounded to f16 (2^-11)
// anyway; the tensor-core epilogue, which evaluates one activation per
// output element and token, uses these so that it keeps pace with the MMAs.
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float sigmoid_fast(float x) {
    // 1 / (1 + e^-x) with e^-x = 2^(-x log2 e); saturates to 0 / 1 at the ends.
    float t, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(-1.4426950408889634f * x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + t));
    return r;
}
// ia, ib: 1/a and 1/b, computed once per launch by the caller.
__device__ __forceinline__ float apply_act_fast(float g, float u, int act, float a, float b,
                                                float ia, float ib) {
    if (act == MVLLM_ACT_CLAMP_SWIGLU) {
        if (a > 0.f && g > a)
            g = a;
        const float s = g * sigmoid_fast(g);
        if (a > 0.f) {
            if (u > a)
                u = a;
            if (u < -a)
                u = -a;
        }
        return s * u;
    }
    if (act == MVLLM_ACT_SITU)
        return a * tanh_fast(g * ia) * sigmoid_fast(g) * b * tanh_fast(u * ib);
    return g * sigmoid_fast(g) * u;
}

// Position of source column k inside the f16 operand layout of a format.
// MXFP4 keeps natural order; int4-g64 interleaves each aligned 8-chunk as
// k0,k4,k1,k5,k2,k6,k3,k7 to match int4x8_to_f16x8's pair order.
__device__ __forceinline__ int stage_pos(int k, int fmt) {
    if (fmt != MVLLM_FMT_INT4_G64)
        return k;
    const int j = k & 7;
    return (k & ~7) | ((j & 3) << 1) | (j >> 2);
}

} // namespace mvb
