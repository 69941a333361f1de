// eacs_common.cuh -- shared device helpers for the EACS sm_100a kernels.
//
// Complex arithmetic on float2 (complex64 layout), the ZOH discretisation of
// one (h, n) chain, warp reductions, the device status word, and the
// TMA / mbarrier PTX wrappers.  Every spin-wait here is bounded: on expiry the
// kernel records EACS_ERR_TIMEOUT in the status word and returns.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/eacs_b200.h"

namespace eacs {

// ----------------------------------------------------------------------------
// device status word.  Each translation unit has its own copy (internal
// linkage, no relocatable device code); eacs_device_status() reads and clears
// all of them through the per-unit accessors declared in eacs_host.h.
// ----------------------------------------------------------------------------
static __device__ int g_status;

// Host side: copy this unit's status word to *out and clear it (synchronous on
// `stream`).
static inline cudaError_t read_clear_status(int* out, cudaStream_t stream) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

__device__ __forceinline__ void set_status(int code) { atomicCAS(&g_status, 0, code); }

// ----------------------------------------------------------------------------
// complex64 helpers (float2: x = real, y = imag)
// ----------------------------------------------------------------------------
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
// Re(c * h)
__device__ __forceinline__ float cre_mul(float2 c, float2 h) { return c.x * h.x - c.y * h.y; }
// 1/lam as conj(lam)/|lam|^2
__device__ __forceinline__ float2 crecip(float2 z) {
    float d = z.x * z.x + z.y * z.y;
    return make_float2(z.x / d, -z.y / d);
}

// sin and cos of x.  Cody & Waite range reduction, x = k pi/2 + r, with a
// three-part float split of pi/2 applied by FMA, then the Taylor series of
// sin to r^9 and cos to r^10 on |r| <= pi/4 (truncation below 2.5e-9
// relative) and the quadrant rotation by k mod 4.  Beyond |x| = 8192 the
// three-part split loses accuracy, so CUDA's sincosf (Payne-Hanek reduction)
// takes over.
__device__ __forceinline__ void sincos_cw(float x, float& s, float& c) {
    if (fabsf(x) > 8192.0f) {
        sincosf(x, &s, &c);
        return;
    }
    const float q = rintf(x * 0.636619772f);  // 2/pi
    float r = fmaf(-q, 1.57079637e+00f, x);   // pi/2 = hi + mid + lo
    r = fmaf(-q, -4.37113883e-08f, r);
    r = fmaf(-q, -1.71512451e-15f, r);
    const int k = __float2int_rn(q);
    const float r2 = r * r;
    // sin r = r + r^3 (-1/3! + r^2 (1/5! + r^2 (-1/7! + r^2 / 9!)))
    float ps = fmaf(r2, 2.75573192e-06f, -1.98412698e-04f);
    ps = fmaf(r2, ps, 8.33333333e-03f);
    ps = fmaf(r2, ps, -1.66666667e-01f);
    const float sr = fmaf(r * r2, ps, r);
    // cos r = 1 + r^2 (-1/2! + r^2 (1/4! + r^2 (-1/6! + r^2 (1/8! - r^2 / 10!))))
    float pc = fmaf(r2, -2.75573192e-07f, 2.48015873e-05f);
    pc = fmaf(r2, pc, -1.38888889e-03f);
    pc = fmaf(r2, pc, 4.16666667e-02f);
    pc = fmaf(r2, pc, -0.5f);
    const float cr = fmaf(r2, pc, 1.0f);
    const float ss = (k & 1) ? cr : sr;
    const float cc = (k & 1) ? sr : cr;
    s = (k & 2) ? -ss : ss;
    c = ((k + 1) & 2) ? -cc : cc;
}

// expm1(a) and exp(a) together by Tang's table-free method: a = k ln2 + r with
// a two-part float ln2 applied by FMA, |r| <= ln2/2, expm1(r) from its Taylor
// series to r^8 (truncation below 1e-9 relative), then
// e^a - 1 = 2^k expm1(r) + (2^k - 1) and e^a = 2^k expm1(r) + 2^k.
// Below a = -87 the results are exactly -1 and 0, as float expm1 gives there.
__device__ __forceinline__ void expm1_exp(float a, float& em1, float& ea) {
    const float ac = fminf(fmaxf(a, -87.0f), 88.0f);
    const float k = rintf(ac * 1.44269502f);  // log2(e)
    float r = fmaf(-k, 6.93147182e-01f, ac);   // ln2 = hi + lo
    r = fmaf(-k, -1.90465421e-09f, r);
    float p = fmaf(r, 2.48015873e-05f, 1.98412698e-04f);  // 1/8!, 1/7!
    p = fmaf(r, p, 1.38888889e-03f);                      // 1/6!
    p = fmaf(r, p, 8.33333333e-03f);                      // 1/5!
    p = fmaf(r, p, 4.16666667e-02f);                      // 1/4!
    p = fmaf(r, p, 1.66666667e-01f);                      // 1/3!
    p = fmaf(r, p, 0.5f);                                 // 1/2!
    p = fmaf(r * r, p, r);                                // expm1(r)
    const float s2k = __int_as_float((__float2int_rn(k) + 127) << 23);
    em1 = fmaf(s2k, p, s2k - 1.0f);
    ea = fmaf(s2k, p, s2k);
    if (a < -87.0f) {
        em1 = -1.0f;
        ea = 0.0f;
    }
    if (a != a) em1 = ea = a;  // NaN in, NaN out
}

// Zero-order-hold kernels of one chain (discretization.py:20-36):
//   z = lam * dt,  dA = e^z,  dB_bar = expm1(z) / lam
// with expm1(z) = (expm1(a) cos b - 2 sin^2(b/2), e^a sin b), the branch-free
// form of discretization.py:10-17.  sin b and cos b come from the half angle
// (sin b = 2 s c, cos b = 1 - 2 s^2 with s, c = sin, cos of b/2), so one
// sincos evaluation serves all three trigonometric terms.
__device__ __forceinline__ void zoh(float2 lam, float2 ilam, float dte, float2& dA, float2& dBbar) {
    const float a = lam.x * dte;
    const float b = lam.y * dte;
    float em1, ea;
    expm1_exp(a, em1, ea);
    float s, c;
    sincos_cw(0.5f * b, s, c);
    const float s2 = s + s;
    const float sb = s2 * c;
    const float cb = fmaf(-s2, s, 1.0f);
    const float im = ea * sb;
    dA = make_float2(ea * cb, im);
    const float2 E = make_float2(fmaf(em1, cb, -(s2 * s)), im);
    dBbar = cmul(E, ilam);
}

// effective_dt (discretization.py:63-82): clamp(delta * scale, dt_min, dt_max)
__device__ __forceinline__ float eff_dt(float delta, float scale, float dt_min, float dt_max) {
    return fminf(fmaxf(delta * scale, dt_min), dt_max);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ----------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk[.tensor]) wrappers.  No cluster multicast.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase.  Returns false (and records a timeout)
// when the phase has not completed after `limit` polls.
constexpr uint32_t kWaitLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    set_status(EACS_ERR_TIMEOUT);
    return false;
}

// 3-D tiled TMA load global -> shared, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ----------------------------------------------------------------------------
// warp helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace eacs
