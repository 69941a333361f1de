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

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// e^a, 2 e^a and e^a - 1.  2 e^a = 2^(a log2(e) + 1) from the hardware
// base-2 exponential (about 2^-22 relative; for a <= 0 the argument's
// rounding adds at most 2^-25 absolute, 2.1e-8 relative to the result), so
// the factor 2 costs no multiply, and e^a as its exact half.  e^a - 1 from it
// when |a| >= 0.35, where the subtraction loses at
// most a factor 2.4 of that (a = Re(lam) dt <= 0: 6e-7 relative at a = -0.35),
// and below from the Taylor series of expm1 to a^6 (alternating for a < 0, so
// the error is under the first dropped term, |a|^7/7! / |expm1(a)| < 4.3e-7
// at a = -0.35 and shrinking fast below), which keeps small |a| -- the slow
// modes, where dB_bar ~ dt -- relatively exact.
__device__ __forceinline__ void expm1_exp(float a, float& em1, float& ea, float& ea2) {
    ea2 = ex2_approx(fmaf(a, 1.44269504f, 1.0f));  // log2(e)
    ea = 0.5f * ea2;
    float p = fmaf(a, 1.38888889e-03f, 8.33333333e-03f);  // 1/6!, 1/5!
    p = fmaf(a, p, 4.16666667e-02f);                      // 1/4!
    p = fmaf(a, p, 1.66666667e-01f);                      // 1/3!
    p = fmaf(a, p, 0.5f);                                 // 1/2!
    p = fmaf(a * a, p, a);
    em1 = fabsf(a) < 0.35f ? p : ea - 1.0f;
}

// s = sin h and c = cos h of the reduced half angle h = b/2 - pi k (both
// carry the sign (-1)^k, which cancels in s c and s^2).
// Cody & Waite reduction bh = pi k + h with a two-part float split of pi
// applied by FMA (|h| <= pi/2; each FMA rounds once; the dropped third part
// of pi, 3.4e-15, adds 3.4e-15 |k| to h, under 1e-7 of |h| unless
// |h| < 3.4e-8 |k|); the constants are the exact halves of a split of 2 pi,
// so h is bit for bit half of the full-angle remainder b - 2 pi k.  Then:
// s = sin h from its Taylor series to h^11 (truncation below 6e-8 on
// |h| <= pi/2, relative near 0) and c = cos h from the hardware cosine
// (absolute error about 2^-21 on [-pi, pi]).  The caller forms sin b = 2 s c,
// 1 - cos b = 2 s^2; every error term is proportional to s, so expm1(z) built
// from these keeps its relative accuracy as |z| -> 0.  Branch-free, so
// unrolled steps and chains interleave.
__device__ __forceinline__ void trig_half(float bh, float& s, float& c) {
    constexpr float kInvPi = 2.0f * 0.159154943f;    // 2 / (2 pi)
    constexpr float kPiHi = 0.5f * 6.28318548e+00f;  // (2 pi = hi + mid) / 2
    constexpr float kPiMid = 0.5f * -1.74845553e-07f;
    const float k = rintf(bh * kInvPi);
    float h = fmaf(-k, kPiHi, bh);
    h = fmaf(-k, kPiMid, h);
    const float h2 = h * h;
    // sin h = h + h^3 (-1/3! + h^2 (1/5! + h^2 (-1/7! + h^2 (1/9! - h^2/11!))))
    float ps = fmaf(h2, -2.50521084e-08f, 2.75573192e-06f);
    ps = fmaf(h2, ps, -1.98412698e-04f);
    ps = fmaf(h2, ps, 8.33333333e-03f);
    ps = fmaf(h2, ps, -1.66666667e-01f);
    s = fmaf(h * h2, ps, h);
    c = __cosf(h);
}

// Zero-order-hold kernels of one chain (discretization.py:20-36):
//   z = lam * dt,  dA = e^z,  dB_bar = expm1(z) / lam
// with expm1(z) = (expm1(a) cos b - 2 sin^2(b/2), e^a sin b), the branch-free
// form of discretization.py:10-17, here as (expm1(a) - 2 e^a s^2, 2 e^a s c)
// and e^z = (e^a - 2 e^a s^2, 2 e^a s c) with s, c the half-angle sine and
// cosine (cos b = 1 - 2 s^2, sin b = 2 s c).
// zoh_e returns expm1(z) itself (E, with dB_bar = E / lam), for callers that
// fold 1/lam into the input term.
__device__ __forceinline__ void zoh_e(float2 lam, float dte, float2& dA, float2& E) {
    const float a = lam.x * dte;
    // b/2 = (Im(lam)/2) dt, exactly half of Im(lam) dt; callers that keep lam
    // in registers across steps compute Im(lam)/2 once
    const float bh = (0.5f * lam.y) * dte;
    float em1, ea, ea2, s, c;
    expm1_exp(a, em1, ea, ea2);
    trig_half(bh, s, c);
    const float t = s * s;
    const float im = (ea2 * s) * c;
    dA = make_float2(fmaf(-ea2, t, ea), im);
    E = make_float2(fmaf(-ea2, t, em1), im);
}
__device__ __forceinline__ void zoh(float2 lam, float2 ilam, float dte, float2& dA, float2& dBbar) {
    float2 E;
    zoh_e(lam, dte, dA, E);
    dBbar = cmul(E, ilam);
}

// a * b + c for complex a, b, c (four FMAs)
__device__ __forceinline__ float2 cfma(float2 a, float2 b, float2 c) {
    return make_float2(fmaf(a.x, b.x, fmaf(-a.y, b.y, c.x)), fmaf(a.x, b.y, fmaf(a.y, b.x, c.y)));
}

// ----------------------------------------------------------------------------
// warp reductions of several sums at once
// ----------------------------------------------------------------------------
// Transposed butterfly over the lane offsets O, O/2, ..., S.  A lane enters
// with V partial sums; at each level while V > M it keeps half and trades the
// other half with its partner (V-M shuffles for V sums down to M); once M
// values are left the remaining levels are plain reductions of all M.
template <int V, int O, int S, int M = 1>
struct Fold {
    static __device__ __forceinline__ void run(float* v, int lane) {
        if constexpr (O >= S && O > 0) {
            if constexpr (V <= M) {
#pragma unroll
                for (int k = 0; k < V; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], O);
                Fold<V, O / 2, S, M>::run(v, lane);
            } else {
                const bool up = (lane & O) != 0;
#pragma unroll
                for (int k = 0; k < V / 2; ++k) {
                    const float send = up ? v[k] : v[k + V / 2];
                    const float keep = up ? v[k + V / 2] : v[k];
                    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, O);
                }
                Fold<V / 2, O / 2, S, M>::run(v, lane);
            }
        }
    }
};

template <int V, int O, int S, int M = 1>
struct FoldShape {
    static constexpr int levels(int v, int o) { return (o < S || o == 0 || v <= M) ? 0 : 1 + levels(v / 2, o / 2); }
    static constexpr int kHalve = levels(V, O);
    static constexpr int kRem = V >> kHalve;  // sums a lane holds afterwards
    // first original index of the sums lane `lane` holds
    static __device__ __forceinline__ int held(int lane) {
        int idx = 0;
#pragma unroll
        for (int j = 0; j < kHalve; ++j)
            if (lane & (O >> j)) idx += V >> (j + 1);
        return idx;
    }
    // one lane per distinct set of sums: the bits of the plain levels are zero
    static __device__ __forceinline__ bool writer(int lane) {
        bool w = true;
#pragma unroll
        for (int o = O >> kHalve; o >= S && o > 0; o >>= 1) w = w && !(lane & o);
        return w;
    }
};

// effective_dt (discretization.py:63-82): clamp(delta * scale, dt_min, dt_max)
__device__ __forceinline__ float eff_dt(float delta, float scale, float dt_min, float dt_max) {
    return fminf(fmaxf(delta * scale, dt_min), dt_max);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ----------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk[.tensor]) wrappers; every copy targets this
// CTA's own shared memory from this GPU's memory.
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
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t limit = kWaitLimit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    set_status(EACS_ERR_TIMEOUT);
    return false;
}

// Bounded wait on an mbarrier phase completed by other CTAs of the cluster
// (acquire at cluster scope, so their st.async data is visible afterwards).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t phase, uint32_t limit = kWaitLimit) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    set_status(EACS_ERR_TIMEOUT);
    return false;
}

// The same bounded wait by polling with mbarrier.test_wait, which never
// suspends the thread (try_wait may suspend it for a system-dependent time).
__device__ __forceinline__ bool mbar_poll_cluster(uint64_t* bar, uint32_t phase, uint32_t limit = kWaitLimit) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    set_status(EACS_ERR_TIMEOUT);
    return false;
}

// Wait used by the cluster reductions of the repair and training passes.
#ifndef EACS_MBAR_POLL
#define EACS_MBAR_POLL 0
#endif
__device__ __forceinline__ bool mbar_wait_row(uint64_t* bar, uint32_t phase, uint32_t limit = kWaitLimit) {
#if EACS_MBAR_POLL
    return mbar_poll_cluster(bar, phase, limit);
#else
    return mbar_wait_cluster(bar, phase, limit);
#endif
}

// Address of `local` in the shared memory of CTA `cta` of this cluster.
__device__ __forceinline__ uint32_t mapa_u32(const void* local, int cta) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(cta));
    return ra;
}

// Store a float into another CTA's shared memory, counting 4 bytes of
// transaction on that CTA's mbarrier (both addresses from mapa_u32).
__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
                 "r"(__float_as_uint(v)), "r"(rbar)
                 : "memory");
}

// Asynchronous global -> shared copies of 4 or 8 bytes (cp.async); with
// `valid` false nothing is read and the destination is zero-filled.
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

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
