// project.cu -- EACS layer input projections on the 5th-generation tensor
// cores (sm_100a): LayerNorm -> proj_u / proj_B / proj_C in one kernel.
//
// Semantics: cst_ssm/modules/eacs.py:334 and :376 (x = self.norm(x)) and
// :261-267 (_project: u = proj_u(x), b = proj_B(x), Bc = complex(b[..., :N],
// b[..., N:]), likewise Cc), as they run under a float16 / bfloat16 autocast
// region: LayerNorm in float32, its output rounded to the GEMM type T, the
// GEMM accumulated in float32 with the bias (rounded to T) added, the result
// rounded to T; u is written in the cell's input type, Bc / Cc as complex64
// of the T-rounded values (the reference's .float()).
//
// A first kernel takes each row's LayerNorm statistics (mean and 1/std, one
// warp per row) into the caller's workspace.  The main kernel: one CTA owns
// 128 rows (the MMA's M) and 256 output columns (its N) of [proj_u; proj_B;
// proj_C] stacked as one (Ncat, d) weight.  Everything it reads in bulk comes
// by TMA (cp.async.bulk.tensor, 128-byte swizzle), so the loads run ahead of
// the math through a ring of shared-memory stages with full/empty mbarriers:
//   warp 0      one thread loads, per 64-column k-block, the CTA's x tile and
//               the weight tile into a stage;
//   warp 1      allocates 256 TMEM columns for the float32 accumulator; one
//               thread issues tcgen05.mma (kind::f16, 128 x 256 x 16, four per
//               k-block) and frees each stage with tcgen05.commit;
//   warps 2-5   thread t owns row t: it normalises its row of the x stage
//               (16-bit x in place, as the x tile already sits in the
//               128-byte-swizzled K-major layout the MMA reads; float32 x into
//               a separate A stage), rounded to T; after the last k-block the
//               accumulator row comes back (tcgen05.ld), the bias is added,
//               and u, Bc, Cc are stored.
// Every wait is bounded (EACS_ERR_TIMEOUT in the status word on expiry).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kBM = 128;       // rows per CTA (MMA M)
constexpr int kBN = 256;       // output columns per CTA (MMA N), TMEM columns
constexpr int kBK = 64;        // k-block: 64 16-bit elements = one 128-byte swizzle row
constexpr int kUK = 16;        // K of one tcgen05.mma kind::f16
constexpr int kThreads = 192;  // 6 warps
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kWBytes = kBN * kBK * 2;  // 32 KB
// Stages: 16-bit x is normalised in place (the x stage becomes the A
// stage: same 128 x 128-byte swizzled layout); float32 x has its own 32 KB x
// stage (two 16 KB boxes of 32 columns) beside a 16 KB A stage.
template <typename XT> constexpr bool inplace() { return sizeof(XT) == 2; }
template <typename XT> constexpr uint32_t x_bytes() { return kBM * kBK * sizeof(XT); }
template <typename XT> constexpr uint32_t a_bytes() { return inplace<XT>() ? 0u : kABytes; }
// Two stages per CTA leave room for two CTAs per SM (and two 256-column TMEM
// accumulators), so one CTA's epilogue overlaps the other's main loop:
// 181 against 215 us (four stages, one CTA per SM) at 8 x 4096 rows, d = 768.
#ifndef EACS_PROJ_STAGES
#define EACS_PROJ_STAGES 2
#endif
constexpr int kMaxStages = EACS_PROJ_STAGES;
// Dynamic shared memory for S stages: the stages (1024-aligned), LayerNorm's
// gamma and beta for d rounded up to whole k-blocks, the CTA's bias slice,
// the mbarriers and the TMEM address.
template <typename XT> size_t smem_bytes(int S, int64_t d) {
    const size_t dpad = static_cast<size_t>((d + kBK - 1) / kBK) * kBK;
    return 1024 + S * (x_bytes<XT>() + a_bytes<XT>() + kWBytes) + (2 * dpad + kBN) * sizeof(float) +
           (4 * kMaxStages + 1) * 8 + 16;
}
// The most stages (at most kMaxStages) whose shared memory fits 227 KB; 0 if none.
template <typename XT> int stages_for(int64_t d) {
    for (int S = kMaxStages; S >= 2; --S)
        if (smem_bytes<XT>(S, d) <= 227u * 1024u) return S;
    return 0;
}

struct PArgs {
    const void* x;     // (M, d), x_dtype
    const float2* stats;  // (M) mean, 1/sqrt(var + eps) of each row
    const float* gamma;
    const float* beta;
    const float* bias;  // (Ncat) float32
    void* u;            // (M, H), u_dtype
    float2* Bc;         // (M, N)
    float2* Cc;
    int M, d, H, N, Ncat;
    int x_dtype, u_dtype, t_bf16;  // T = bfloat16 (1) or float16 (0)
    float ln_eps;
    int stages;
};

// round to the GEMM type T and back
__device__ __forceinline__ float round_t(float v, int t_bf16) {
    return t_bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}
__device__ __forceinline__ uint32_t pack_t(float lo, float hi, int t_bf16) {
    if (t_bf16) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&p);
    }
    const __half2 p = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1,
// layout type 2 (SWIZZLE_128B).  The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Bounded wait for a phase (returns false after the poll limit).
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity) { return mbar_wait(bar, parity); }

template <typename XT> struct Vec16;  // 16-byte vector of x elements, as float
template <> struct Vec16<float> {
    static __device__ __forceinline__ void load(const float* p, float* v) {
        const float4 q = *reinterpret_cast<const float4*>(p);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
};
template <> struct Vec16<__half> {
    static __device__ __forceinline__ void load(const __half* p, float* v) {
        const uint4 q = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};
template <> struct Vec16<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
        const uint4 q = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};

template <typename UT>
__device__ __forceinline__ void store_u(UT* p, float v);
template <> __device__ __forceinline__ void store_u<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_u<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <> __device__ __forceinline__ void store_u<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}

// Row statistics of LayerNorm (float32): one warp per row, two passes
// (mean, then the mean square deviation) with 16-byte loads.
template <typename XT>
__global__ void __launch_bounds__(256) ln_stats_k(const XT* __restrict__ x, float2* __restrict__ stats, int M, int d,
                                                  float eps) {
    constexpr int VN = 16 / sizeof(XT);
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (m >= M) return;
    const XT* row = x + static_cast<size_t>(m) * d;
    float s = 0.f;
    for (int c = lane * VN; c < d; c += 32 * VN) {
        float v[VN];
        Vec16<XT>::load(row + c, v);
#pragma unroll
        for (int e = 0; e < VN; ++e) s += v[e];
    }
    const float mean = warp_sum(s) / static_cast<float>(d);
    float q = 0.f;
    for (int c = lane * VN; c < d; c += 32 * VN) {
        float v[VN];
        Vec16<XT>::load(row + c, v);
#pragma unroll
        for (int e = 0; e < VN; ++e) {
            const float dv = v[e] - mean;
            q = fmaf(dv, dv, q);
        }
    }
    const float var = warp_sum(q) / static_cast<float>(d);
    if (lane == 0) stats[m] = make_float2(mean, rsqrtf(var + eps));
}

template <typename XT, typename UT>
__global__ void __launch_bounds__(kThreads, 2)
    project_k(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw, PArgs a) {
    const int S = a.stages;
    constexpr uint32_t XB = x_bytes<XT>(), AB = a_bytes<XT>();
    constexpr int XBOX = 128 / sizeof(XT);  // x columns per 128-byte swizzled row of a TMA box
    extern __shared__ __align__(1024) unsigned char psmem[];
    const uint32_t base_u32 = smem_u32(psmem);
    unsigned char* sbase = psmem + ((1024u - (base_u32 & 1023u)) & 1023u);  // 1024-aligned stages
    unsigned char* sX = sbase;                 // S x XB
    unsigned char* sA = inplace<XT>() ? sX : sX + S * XB;  // S x 16 KB (the x stages themselves for 16-bit x)
    unsigned char* sW = sX + S * (XB + AB);    // S x 32 KB
    const int nkb = (a.d + kBK - 1) / kBK;
    float* sGamma = reinterpret_cast<float*>(sW + S * kWBytes);  // LayerNorm affine, zero past d
    float* sBeta = sGamma + nkb * kBK;
    float* sBias = sBeta + nkb * kBK;                             // this CTA's output columns
    uint64_t* fullX = reinterpret_cast<uint64_t*>(sBias + kBN);
    uint64_t* fullA = fullX + kMaxStages;
    uint64_t* fullW = fullA + kMaxStages;
    uint64_t* empty = fullW + kMaxStages;  // the x, A and W stages of one k-block, freed by the MMAs' commit
    uint64_t* accb = empty + kMaxStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kBN;
    const int m0 = blockIdx.y * kBM;
    for (int i = tid; i < nkb * kBK; i += kThreads) {
        sGamma[i] = i < a.d ? a.gamma[i] : 0.f;
        sBeta[i] = i < a.d ? a.beta[i] : 0.f;
    }
    for (int i = tid; i < kBN; i += kThreads)  // the bias as autocast adds it: rounded to T
        sBias[i] = n0 + i < a.Ncat ? round_t(a.bias[n0 + i], a.t_bf16) : 0.f;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&fullX[s], 1);
            mbar_init(&fullA[s], 4);  // one arrival per LayerNorm warp
            mbar_init(&fullW[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accb, 1);
        fence_mbar_init();
    }
    if (warp == 1) {  // the accumulator: 256 TMEM columns (the warp allocates)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kBN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {  // TMA: the x tile and the weight, one k-block per stage
            prefetch_tmap(&tx);
            prefetch_tmap(&tw);
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % S;
                const uint32_t round = kb / S;
                ok = pwait(&empty[s], (round & 1) ^ 1);
                mbar_expect_tx(&fullX[s], XB);
#pragma unroll
                for (int h = 0; h < kBK / XBOX; ++h)
                    tma_load_2d(sX + s * XB + h * (kBM * 128), &tx, &fullX[s], kb * kBK + h * XBOX, m0);
                mbar_expect_tx(&fullW[s], kWBytes);
                tma_load_2d(sW + s * kWBytes, &tw, &fullW[s], kb * kBK, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // the MMA issuer
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(a.t_bf16) << 7) |
                                   (static_cast<uint32_t>(a.t_bf16) << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                                   (static_cast<uint32_t>(kBM >> 4) << 24);
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % S;
                const uint32_t round = kb / S;
                ok = pwait(&fullA[s], round & 1) && pwait(&fullW[s], round & 1);
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + s * kABytes), b0 = smem_u32(sW + s * kWBytes);
#pragma unroll
                for (int k = 0; k < kBK / kUK; ++k)  // +32 bytes per 16 elements within the swizzled row
                    mma_f16(tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc, (kb | k) != 0);
                mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            mma_commit(accb);  // the accumulator is complete
        }
    } else {
        // ---- LayerNorm: thread t owns row t of the tile ----
        const int q4 = warp & 3;  // TMEM lane group of this warp
        const int row = q4 * 32 + lane;
        const bool rv = m0 + row < a.M;
        constexpr int VN = 16 / sizeof(XT);  // x elements per 16-byte chunk
        const float2 st = rv ? a.stats[m0 + row] : make_float2(0.f, 0.f);
        for (int kb = 0; kb < nkb && ok; ++kb) {
            const int s = kb % S;
            ok = pwait(&fullX[s], (kb / S) & 1);
            const int ncols = min(kBK, a.d - kb * kBK);
            const unsigned char* xs = sX + s * XB;
            unsigned char* arow = sA + s * kABytes + row * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // 16-byte chunk j of the A row: columns 8j .. 8j+7
                const int c = 8 * j;
                const int pj = (j ^ (row & 7)) << 4;  // its swizzled position
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = 0.f;
                if (rv && c < ncols) {
#pragma unroll
                    for (int e0 = 0; e0 < 8; e0 += VN) {  // those 8 columns in the x boxes
                        const int cx = c + e0, h = cx / XBOX, jx = (cx % XBOX) / VN;
                        float t[VN];
                        Vec16<XT>::load(reinterpret_cast<const XT*>(xs + h * (kBM * 128) + row * 128 +
                                                                    ((jx ^ (row & 7)) << 4)), t);
#pragma unroll
                        for (int e = 0; e < VN; ++e) v[e0 + e] = t[e];
                    }
                    const int cg = kb * kBK + c;  // a multiple of 8 (16-byte aligned in shared memory)
                    const float4 g0 = *reinterpret_cast<const float4*>(sGamma + cg);
                    const float4 g1 = *reinterpret_cast<const float4*>(sGamma + cg + 4);
                    const float4 b0 = *reinterpret_cast<const float4*>(sBeta + cg);
                    const float4 b1 = *reinterpret_cast<const float4*>(sBeta + cg + 4);
                    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
                    const float bt[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = fmaf((v[e] - st.x) * st.y, g[e], bt[e]);
                }
                uint4 w;
                w.x = pack_t(v[0], v[1], a.t_bf16);
                w.y = pack_t(v[2], v[3], a.t_bf16);
                w.z = pack_t(v[4], v[5], a.t_bf16);
                w.w = pack_t(v[6], v[7], a.t_bf16);
                // in place for 16-bit x: this thread alone reads and writes row `row`'s chunk
                *reinterpret_cast<uint4*>(arow + pj) = w;
            }
            fence_proxy_async();  // the generic-proxy stores, visible to the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullA[s]);
        }
        // ---- epilogue: the accumulator row of this thread ----
        if (ok) ok = pwait(accb, 0);
        tc_fence_after();
        const int m = m0 + row;
        const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
        for (int c0 = 0; c0 < kBN; c0 += 16) {
            uint32_t r[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                : "r"(tmem + lane_base + static_cast<uint32_t>(c0)));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (m >= a.M || !ok) continue;
            const int nb = n0 + c0;
            float vv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                vv[j] = nb + j < a.Ncat ? round_t(__uint_as_float(r[j]) + sBias[c0 + j], a.t_bf16)
                                        : 0.f;
            UT* urow = static_cast<UT*>(a.u) + static_cast<size_t>(m) * a.H;
            if (nb + 16 <= a.H && (a.H % 8) == 0) {  // 16 columns of u: vector stores
                if constexpr (sizeof(UT) == 2) {
                    uint4 w0, w1;
                    const int tb = sizeof(UT) == 2 && std::is_same<UT, __nv_bfloat16>::value;
                    w0.x = pack_t(vv[0], vv[1], tb);   w0.y = pack_t(vv[2], vv[3], tb);
                    w0.z = pack_t(vv[4], vv[5], tb);   w0.w = pack_t(vv[6], vv[7], tb);
                    w1.x = pack_t(vv[8], vv[9], tb);   w1.y = pack_t(vv[10], vv[11], tb);
                    w1.z = pack_t(vv[12], vv[13], tb); w1.w = pack_t(vv[14], vv[15], tb);
                    reinterpret_cast<uint4*>(urow + nb)[0] = w0;
                    reinterpret_cast<uint4*>(urow + nb)[1] = w1;
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4*>(urow + nb + j) = make_float4(vv[j], vv[j + 1], vv[j + 2], vv[j + 3]);
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int n = nb + j;
                if (n >= a.Ncat) break;
                if (n < a.H) {
                    store_u<UT>(urow + n, vv[j]);
                } else {
                    int k = n - a.H;
                    float2* dst = a.Bc;
                    if (k >= 2 * a.N) {
                        k -= 2 * a.N;
                        dst = a.Cc;
                    }
                    float* f = reinterpret_cast<float*>(dst + static_cast<size_t>(m) * a.N + (k < a.N ? k : k - a.N));
                    f[k < a.N ? 0 : 1] = vv[j];
                }
            }
        }
    }
    if (!ok) set_status(EACS_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

size_t project_workspace_size(int64_t M) { return M > 0 ? static_cast<size_t>(M) * sizeof(float2) : 0; }

int project_fwd(const ProjectCall& c, cudaStream_t stream) {
    const char* fn = "eacs_project";
    if (c.M < 0 || c.d <= 0 || c.H <= 0 || c.N <= 0)
        return fail(EACS_ERR_INVALID, "%s: sizes must be positive (M may be 0)", fn);
    if (c.M == 0) return EACS_OK;
    if (!c.x || !c.gamma || !c.beta || !c.weight || !c.bias || !c.u || !c.Bc || !c.Cc)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (c.w_dtype != EACS_DTYPE_F16 && c.w_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: the weight must be float16 or bfloat16", fn);
    for (int dt : {c.x_dtype, c.u_dtype})
        if (dt != EACS_DTYPE_F32 && dt != EACS_DTYPE_F16 && dt != EACS_DTYPE_BF16)
            return fail(EACS_ERR_INVALID, "%s: unknown dtype %d", fn, dt);
    if (c.d % 8 != 0) return fail(EACS_ERR_UNSUPPORTED, "%s: d=%lld must be a multiple of 8", fn, (long long)c.d);
    const int64_t ncat = c.H + 4 * c.N;
    if (c.w_rows < ncat || c.w_rows % kBN != 0)
        return fail(EACS_ERR_INVALID, "%s: the weight needs a multiple of %d rows >= H + 4N = %lld (zero padded)", fn,
                    kBN, (long long)ncat);
    if (c.M > (1LL << 31) - 1 || c.d > (1LL << 24) || c.w_rows > (1LL << 24))
        return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    for (const void* ptr : {c.weight, c.x, static_cast<const void*>(c.gamma), static_cast<const void*>(c.beta)})
        if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
            return fail(EACS_ERR_INVALID, "%s: x, weight, gamma and beta must be 16-byte aligned", fn);
    const size_t ws_need = project_workspace_size(c.M);
    if (!c.workspace || c.workspace_bytes < ws_need || (reinterpret_cast<uintptr_t>(c.workspace) & 7) != 0)
        return fail(EACS_ERR_WORKSPACE, "%s: an 8-byte aligned workspace of %zu bytes is needed, %zu given", fn,
                    ws_need, c.workspace_bytes);
    auto enc = encode_fn();
    if (!enc) return fail(EACS_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", fn);
    cuuint32_t estr[2] = {1, 1};
    // weight (w_rows, d): boxes of 64 columns x 256 rows, 128-byte swizzle
    CUtensorMap tw;
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(c.d), static_cast<cuuint64_t>(c.w_rows)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(c.d * 2)};
        cuuint32_t box[2] = {kBK, kBN};
        const CUresult r = enc(&tw, c.w_dtype == EACS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                               2, const_cast<void*>(c.weight), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(EACS_ERR_CUDA, "%s: weight tensor map (%d)", fn, static_cast<int>(r));
    }
    // x (M, d): boxes of 128 bytes x 128 rows, 128-byte swizzle; rows past M
    // and columns past d read as zeros
    CUtensorMap tx;
    {
        const int esz = c.x_dtype == EACS_DTYPE_F32 ? 4 : 2;
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(c.d), static_cast<cuuint64_t>(c.M)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(c.d * esz)};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), kBM};
        const CUtensorMapDataType dt = c.x_dtype == EACS_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : c.x_dtype == EACS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        const CUresult r = enc(&tx, dt, 2, const_cast<void*>(c.x), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(EACS_ERR_CUDA, "%s: x tensor map (%d)", fn, static_cast<int>(r));
    }
    PArgs a{};
    a.x = c.x;
    a.stats = static_cast<const float2*>(c.workspace);
    a.gamma = c.gamma;
    a.beta = c.beta;
    a.bias = c.bias;
    a.u = c.u;
    a.Bc = static_cast<float2*>(c.Bc);
    a.Cc = static_cast<float2*>(c.Cc);
    a.M = static_cast<int>(c.M);
    a.d = static_cast<int>(c.d);
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    a.Ncat = static_cast<int>(ncat);
    a.x_dtype = c.x_dtype;
    a.u_dtype = c.u_dtype;
    a.t_bf16 = c.w_dtype == EACS_DTYPE_BF16 ? 1 : 0;
    a.ln_eps = c.ln_eps;
    const dim3 grid(static_cast<unsigned>(c.w_rows / kBN), static_cast<unsigned>((c.M + kBM - 1) / kBM));
    if (grid.y > 65535u) return fail(EACS_ERR_UNSUPPORTED, "%s: M too large for one launch", fn);
    cudaError_t e = cudaSuccess;
    a.stages = c.x_dtype == EACS_DTYPE_F32 ? stages_for<float>(c.d) : stages_for<__half>(c.d);
    if (a.stages == 0) return fail(EACS_ERR_UNSUPPORTED, "%s: d=%lld too large", fn, (long long)c.d);
    // LayerNorm statistics of every row, then the fused normalisation + GEMM
    float2* stats = static_cast<float2*>(c.workspace);
    const unsigned sgrid = static_cast<unsigned>((c.M + 7) / 8);
    if (c.x_dtype == EACS_DTYPE_F32)
        ln_stats_k<float><<<sgrid, 256, 0, stream>>>(static_cast<const float*>(c.x), stats, a.M, a.d, c.ln_eps);
    else if (c.x_dtype == EACS_DTYPE_F16)
        ln_stats_k<__half><<<sgrid, 256, 0, stream>>>(static_cast<const __half*>(c.x), stats, a.M, a.d, c.ln_eps);
    else
        ln_stats_k<__nv_bfloat16><<<sgrid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(c.x), stats, a.M,
                                                             a.d, c.ln_eps);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);
    mark_start(stream);
    switch (c.x_dtype * 3 + c.u_dtype) {
#define EACS_PROJ_CASE(XD, UD, XT, UT)                                                                         \
    case XD * 3 + UD:                                                                                      \
        e = cudaFuncSetAttribute(project_k<XT, UT>, cudaFuncAttributeMaxDynamicSharedMemorySize,              \
                                 static_cast<int>(smem_bytes<XT>(a.stages, c.d)));                          \
        if (e == cudaSuccess)                                                                              \
            project_k<XT, UT><<<grid, kThreads, smem_bytes<XT>(a.stages, c.d), stream>>>(tx, tw, a);       \
        break;
        EACS_PROJ_CASE(0, 0, float, float)
        EACS_PROJ_CASE(0, 1, float, __half)
        EACS_PROJ_CASE(0, 2, float, __nv_bfloat16)
        EACS_PROJ_CASE(1, 0, __half, float)
        EACS_PROJ_CASE(1, 1, __half, __half)
        EACS_PROJ_CASE(1, 2, __half, __nv_bfloat16)
        EACS_PROJ_CASE(2, 0, __nv_bfloat16, float)
        EACS_PROJ_CASE(2, 1, __nv_bfloat16, __half)
        EACS_PROJ_CASE(2, 2, __nv_bfloat16, __nv_bfloat16)
#undef EACS_PROJ_CASE
    }
    mark_stop(stream);
    note_launch();
    if (e != cudaSuccess) return cuda_check(e, fn);
    return cuda_check(cudaGetLastError(), fn);
}

}  // namespace eacs
