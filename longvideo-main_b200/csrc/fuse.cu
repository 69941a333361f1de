// fuse.cu -- MultiScaleEACS branch epilogue in one pass (sm_100a).
//
// Reference: cst_ssm/modules/multiscale.py:176-179 --
//   w = softmax(fusion(x)),  fused = sum_s w_s delta_s,  y = LayerNorm(x + fused)
// with fusion a Linear(d, S) and delta_s the branches' proj_out outputs.  The
// reference runs a GEMM, a softmax, a stack, an einsum, an add and a
// LayerNorm, each a pass over (B, L, d) tensors; here one warp per row reads
// x and the S deltas once, computes the S logits against the fusion weights
// held in shared memory, the softmax, the blend and the LayerNorm (two-pass
// mean / variance in registers, fp32 throughout) and writes y and w.
// Rows are read as 16-byte vectors (8 bf16/fp16 or 4 fp32 elements a lane).
#include <algorithm>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kFuseRows = 8;  // warps (rows) per CTA
constexpr int kMaxBranch = 8;

struct FuseArgs {
    const void* x;
    const void* delta[kMaxBranch];
    const float* wf;     // (S, d) fusion weight
    const float* bf;     // (S) fusion bias or null
    const float* gamma;  // (d) LayerNorm weight or null
    const float* beta;   // (d) or null
    float ln_eps;
    void* y;
    float* w;            // (rows, S) or null
    int64_t rows;
    int d, S;
};

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int E = 4; };
template <> struct Vec<__half> { static constexpr int E = 8; };
template <> struct Vec<__nv_bfloat16> { static constexpr int E = 8; };

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* f) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::E; ++i) f[i] = to_f32(e[i]);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* f) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::E; ++i) e[i] = from_f32<T>(f[i]);
    *reinterpret_cast<uint4*>(p) = raw;
}

template <typename T, int VPL>
__global__ void __launch_bounds__(kFuseRows * 32) branch_fuse_k(FuseArgs a) {
    constexpr int E = Vec<T>::E;
    extern __shared__ float sw[];  // (S, d)
    const int d = a.d, S = a.S;
    for (int i = threadIdx.x; i < S * d; i += blockDim.x) sw[i] = a.wf[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    // rows in a grid-stride loop, so each CTA loads the fusion weights once
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kFuseRows + wid; r < a.rows;
         r += static_cast<int64_t>(gridDim.x) * kFuseRows) {
    const T* xr = static_cast<const T*>(a.x) + r * d;
    float v[VPL][E];
    bool in[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const int i0 = (k * 32 + lane) * E;
        in[k] = i0 < d;
        if (in[k]) load_vec(xr + i0, v[k]);
        else
#pragma unroll
            for (int e = 0; e < E; ++e) v[k][e] = 0.f;
    }
    // fusion logits and softmax over the branches
    float logit[kMaxBranch];
    float mx = -INFINITY;
#pragma unroll
    for (int s = 0; s < kMaxBranch; ++s) {
        if (s >= S) break;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k)
            if (in[k]) {
                const float* wr = sw + s * d + (k * 32 + lane) * E;
#pragma unroll
                for (int e = 0; e < E; ++e) acc = fmaf(v[k][e], wr[e], acc);
            }
        acc = warp_sum(acc) + (a.bf ? a.bf[s] : 0.f);
        logit[s] = acc;
        mx = fmaxf(mx, acc);
    }
    float den = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxBranch; ++s) {
        if (s >= S) break;
        logit[s] = expf(logit[s] - mx);
        den += logit[s];
    }
    const float inv = 1.0f / den;
    // x + sum_s w_s delta_s
#pragma unroll
    for (int s = 0; s < kMaxBranch; ++s) {
        if (s >= S) break;
        const float ws = logit[s] * inv;
        if (a.w && lane == 0) a.w[r * S + s] = ws;
        const T* dr = static_cast<const T*>(a.delta[s]) + r * d;
#pragma unroll
        for (int k = 0; k < VPL; ++k)
            if (in[k]) {
                float dv[E];
                load_vec(dr + (k * 32 + lane) * E, dv);
#pragma unroll
                for (int e = 0; e < E; ++e) v[k][e] = fmaf(ws, dv[e], v[k][e]);
            }
    }
    // LayerNorm over d (two passes over the registers)
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
        for (int e = 0; e < E; ++e) sum += v[k][e];
    const float mean = warp_sum(sum) / d;
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
        if (in[k])
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float c = v[k][e] - mean;
                sq = fmaf(c, c, sq);
            }
    const float rstd = 1.0f / sqrtf(warp_sum(sq) / d + a.ln_eps);
    T* yr = static_cast<T*>(a.y) + r * d;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
        if (in[k]) {
            const int i0 = (k * 32 + lane) * E;
            float o[E];
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float g = a.gamma ? a.gamma[i0 + e] : 1.f;
                const float bb = a.beta ? a.beta[i0 + e] : 0.f;
                o[e] = fmaf((v[k][e] - mean) * rstd, g, bb);
            }
            store_vec(yr + i0, o);
        }
    }
}

template <typename T>
cudaError_t launch_fuse(const FuseArgs& a, cudaStream_t s) {
    constexpr int E = Vec<T>::E;
    const int vpl = (a.d + 32 * E - 1) / (32 * E);
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((a.rows + kFuseRows - 1) / kFuseRows, static_cast<int64_t>(n_sm) * 8));
    const size_t smem = sizeof(float) * a.S * a.d;
    cudaError_t e;
#define EACS_FUSE(V)                                                                                \
    do {                                                                                            \
        e = cudaFuncSetAttribute(branch_fuse_k<T, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(smem));                                           \
        if (e != cudaSuccess) return e;                                                             \
        branch_fuse_k<T, V><<<grid, kFuseRows * 32, smem, s>>>(a);                                 \
    } while (0)
    if (vpl <= 1) EACS_FUSE(1);
    else if (vpl <= 2) EACS_FUSE(2);
    else if (vpl <= 4) EACS_FUSE(4);
    else EACS_FUSE(8);
#undef EACS_FUSE
    note_launch();
    return cudaGetLastError();
}

}  // namespace

int branch_fuse(const FuseCall& c, cudaStream_t stream) {
    const char* fn = "eacs_branch_fuse";
    if (c.rows < 0 || c.d <= 0 || c.S <= 0) return fail(EACS_ERR_INVALID, "%s: bad sizes", fn);
    if (c.S > kMaxBranch) return fail(EACS_ERR_UNSUPPORTED, "%s: S=%d > %d branches", fn, c.S, kMaxBranch);
    if (c.dtype != EACS_DTYPE_F32 && c.dtype != EACS_DTYPE_F16 && c.dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown dtype %d", fn, c.dtype);
    const int E = c.dtype == EACS_DTYPE_F32 ? 4 : 8;
    if (c.d % E != 0 || c.d > 8 * 32 * E || static_cast<size_t>(c.S) * c.d * 4 > 200u * 1024u)
        return fail(EACS_ERR_UNSUPPORTED, "%s: d=%d must be a multiple of %d and at most %d", fn, c.d, E,
                    8 * 32 * E);
    if (c.rows == 0) return EACS_OK;
    if (!c.x || !c.wf || !c.y) return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    FuseArgs a{};
    a.x = c.x;
    for (int s = 0; s < c.S; ++s) {
        if (!c.delta[s]) return fail(EACS_ERR_INVALID, "%s: null branch output %d", fn, s);
        a.delta[s] = c.delta[s];
    }
    // 16-byte vectors: every row start must be 16-byte aligned
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    bool ok = aligned(c.x) && aligned(c.y);
    for (int s = 0; s < c.S; ++s) ok = ok && aligned(c.delta[s]);
    if (!ok) return fail(EACS_ERR_INVALID, "%s: x, y and the branch outputs must be 16-byte aligned", fn);
    a.wf = c.wf;
    a.bf = c.bf;
    a.gamma = c.gamma;
    a.beta = c.beta;
    a.ln_eps = c.ln_eps;
    a.y = c.y;
    a.w = c.w;
    a.rows = c.rows;
    a.d = c.d;
    a.S = c.S;
    cudaError_t e;
    if (c.dtype == EACS_DTYPE_F16) e = launch_fuse<__half>(a, stream);
    else if (c.dtype == EACS_DTYPE_BF16) e = launch_fuse<__nv_bfloat16>(a, stream);
    else e = launch_fuse<float>(a, stream);
    return cuda_check(e, fn);
}

}  // namespace eacs
