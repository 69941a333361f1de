// fuse.cu -- MultiScaleEACS branch epilogue in one pass (sm_100a).
//
// Reference: cst_ssm/modules/multiscale.py:176-179 --
//   w = softmax(fusion(x)),  fused = sum_s w_s delta_s,  y = LayerNorm(x + fused)
// with fusion a Linear(d, S) and delta_s the branches' proj_out outputs.  The
// reference runs a GEMM, a softmax, a stack, an einsum, an add and a
// LayerNorm, each a pass over (B, L, d) tensors; here one warp per row reads
// x and the S deltas once, computes the S logits against the fusion weights
// held in shared memory (with the LayerNorm weights, lane-interleaved), the
// softmax, the blend and the LayerNorm (two-pass mean / variance in
// registers, fp32 throughout) and writes y and w.
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
    constexpr int Q = E / 4;  // float4 per lane vector
    // The S fusion weight rows, then the LayerNorm gamma and beta, each laid
    // out as [k][q][lane] float4: lane l's elements (k*32 + l)*E + 4q .. +3
    // sit at consecutive 16-byte slots across the lanes (no bank conflicts).
    extern __shared__ float4 sw4[];
    const int d = a.d, S = a.S;
    const int per = VPL * 32 * E;  // padded row length
    float* swf = reinterpret_cast<float*>(sw4);
    for (int i = threadIdx.x; i < (S + 2) * per; i += blockDim.x) {
        const int s = i / per, col = i - s * per;
        const int k = col / (32 * E), ln_ = (col / E) % 32, e = col % E;
        float v = 0.f;
        if (col < d) {
            if (s < S) v = a.wf[static_cast<size_t>(s) * d + col];
            else if (s == S) v = a.gamma ? a.gamma[col] : 1.f;
            else v = a.beta ? a.beta[col] : 0.f;
        }
        swf[((((s * VPL + k) * Q + (e >> 2)) * 32 + ln_) << 2) + (e & 3)] = v;
    }
    __syncthreads();
    auto w4 = [&](int s, int k, int q, int l) { return sw4[((s * VPL + k) * Q + q) * 32 + l]; };
    float bias[kMaxBranch];
#pragma unroll
    for (int s = 0; s < kMaxBranch; ++s) bias[s] = (s < S && a.bf) ? a.bf[s] : 0.f;
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
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    const float4 w = w4(s, k, q, lane);
                    acc = fmaf(v[k][4 * q], w.x, acc);
                    acc = fmaf(v[k][4 * q + 1], w.y, acc);
                    acc = fmaf(v[k][4 * q + 2], w.z, acc);
                    acc = fmaf(v[k][4 * q + 3], w.w, acc);
                }
            }
        acc = warp_sum(acc) + bias[s];
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
            for (int q = 0; q < Q; ++q) {
                const float4 g = w4(S, k, q, lane), bb = w4(S + 1, k, q, lane);
                o[4 * q] = fmaf((v[k][4 * q] - mean) * rstd, g.x, bb.x);
                o[4 * q + 1] = fmaf((v[k][4 * q + 1] - mean) * rstd, g.y, bb.y);
                o[4 * q + 2] = fmaf((v[k][4 * q + 2] - mean) * rstd, g.z, bb.z);
                o[4 * q + 3] = fmaf((v[k][4 * q + 3] - mean) * rstd, g.w, bb.w);
            }
            store_vec(yr + i0, o);
        }
    }
}

// the vectors per lane the launched instance uses (a power of two)
int vpl_pad(int vpl) { return vpl <= 1 ? 1 : vpl <= 2 ? 2 : vpl <= 4 ? 4 : 8; }

template <typename T>
cudaError_t launch_fuse(const FuseArgs& a, cudaStream_t s) {
    constexpr int E = Vec<T>::E;
    const int vpl = (a.d + 32 * E - 1) / (32 * E);
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((a.rows + kFuseRows - 1) / kFuseRows, static_cast<int64_t>(n_sm) * 8));
    const size_t smem = sizeof(float) * (a.S + 2) * vpl_pad(vpl) * 32 * E;
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
    if (c.d % E != 0 || c.d > 8 * 32 * E)  // shared memory: (S + 2) x 256 E floats, at most 80 KiB
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
