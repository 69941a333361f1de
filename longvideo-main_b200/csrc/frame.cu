// frame.cu -- one streaming frame of a MultiScaleEACS in S + 3 launches (sm_100a).
//
// Reference: cst_ssm/modules/streaming.py:45-85 (temporal_step) with the
// layers' norm / _project / proj_out (modules/eacs.py:261-267) and the
// module's fusion and out_norm (modules/multiscale.py:45-46, :177-179), in
// inference.  Per frame of B rows (B <= 8), d features:
//   1. frame_proj_k: every branch's LayerNorm and input projections and the
//      fusion logits: one warp per output row of the stacked weights
//      [proj_u; proj_B; proj_C] of every branch and of the fusion layer, dot
//      products with the B centred rows held in shared memory (the row
//      statistics are shared by all branches; each branch applies its own
//      affine);
//   2. the cell step of each branch: stream_chunk with K = 1 (stream.cu);
//   3. frame_out_k: each branch's proj_out, masked by valid, blended with the
//      softmax of the fusion logits, plus the residual x: one warp per output
//      feature and branch, the blend through shared memory;
//   4. frame_ln_k: out_norm and the valid mask, one CTA per row.
// The frame's GEMVs read the weights once (fp32, ~26 MB for config 2's three
// branches at d = 1024, resident in L2 from frame to frame).
#include <algorithm>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kFT = 256;           // threads a CTA
constexpr int kFW = kFT / 32;      // warps a CTA (one output row each)

struct ProjBranch {
    const float* ln_w;
    const float* ln_b;
    float ln_eps;
    const float* w[3];   // proj_u (H,d), proj_B (2N,d), proj_C (2N,d)
    const float* b[3];
    int H, N;
    float* u;            // (B,H)
    float2* Bc;          // (B,N)
    float2* Cc;
};

struct ProjArgs {
    const float* x;      // (B,d)
    ProjBranch br[kFrameMaxBranches];
    const float* wf;     // fusion (S,d), (S)
    const float* bf;
    float* logits;       // (B,S)
    int row0[kFrameMaxBranches + 1];
    int rows;
    int B, d, S;
};

__global__ void __launch_bounds__(kFT) frame_proj_k(ProjArgs a) {
    extern __shared__ float sx[];  // [B][d] centred rows
    __shared__ float svar[kFrameMaxRows], smean[kFrameMaxRows];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int B = a.B, d = a.d;
    for (int b = warp; b < B; b += kFW) {
        const float* xr = a.x + static_cast<size_t>(b) * d;
        float s = 0.f;
        for (int k = lane; k < d; k += 32) s += xr[k];
        const float mean = warp_sum(s) / d;
        float v = 0.f;
        for (int k = lane; k < d; k += 32) {
            const float c = xr[k] - mean;
            sx[b * d + k] = c;
            v += c * c;
        }
        v = warp_sum(v) / d;
        if (lane == 0) {
            smean[b] = mean;
            svar[b] = v;
        }
    }
    __syncthreads();
    const int row = blockIdx.x * kFW + warp;
    if (row >= a.rows) return;
    float acc[kFrameMaxRows];
#pragma unroll
    for (int b = 0; b < kFrameMaxRows; ++b) acc[b] = 0.f;
    if (row >= a.row0[a.S]) {  // fusion logits on the raw rows
        const int o = row - a.row0[a.S];
        const float* w = a.wf + static_cast<size_t>(o) * d;
        for (int k = lane; k < d; k += 32) {
            const float wk = w[k];
#pragma unroll
            for (int b = 0; b < kFrameMaxRows; ++b)
                if (b < B) acc[b] = fmaf(wk, a.x[static_cast<size_t>(b) * d + k], acc[b]);
        }
#pragma unroll
        for (int b = 0; b < kFrameMaxRows; ++b) {
            const float v = warp_sum(acc[b]);
            if (lane == 0 && b < B) a.logits[b * a.S + o] = v + a.bf[o];
        }
        return;
    }
    int s = 0;
    while (row >= a.row0[s + 1]) ++s;
    const ProjBranch& p = a.br[s];
    int o = row - a.row0[s], m = 0;
    if (o >= p.H) {
        o -= p.H;
        m = 1 + o / (2 * p.N);
        o %= 2 * p.N;
    }
    const float* w = p.w[m] + static_cast<size_t>(o) * d;
    float rstd[kFrameMaxRows];
#pragma unroll
    for (int b = 0; b < kFrameMaxRows; ++b) rstd[b] = b < B ? 1.0f / sqrtf(svar[b] + p.ln_eps) : 0.f;
    if ((d & 3) == 0 &&
        ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(p.ln_w) | reinterpret_cast<uintptr_t>(p.ln_b)) &
         15u) == 0) {
        // 16-byte loads, several in flight per lane
        const float4* w4 = reinterpret_cast<const float4*>(w);
        const float4* g4 = reinterpret_cast<const float4*>(p.ln_w);
        const float4* be4 = reinterpret_cast<const float4*>(p.ln_b);
        const float4* sx4 = reinterpret_cast<const float4*>(sx);
        const int d4 = d >> 2;
#pragma unroll 2
        for (int k = lane; k < d4; k += 32) {
            const float4 wk = w4[k], g = g4[k], be = be4[k];
#pragma unroll
            for (int b = 0; b < kFrameMaxRows; ++b)
                if (b < B) {
                    const float4 xv = sx4[b * d4 + k];
                    float t = acc[b];
                    t = fmaf(wk.x, fmaf(xv.x * rstd[b], g.x, be.x), t);
                    t = fmaf(wk.y, fmaf(xv.y * rstd[b], g.y, be.y), t);
                    t = fmaf(wk.z, fmaf(xv.z * rstd[b], g.z, be.z), t);
                    acc[b] = fmaf(wk.w, fmaf(xv.w * rstd[b], g.w, be.w), t);
                }
        }
    } else {
        for (int k = lane; k < d; k += 32) {
            const float wk = w[k], g = p.ln_w[k], be = p.ln_b[k];
#pragma unroll
            for (int b = 0; b < kFrameMaxRows; ++b)
                if (b < B) acc[b] = fmaf(wk, fmaf(sx[b * d + k] * rstd[b], g, be), acc[b]);
        }
    }
#pragma unroll
    for (int b = 0; b < kFrameMaxRows; ++b) {
        const float v = warp_sum(acc[b]);
        if (lane == 0 && b < B) {
            const float val = v + p.b[m][o];
            if (m == 0) p.u[static_cast<size_t>(b) * p.H + o] = val;
            else {
                float2* dst = (m == 1 ? p.Bc : p.Cc) + static_cast<size_t>(b) * p.N + (o % p.N);
                reinterpret_cast<float*>(dst)[o < p.N ? 0 : 1] = val;  // (re, im) = rows [0, N), [N, 2N)
            }
        }
    }
}

struct OutBranch {
    const float* w;  // proj_out (d,H)
    const float* b;  // (d)
    const float* y;  // (B,H) the cell's output
    int H;
};

struct OutArgs {
    const float* x;          // (B,d)
    const uint8_t* valid;    // (B) or null
    const float* logits;     // (B,S)
    OutBranch br[kFrameMaxBranches];
    float* z;                // (B,d) x + sum_s w_s valid (proj_out_s y_s)
    float* weights;          // (B,S) softmax of the logits
    int B, d, S;
};

constexpr int kFOut = 8;  // output features a CTA; one warp per (feature, branch)

__global__ void __launch_bounds__(kFOut * kFrameMaxBranches * 32) frame_out_k(OutArgs a) {
    __shared__ float sw[kFrameMaxRows][kFrameMaxBranches];
    __shared__ float sdelta[kFOut][kFrameMaxBranches][kFrameMaxRows];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int B = a.B, d = a.d, S = a.S;
    if (threadIdx.x < B) {  // softmax over the branches, one thread a row
        const int b = threadIdx.x;
        float mx = -INFINITY;
        for (int s = 0; s < S; ++s) mx = fmaxf(mx, a.logits[b * S + s]);
        float e[kFrameMaxBranches], sum = 0.f;
        for (int s = 0; s < S; ++s) {
            e[s] = expf(a.logits[b * S + s] - mx);
            sum += e[s];
        }
        for (int s = 0; s < S; ++s) {
            sw[b][s] = e[s] / sum;
            if (blockIdx.x == 0) a.weights[b * S + s] = sw[b][s];
        }
    }
    // this warp's (feature, branch): proj_out's dot product for every row
    const int ol = warp / S, s = warp % S;
    const int o = blockIdx.x * kFOut + ol;
    if (o < d) {
        const OutBranch& p = a.br[s];
        const float* w = p.w + static_cast<size_t>(o) * p.H;
        float dot[kFrameMaxRows];
#pragma unroll
        for (int b = 0; b < kFrameMaxRows; ++b) dot[b] = 0.f;
        if ((p.H & 3) == 0 && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(p.y)) & 15u) == 0) {
            // 16-byte loads, several in flight per lane (the weights stream from L2)
            const float4* w4 = reinterpret_cast<const float4*>(w);
            const int H4 = p.H >> 2;
#pragma unroll 4
            for (int k = lane; k < H4; k += 32) {
                const float4 wk = w4[k];
#pragma unroll
                for (int b = 0; b < kFrameMaxRows; ++b)
                    if (b < B) {
                        const float4 yv = reinterpret_cast<const float4*>(p.y + static_cast<size_t>(b) * p.H)[k];
                        dot[b] = fmaf(wk.x, yv.x, fmaf(wk.y, yv.y, fmaf(wk.z, yv.z, fmaf(wk.w, yv.w, dot[b]))));
                    }
            }
        } else {
            for (int k = lane; k < p.H; k += 32) {
                const float wk = w[k];
#pragma unroll
                for (int b = 0; b < kFrameMaxRows; ++b)
                    if (b < B) dot[b] = fmaf(wk, p.y[static_cast<size_t>(b) * p.H + k], dot[b]);
            }
        }
#pragma unroll
        for (int b = 0; b < kFrameMaxRows; ++b) {
            const float v = warp_sum(dot[b]);
            if (lane == 0 && b < B) sdelta[ol][s][b] = v + p.b[o];
        }
    }
    __syncthreads();
    // blend the branches (masked by valid, weighted by the softmax) and add x
    for (int i = threadIdx.x; i < kFOut * B; i += blockDim.x) {
        const int l = i / B, b = i % B, oo = blockIdx.x * kFOut + l;
        if (oo >= d) continue;
        const float m = (a.valid && !a.valid[b]) ? 0.f : 1.f;
        float acc = 0.f;
        for (int t = 0; t < S; ++t) acc += (sdelta[l][t][b] * m) * sw[b][t];
        a.z[static_cast<size_t>(b) * d + oo] = a.x[static_cast<size_t>(b) * d + oo] + acc;
    }
}

// out_norm and the valid mask: one CTA a row
__global__ void __launch_bounds__(kFT) frame_ln_k(const float* z, const uint8_t* valid, const float* g,
                                                   const float* be, float eps, float* y, int B, int d) {
    __shared__ float sred[kFW];
    const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* zr = z + static_cast<size_t>(b) * d;
    auto cta_sum = [&](float v) {  // every thread gets the sum, in a fixed order
        v = warp_sum(v);
        if (lane == 0) sred[warp] = v;
        __syncthreads();
        float t = 0.f;
        for (int w = 0; w < kFW; ++w) t += sred[w];
        __syncthreads();
        return t;
    };
    float s = 0.f;
    for (int k = threadIdx.x; k < d; k += kFT) s += zr[k];
    const float mean = cta_sum(s) / d;
    float v = 0.f;
    for (int k = threadIdx.x; k < d; k += kFT) {
        const float c = zr[k] - mean;
        v += c * c;
    }
    const float rstd = 1.0f / sqrtf(cta_sum(v) / d + eps);
    const float m = (valid && !valid[b]) ? 0.f : 1.f;
    for (int k = threadIdx.x; k < d; k += kFT)
        y[static_cast<size_t>(b) * d + k] = fmaf((zr[k] - mean) * rstd, g[k], be[k]) * m;
}

size_t alf(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

size_t stream_frame_workspace_size(const FrameBranch* br, int S, int64_t B, int64_t d) {
    if (!br || S < 1 || S > kFrameMaxBranches || B < 1 || B > kFrameMaxRows || d < 1) return 0;
    size_t o = 0;
    for (int s = 0; s < S; ++s) {
        if (br[s].H < 1 || br[s].N < 1) return 0;
        o += 2 * alf(sizeof(float) * B * br[s].H) + 2 * alf(sizeof(float2) * B * br[s].N);
    }
    return o + alf(sizeof(float) * B * S) + alf(sizeof(float) * B * d);
}

int stream_frame(const FrameCall& c, cudaStream_t stream) {
    const char* fn = "eacs_stream_frame";
    if (c.S < 1 || c.S > kFrameMaxBranches)
        return fail(EACS_ERR_UNSUPPORTED, "%s: %d branches (1..%d supported)", fn, c.S, kFrameMaxBranches);
    if (c.B < 0 || c.d < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.B == 0) return EACS_OK;
    if (c.B > kFrameMaxRows || c.d == 0 || c.d > (1 << 16))
        return fail(EACS_ERR_UNSUPPORTED, "%s: B=%lld (1..%d) d=%lld", fn, (long long)c.B, kFrameMaxRows,
                    (long long)c.d);
    if (!c.x || !c.t || !c.br || !c.wf || !c.bf || !c.out_w || !c.out_b || !c.y || !c.weights || !c.gate ||
        !c.resid || !c.innov)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    for (int s = 0; s < c.S; ++s) {
        const FrameBranch& b = c.br[s];
        if (!b.ln_w || !b.ln_b || !b.wu || !b.bu || !b.wB || !b.bB || !b.wC || !b.bC || !b.wo || !b.bo)
            return fail(EACS_ERR_INVALID, "%s: branch %d: null weight", fn, s);
        if (b.H < 1 || b.N < 1 || b.N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: branch %d: H=%d N=%d", fn, s, b.H, b.N);
    }
    const size_t need = stream_frame_workspace_size(c.br, c.S, c.B, c.d);
    if (!c.workspace || c.workspace_bytes < need)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, need, c.workspace_bytes);
    const size_t smem = sizeof(float) * c.B * c.d;
    if (smem > 200u * 1024u) return fail(EACS_ERR_UNSUPPORTED, "%s: B*d=%lld too large", fn, (long long)(c.B * c.d));
    const int B = static_cast<int>(c.B), d = static_cast<int>(c.d), S = c.S;
    char* ws = static_cast<char*>(c.workspace);
    size_t o = 0;
    float* u[kFrameMaxBranches];
    float* yb[kFrameMaxBranches];
    float2* Bc[kFrameMaxBranches];
    float2* Cc[kFrameMaxBranches];
    for (int s = 0; s < S; ++s) {
        u[s] = reinterpret_cast<float*>(ws + o);
        o += alf(sizeof(float) * B * c.br[s].H);
        yb[s] = reinterpret_cast<float*>(ws + o);
        o += alf(sizeof(float) * B * c.br[s].H);
        Bc[s] = reinterpret_cast<float2*>(ws + o);
        o += alf(sizeof(float2) * B * c.br[s].N);
        Cc[s] = reinterpret_cast<float2*>(ws + o);
        o += alf(sizeof(float2) * B * c.br[s].N);
    }
    float* logits = reinterpret_cast<float*>(ws + o);
    o += alf(sizeof(float) * B * S);
    float* z = reinterpret_cast<float*>(ws + o);

    // 1. norms, input projections, fusion logits
    ProjArgs pa{};
    pa.x = c.x;
    pa.wf = c.wf;
    pa.bf = c.bf;
    pa.logits = logits;
    pa.B = B;
    pa.d = d;
    pa.S = S;
    int rows = 0;
    for (int s = 0; s < S; ++s) {
        const FrameBranch& b = c.br[s];
        ProjBranch& p = pa.br[s];
        p.ln_w = b.ln_w;
        p.ln_b = b.ln_b;
        p.ln_eps = b.ln_eps;
        p.w[0] = b.wu;
        p.w[1] = b.wB;
        p.w[2] = b.wC;
        p.b[0] = b.bu;
        p.b[1] = b.bB;
        p.b[2] = b.bC;
        p.H = b.H;
        p.N = b.N;
        p.u = u[s];
        p.Bc = Bc[s];
        p.Cc = Cc[s];
        pa.row0[s] = rows;
        rows += b.H + 4 * b.N;
    }
    pa.row0[S] = rows;
    rows += S;
    pa.rows = rows;
    cudaError_t e = cudaFuncSetAttribute(frame_proj_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_check(e, fn);
    frame_proj_k<<<(rows + kFW - 1) / kFW, kFT, smem, stream>>>(pa);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);

    // 2. each branch's cell step
    for (int s = 0; s < S; ++s) {
        const FrameBranch& b = c.br[s];
        StreamCall sc{b.lam,   b.log_dt, b.D,      b.mean,  b.var,   u[s],    EACS_DTYPE_F32, Bc[s],  Cc[s],
                      c.t,     c.valid,  c.cpi,    b.h_in,  b.t_in,  b.u_in,  b.B_in,  b.C_in, b.init_in,
                      b.h_out, b.t_out,  b.u_out,  b.B_out, b.C_out, b.init_out, yb[s], c.gate + s * B,
                      c.resid + s * B, c.innov + s * B, b.eps, b.eta, b.var_eps, b.dt_init, b.dt_min, b.dt_max,
                      b.cpi_modulation, b.temperature, b.gate_mode, c.B, 1, b.H, b.N};
        const int rc = stream_chunk(sc, stream);
        if (rc) return rc;
    }

    // 3. proj_out, mask, fusion blend, residual
    OutArgs oa{};
    oa.x = c.x;
    oa.valid = c.valid;
    oa.logits = logits;
    oa.z = z;
    oa.weights = c.weights;
    oa.B = B;
    oa.d = d;
    oa.S = S;
    for (int s = 0; s < S; ++s) oa.br[s] = OutBranch{c.br[s].wo, c.br[s].bo, yb[s], c.br[s].H};
    frame_out_k<<<(d + kFOut - 1) / kFOut, kFOut * S * 32, 0, stream>>>(oa);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);

    // 4. out_norm
    frame_ln_k<<<B, kFT, 0, stream>>>(z, c.valid, c.out_w, c.out_b, c.out_eps, c.y, B, d);
    note_launch();
    return cuda_check(cudaGetLastError(), fn);
}

}  // namespace eacs
