// stream.cu -- streaming EACS steps with explicit branch state (sm_100a).
//
// Reference: cst_ssm/modules/streaming.py:45-85 (temporal_step, one branch)
// with eacs_step (modules/eacs.py:78-142) and EventGate.forward
// (modules/event_gate.py:86-105).  Per row and step, with the row's state
// (h_pi, t_pi, u_pi, B_pi, C_pi, initialized) and the frame's (u, B, C, t,
// valid):
//   first  = valid & !initialized: the predecessor is the frame itself
//            (t_pi = t - dt_init, u/B/C_pi = u/B/C) and the gate is forced
//            open (eps = -1 before CPI modulation, gate output 1);
//   eps_l  = cpi given and modulation > 0 ? max(eps (1 - m clamp(cpi,0,1)), 1e-3) : eps;
//   x_hat  = dA h_pi + dB_bar B_pi u_pi, r = ||obs - pred|| / (||obs|| + eta);
//   g      = r > eps_l (hard) or sigmoid((r - eps_l) / max(T, 1e-4)) (soft);
//   h_cur  = g h_upd + (1 - g) x_hat,  y = Re sum_n C h_cur + D u;
//   state' = g (h_upd, t, u, B, C) + (1 - g) state (first: h_cur and the frame),
//   rows with valid = 0 keep their state and output zeros.
// One CTA per row runs the chunk's K steps in order (K = 1 is temporal_step);
// state in and state out are separate buffers, so a caller may replay a step
// from the same state.
#include <algorithm>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kST = 1024;  // CTA threads

struct StArgs {
    const float2* lam;
    const float* log_dt;
    const float* D;
    const float* mean;
    const float* var;
    const void* u;         // (B,K,H)
    const float2* Bc;      // (B,K,N)
    const float2* Cc;
    const float* t;        // (B,K)
    const uint8_t* valid;  // (B,K) or null (all valid)
    const float* cpi;      // (B,K) or null
    // state in
    const float2* h_in;    // (B,H,N)
    const float* t_in;     // (B)
    const float* u_in;     // (B,H)
    const float2* B_in;    // (B,N)
    const float2* C_in;
    const uint8_t* init_in;  // (B)
    // state out
    float2* h_out;
    float* t_out;
    float* u_out;
    float2* B_out;
    float2* C_out;
    uint8_t* init_out;
    // outputs
    float* y;     // (B,K,H)
    float* gate;  // (B,K)
    float* resid;
    float* innov;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, Tp;
    int gate_mode;  // 0 hard, 1 soft
    int B, K, H, N;
};

template <int LANES, int NPT, typename UT>
__global__ void __launch_bounds__(kST) stream_chunk(StArgs a) {
    constexpr int HG = kST / LANES;  // channel groups per pass
    constexpr int NP = LANES * NPT;
    __shared__ float2 sBp[NP], sCp[NP];
    __shared__ float2 sred[kST / 32];
    __shared__ float sg;

    const int b = blockIdx.x;
    const int tid = threadIdx.x, ln = tid % LANES, hg = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const int H = a.H, N = a.N, K = a.K;
    const UT* u = static_cast<const UT*>(a.u);
    const size_t HN = static_cast<size_t>(H) * N;
    float2* hst = a.h_out + b * HN;  // the chunk works on the output state
    float* ust = a.u_out + static_cast<size_t>(b) * H;

    // copy the state in -> out, then step on the output buffers
    for (size_t i = tid; i < HN; i += kST) hst[i] = a.h_in[b * HN + i];
    for (int hh = tid; hh < H; hh += kST) ust[hh] = a.u_in[static_cast<size_t>(b) * H + hh];
    for (int n = tid; n < NP; n += kST) {
        sBp[n] = n < N ? a.B_in[static_cast<size_t>(b) * N + n] : make_float2(0.f, 0.f);
        sCp[n] = n < N ? a.C_in[static_cast<size_t>(b) * N + n] : make_float2(0.f, 0.f);
    }
    float t_pi = a.t_in[b];
    bool init = a.init_in[b] != 0;
    __syncthreads();

    for (int k = 0; k < K; ++k) {
        const size_t rk = static_cast<size_t>(b) * K + k;
        const bool v = a.valid ? a.valid[rk] != 0 : true;
        if (!v) {  // masked rows: state untouched, zero outputs
            for (int hh = tid; hh < H; hh += kST) a.y[rk * H + hh] = 0.f;
            if (tid == 0) {
                a.gate[rk] = 0.f;
                a.resid[rk] = 0.f;
                a.innov[rk] = 0.f;
            }
            continue;
        }
        const bool first = !init;
        const float tl = a.t[rk];
        if (first) {  // the frame is its own predecessor
            for (int n = tid; n < NP; n += kST) {
                sBp[n] = n < N ? a.Bc[rk * N + n] : make_float2(0.f, 0.f);
                sCp[n] = n < N ? a.Cc[rk * N + n] : make_float2(0.f, 0.f);
            }
            for (int hh = tid; hh < H; hh += kST) ust[hh] = to_f32(u[rk * H + hh]);
            t_pi = tl - a.dt_init;
            __syncthreads();
        }
        const float delta = fmaxf(tl - t_pi, 0.f);
        // phase A: prediction and residual
        float acc1 = 0.f, acc2 = 0.f;
        for (int h0 = 0; h0 < H; h0 += HG) {
            const int h = h0 + hg;
            const bool hv = h < H;
            float yhp = 0.f, dte = 0.f, upv = 0.f;
            if (hv) {
                dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
                upv = ust[h];
            }
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                if (hv && n < N) {
                    const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                    float2 dA, dB;
                    zoh(lm, crecip(lm), dte, dA, dB);
                    const float2 P = cmul(dA, hst[static_cast<size_t>(h) * N + n]);
                    const float2 q = cmul(dB, sBp[n]);
                    const float2 xh = make_float2(fmaf(q.x, upv, P.x), fmaf(q.y, upv, P.y));
                    yhp += cre_mul(sCp[n], xh);
                }
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yhp += __shfl_xor_sync(0xffffffffu, yhp, o);
            if (ln == 0 && hv) {
                const float sd = sqrtf(a.var[h] + a.var_eps);
                const float ul = to_f32(u[rk * H + h]);
                const float obs = (ul - a.mean[h]) / sd;
                const float pred = (yhp - a.mean[h]) / sd;
                const float d = obs - pred;
                acc1 += d * d;
                acc2 += obs * obs;
            }
        }
        acc1 = warp_sum(acc1);
        acc2 = warp_sum(acc2);
        if (lane == 0) sred[wid] = make_float2(acc1, acc2);
        __syncthreads();
        if (tid == 0) {
            float s1 = 0.f, s2 = 0.f;
            for (int w = 0; w < kST / 32; ++w) {
                s1 += sred[w].x;
                s2 += sred[w].y;
            }
            const float r = sqrtf(s1) / (sqrtf(s2) + a.eta);
            float eps_l = first ? -1.f : a.eps;
            if (a.cpi && a.cpi_mod > 0.f)
                eps_l = fmaxf(eps_l * (1.f - a.cpi_mod * fminf(fmaxf(a.cpi[rk], 0.f), 1.f)), 1e-3f);
            float g;
            if (a.gate_mode == 1) g = 1.0f / (1.0f + expf(-((r - eps_l) / a.Tp)));
            else g = r > eps_l ? 1.f : 0.f;
            a.gate[rk] = first ? 1.f : g;
            a.resid[rk] = r;
            a.innov[rk] = init ? r : 0.f;
            sg = g;
        }
        __syncthreads();
        const float g = sg;
        // phase C: update, blend, readout, new state
        for (int h0 = 0; h0 < H; h0 += HG) {
            const int h = h0 + hg;
            const bool hv = h < H;
            float yp = 0.f, dte = 0.f, upv = 0.f, ul = 0.f;
            if (hv) {
                dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
                upv = ust[h];
                ul = to_f32(u[rk * H + h]);
            }
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                if (hv && n < N) {
                    const size_t o = static_cast<size_t>(h) * N + n;
                    const float2 lm = a.lam[o];
                    float2 dA, dB;
                    zoh(lm, crecip(lm), dte, dA, dB);
                    const float2 hp = hst[o];
                    const float2 P = cmul(dA, hp);
                    const float2 qp = cmul(dB, sBp[n]);
                    const float2 xh = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                    const float2 qc = cmul(dB, a.Bc[rk * N + n]);
                    const float2 hu = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                    const float2 gu = cscale(hu, g);
                    const float2 hc = cadd(gu, cscale(xh, 1.f - g));
                    hst[o] = first ? hc : cadd(gu, cscale(hp, 1.f - g));
                    yp += cre_mul(a.Cc[rk * N + n], hc);
                }
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
            if (ln == 0 && hv) {
                a.y[rk * H + h] = yp + a.D[h] * ul;
                ust[h] = first ? ul : g * ul + (1.f - g) * upv;
            }
        }
        __syncthreads();
        for (int n = tid; n < N; n += kST) {
            const float2 Bl = a.Bc[rk * N + n], Cl = a.Cc[rk * N + n];
            sBp[n] = first ? Bl : cadd(cscale(Bl, g), cscale(sBp[n], 1.f - g));
            sCp[n] = first ? Cl : cadd(cscale(Cl, g), cscale(sCp[n], 1.f - g));
        }
        t_pi = first ? tl : g * tl + (1.f - g) * t_pi;
        init = true;
        __syncthreads();
    }
    for (int n = tid; n < N; n += kST) {
        a.B_out[static_cast<size_t>(b) * N + n] = sBp[n];
        a.C_out[static_cast<size_t>(b) * N + n] = sCp[n];
    }
    if (tid == 0) {
        a.t_out[b] = t_pi;
        a.init_out[b] = init ? 1 : 0;
    }
}

template <typename UT>
cudaError_t launch_stream(const StArgs& a, cudaStream_t s) {
    const int N = a.N;
    // lanes per channel and chains per lane (one pass covers kST / LANES channels)
    if (N <= 4) stream_chunk<4, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 8) stream_chunk<8, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 16) stream_chunk<16, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 32) stream_chunk<32, 1, UT><<<a.B, kST, 0, s>>>(a);
    else stream_chunk<32, 2, UT><<<a.B, kST, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

int stream_chunk(const StreamCall& c, cudaStream_t stream) {
    const char* fn = "eacs_stream_chunk";
    if (c.B < 0 || c.K < 0 || c.H < 0 || c.N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)c.N);
    if (c.B > (1LL << 31) - 1 || c.K > (1LL << 30) || c.H > (1LL << 24))
        return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    if (c.u_dtype != EACS_DTYPE_F32 && c.u_dtype != EACS_DTYPE_F16 && c.u_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, c.u_dtype);
    if (c.gate_mode != 0 && c.gate_mode != 1)
        return fail(EACS_ERR_INVALID, "%s: gate_mode must be 0 (hard) or 1 (soft)", fn);
    if (c.B == 0) return EACS_OK;
    if (c.H == 0 || c.N == 0) return fail(EACS_ERR_INVALID, "%s: H and N must be positive", fn);
    if (!c.lam || !c.log_dt || !c.D || !c.mean || !c.var || !c.u || !c.Bc || !c.Cc || !c.t ||
        !c.h_in || !c.t_in || !c.u_in || !c.B_in || !c.C_in || !c.init_in || !c.h_out ||
        !c.t_out || !c.u_out || !c.B_out || !c.C_out || !c.init_out || !c.y || !c.gate ||
        !c.resid || !c.innov)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (c.h_in == c.h_out || c.u_in == c.u_out)
        return fail(EACS_ERR_INVALID, "%s: state in and state out must be separate buffers", fn);
    StArgs a{};
    a.lam = static_cast<const float2*>(c.lam);
    a.log_dt = c.log_dt;
    a.D = c.D;
    a.mean = c.mean;
    a.var = c.var;
    a.u = c.u;
    a.Bc = static_cast<const float2*>(c.Bc);
    a.Cc = static_cast<const float2*>(c.Cc);
    a.t = c.t;
    a.valid = c.valid;
    a.cpi = c.cpi;
    a.h_in = static_cast<const float2*>(c.h_in);
    a.t_in = c.t_in;
    a.u_in = c.u_in;
    a.B_in = static_cast<const float2*>(c.B_in);
    a.C_in = static_cast<const float2*>(c.C_in);
    a.init_in = c.init_in;
    a.h_out = static_cast<float2*>(c.h_out);
    a.t_out = c.t_out;
    a.u_out = c.u_out;
    a.B_out = static_cast<float2*>(c.B_out);
    a.C_out = static_cast<float2*>(c.C_out);
    a.init_out = c.init_out;
    a.y = c.y;
    a.gate = c.gate;
    a.resid = c.resid;
    a.innov = c.innov;
    a.eps = c.eps;
    a.eta = c.eta;
    a.var_eps = c.var_eps;
    a.dt_init = c.dt_init;
    a.dt_min = c.dt_min;
    a.dt_max = c.dt_max;
    a.cpi_mod = c.cpi_modulation;
    a.Tp = c.temperature > 1e-4f ? c.temperature : 1e-4f;
    a.gate_mode = c.gate_mode;
    a.B = static_cast<int>(c.B);
    a.K = static_cast<int>(c.K);
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    cudaError_t e;
    if (c.u_dtype == EACS_DTYPE_F16) e = launch_stream<__half>(a, stream);
    else if (c.u_dtype == EACS_DTYPE_BF16) e = launch_stream<__nv_bfloat16>(a, stream);
    else e = launch_stream<float>(a, stream);
    return cuda_check(e, fn);
}

}  // namespace eacs
