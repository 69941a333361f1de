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
#include <cooperative_groups.h>

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

// ---------------------------------------------------------------------------
// One step (K = 1) with a row spread over a cluster of kSCL CTAs: CTA r owns
// channels [r*HC, (r+1)*HC).  Same semantics as stream_chunk; the row's two
// residual sums are added over the cluster through distributed shared memory
// (one hardware cluster barrier before the CTAs read one another's partials,
// one after, so that no CTA leaves while its partial may still be read), in
// rank order in every CTA, so all take the same gate decision.  State in and
// state out are separate buffers; nothing is copied in place.
// ---------------------------------------------------------------------------
constexpr int kSCL = 8;     // CTAs a row
constexpr int kSCT = 256;   // threads a CTA

template <int LANES, int NPT, typename UT>
__global__ void __cluster_dims__(kSCL, 1, 1) __launch_bounds__(kSCT) stream_step_cl(StArgs a) {
    namespace cg = cooperative_groups;
    constexpr int HG = kSCT / LANES;
    constexpr int NP = LANES * NPT;
    __shared__ float2 sBp[NP], sCp[NP];
    __shared__ float2 sred[kSCT / 32];
    __shared__ float2 spart;
    __shared__ float sg;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int b = blockIdx.y;
    const int tid = threadIdx.x, ln = tid % LANES, hg = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const int H = a.H, N = a.N;
    const int HC = (H + kSCL - 1) / kSCL;
    const int c0 = rank * HC, c1 = min(H, c0 + HC);
    const UT* u = static_cast<const UT*>(a.u);
    const size_t HN = static_cast<size_t>(H) * N;
    const size_t bH = static_cast<size_t>(b) * H;
    const bool v = a.valid ? a.valid[b] != 0 : true;
    if (!v) {  // masked row (the whole cluster): state through, zero outputs
        for (size_t i = static_cast<size_t>(c0) * N + tid; i < static_cast<size_t>(c1) * N; i += kSCT)
            a.h_out[b * HN + i] = a.h_in[b * HN + i];
        for (int h = c0 + tid; h < c1; h += kSCT) {
            a.u_out[bH + h] = a.u_in[bH + h];
            a.y[bH + h] = 0.f;
        }
        if (rank == 0) {
            for (int n = tid; n < N; n += kSCT) {
                a.B_out[static_cast<size_t>(b) * N + n] = a.B_in[static_cast<size_t>(b) * N + n];
                a.C_out[static_cast<size_t>(b) * N + n] = a.C_in[static_cast<size_t>(b) * N + n];
            }
            if (tid == 0) {
                a.t_out[b] = a.t_in[b];
                a.init_out[b] = a.init_in[b] ? 1 : 0;
                a.gate[b] = a.resid[b] = a.innov[b] = 0.f;
            }
        }
        return;
    }
    const bool init = a.init_in[b] != 0;
    const bool first = !init;
    const float tl = a.t[b];
    const float t_pi = first ? tl - a.dt_init : a.t_in[b];
    for (int n = tid; n < NP; n += kSCT) {
        const size_t o = static_cast<size_t>(b) * N + n;
        sBp[n] = n < N ? (first ? a.Bc[o] : a.B_in[o]) : make_float2(0.f, 0.f);
        sCp[n] = n < N ? (first ? a.Cc[o] : a.C_in[o]) : make_float2(0.f, 0.f);
    }
    __syncthreads();
    const float delta = fmaxf(tl - t_pi, 0.f);
    auto upi_of = [&](int h) { return first ? to_f32(u[bH + h]) : a.u_in[bH + h]; };
    // prediction and this CTA's share of the residual sums
    float acc1 = 0.f, acc2 = 0.f;
    for (int h0 = c0; h0 < c1; h0 += HG) {
        const int h = h0 + hg;
        const bool hv = h < c1;
        float yhp = 0.f, dte = 0.f, upv = 0.f;
        if (hv) {
            dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
            upv = upi_of(h);
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (hv && n < N) {
                const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                float2 dA, dB;
                zoh(lm, crecip(lm), dte, dA, dB);
                const float2 P = cmul(dA, a.h_in[b * HN + static_cast<size_t>(h) * N + n]);
                const float2 q = cmul(dB, sBp[n]);
                const float2 xh = make_float2(fmaf(q.x, upv, P.x), fmaf(q.y, upv, P.y));
                yhp += cre_mul(sCp[n], xh);
            }
        }
#pragma unroll
        for (int o = LANES / 2; o > 0; o >>= 1) yhp += __shfl_xor_sync(0xffffffffu, yhp, o);
        if (ln == 0 && hv) {
            const float sd = sqrtf(a.var[h] + a.var_eps);
            const float obs = (to_f32(u[bH + h]) - a.mean[h]) / sd;
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
        for (int w = 0; w < kSCT / 32; ++w) {
            s1 += sred[w].x;
            s2 += sred[w].y;
        }
        spart = make_float2(s1, s2);
    }
    cluster.sync();  // every CTA's partial is in place
    if (tid == 0) {
        float s1 = 0.f, s2 = 0.f;
        for (int r = 0; r < kSCL; ++r) {
            const float2 p = *cluster.map_shared_rank(&spart, r);
            s1 += p.x;
            s2 += p.y;
        }
        const float r = sqrtf(s1) / (sqrtf(s2) + a.eta);
        float eps_l = first ? -1.f : a.eps;
        if (a.cpi && a.cpi_mod > 0.f)
            eps_l = fmaxf(eps_l * (1.f - a.cpi_mod * fminf(fmaxf(a.cpi[b], 0.f), 1.f)), 1e-3f);
        const float g = a.gate_mode == 1 ? 1.0f / (1.0f + expf(-((r - eps_l) / a.Tp))) : (r > eps_l ? 1.f : 0.f);
        sg = g;
        if (rank == 0) {
            a.gate[b] = first ? 1.f : g;
            a.resid[b] = r;
            a.innov[b] = init ? r : 0.f;
        }
    }
    cluster.sync();  // all partials read: a CTA may now leave; sg is published
    const float g = sg;
    // update, blend, readout, state out for this CTA's channels
    for (int h0 = c0; h0 < c1; h0 += HG) {
        const int h = h0 + hg;
        const bool hv = h < c1;
        float yp = 0.f, dte = 0.f, upv = 0.f, ul = 0.f;
        if (hv) {
            dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
            upv = upi_of(h);
            ul = to_f32(u[bH + h]);
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (hv && n < N) {
                const size_t o = static_cast<size_t>(h) * N + n;
                const float2 lm = a.lam[o];
                float2 dA, dB;
                zoh(lm, crecip(lm), dte, dA, dB);
                const float2 hp = a.h_in[b * HN + o];
                const float2 P = cmul(dA, hp);
                const float2 qp = cmul(dB, sBp[n]);
                const float2 xh = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                const float2 qc = cmul(dB, a.Bc[static_cast<size_t>(b) * N + n]);
                const float2 hu = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                const float2 gu = cscale(hu, g);
                const float2 hc = cadd(gu, cscale(xh, 1.f - g));
                a.h_out[b * HN + o] = first ? hc : cadd(gu, cscale(hp, 1.f - g));
                yp += cre_mul(a.Cc[static_cast<size_t>(b) * N + n], hc);
            }
        }
#pragma unroll
        for (int o = LANES / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
        if (ln == 0 && hv) {
            a.y[bH + h] = yp + a.D[h] * ul;
            a.u_out[bH + h] = first ? ul : g * ul + (1.f - g) * upv;
        }
    }
    if (rank == 0) {
        for (int n = tid; n < N; n += kSCT) {
            const size_t o = static_cast<size_t>(b) * N + n;
            const float2 Bl = a.Bc[o], Cl = a.Cc[o];
            a.B_out[o] = first ? Bl : cadd(cscale(Bl, g), cscale(sBp[n], 1.f - g));
            a.C_out[o] = first ? Cl : cadd(cscale(Cl, g), cscale(sCp[n], 1.f - g));
        }
        if (tid == 0) {
            a.t_out[b] = first ? tl : g * tl + (1.f - g) * t_pi;
            a.init_out[b] = 1;
        }
    }
}

template <typename UT>
cudaError_t launch_stream(const StArgs& a, cudaStream_t s) {
    const int N = a.N;
    if (a.K == 1 && a.H >= 128 && a.B <= 65535) {  // one step: a row over a cluster of kSCL CTAs
        const dim3 grid(kSCL, a.B);
        if (N <= 4) stream_step_cl<4, 1, UT><<<grid, kSCT, 0, s>>>(a);
        else if (N <= 8) stream_step_cl<8, 1, UT><<<grid, kSCT, 0, s>>>(a);
        else if (N <= 16) stream_step_cl<16, 1, UT><<<grid, kSCT, 0, s>>>(a);
        else if (N <= 32) stream_step_cl<32, 1, UT><<<grid, kSCT, 0, s>>>(a);
        else stream_step_cl<32, 2, UT><<<grid, kSCT, 0, s>>>(a);
        note_launch();
        return cudaGetLastError();
    }
    // lanes per channel and chains per lane (one pass covers kST / LANES channels)
    if (N <= 4) stream_chunk<4, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 8) stream_chunk<8, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 16) stream_chunk<16, 1, UT><<<a.B, kST, 0, s>>>(a);
    else if (N <= 32) stream_chunk<32, 1, UT><<<a.B, kST, 0, s>>>(a);
    else stream_chunk<32, 2, UT><<<a.B, kST, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Backward of one step (K = 1: temporal_step under autograd), float32 u.
// Per row, with the step's forward recomputed (one CTA a row, so the residual
// may differ from the forward's in the last bits; the forward's gate output
// pins a hard gate), the vector-Jacobian product with
// respect to the frame (u, B, C, t, cpi), the state in and the parameters,
// given the upstream gradients of y (before proj_out), the gate output (1 on
// a first observation), resid, innov and the state out:
//   hc = g h_upd + (1-g) x_hat:  g_bar += Re(conj(a_hc)(h_upd - x_hat)),
//   state' = g new + (1-g) old:   g_bar += sum Re(conj(a')(new - old)),
//   g = sigmoid((r - eps_l)/T) in the backward (STE / soft; mode 2: none),
//   r = |obs - pred| / (|obs| + eta), innov with obs held constant,
//   eps_l = max(eps (1 - m clamp(cpi, 0, 1)), 1e-3) (-1 on a first step),
// then the readout, prediction and ZOH adjoints as in the cell backward.
// A first observation takes its own frame as predecessor, so the
// predecessor's adjoints go to the frame; a masked row passes the state's
// adjoints through.  Per-row partials of lam, log_dt, D and eps are summed
// by stream_bwd_post in row order.
// ---------------------------------------------------------------------------
struct SbArgs {
    const float2* lam;
    const float* log_dt;
    const float* D;
    const float* mean;
    const float* var;
    const float* u;        // (B,H)
    const float2* Bc;      // (B,N)
    const float2* Cc;
    const float* t;        // (B)
    const uint8_t* valid;  // (B) or null
    const float* cpi;      // (B) or null
    const float2* h_in;    // (B,H,N)
    const float* t_in;
    const float* u_in;
    const float2* B_in;
    const float2* C_in;
    const uint8_t* init_in;
    const float* gate;     // (B) forward gate output or null
    const float* gy;       // (B,H) or null
    const float* gg;       // (B) or null
    const float* gr;
    const float* gn;
    const float2* gh;      // (B,H,N) or null
    const float* gt;       // (B) or null
    const float* gu;       // (B,H) or null
    const float2* gB;      // (B,N) or null
    const float2* gC;
    float* du;
    float2* dBc;
    float2* dCc;
    float* dt;
    float* dcpi;           // or null
    float2* dh_in;
    float* dt_in;
    float* du_in;
    float2* dB_in;
    float2* dC_in;
    float2* dlam;
    float* dlog;
    float* dD;
    float* deps;
    float2* plam;          // [B][H][N] per-row partials
    float* plog;           // [B][H]
    float* pD;
    float* peps;           // [B]
    float eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, Tp;
    int gate_mode;         // 0 STE, 1 soft, 2 hard (no gradient through the gate)
    int B, H, N;
};

__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float redot(float2 a, float2 b) { return a.x * b.x + a.y * b.y; }  // Re(conj(a) b)

template <int LANES>
__device__ __forceinline__ float lane_sum(float v) {
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// sum over the CTA in a fixed order (warps, then warp 0..NW-1); every thread
// gets the total
__device__ __forceinline__ float cta_sum(float v, float* sred, float* sout) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < kST / 32; ++w) s += sred[w];
        *sout = s;
    }
    __syncthreads();
    return *sout;
}

template <int LANES, int NPT>
__global__ void __launch_bounds__(kST) stream_step_bwd_k(SbArgs a) {
    constexpr int HG = kST / LANES;
    constexpr int NP = LANES * NPT;
    constexpr int NW = kST / 32;
    extern __shared__ __align__(16) unsigned char sdyn[];
    float2* sacc = reinterpret_cast<float2*>(sdyn);                // [4][NW][NP]
    float* sdv = reinterpret_cast<float*>(sacc + 4 * NW * NP);     // [H] residual terms, then obs' adjoint / sd
    float* sob = sdv + a.H;                                       // [H] obs, then pred's adjoint / sd
    __shared__ float2 sB0[NP], sC0[NP], sBf[NP], sCf[NP];
    __shared__ float2 sred2[NW];
    __shared__ float sred[NW];
    __shared__ float sv[12];

    const int b = blockIdx.x;
    const int tid = threadIdx.x, ln = tid % LANES, hg = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const int H = a.H, N = a.N;
    const size_t HN = static_cast<size_t>(H) * N;
    const size_t bHN = static_cast<size_t>(b) * HN;
    const size_t bH = static_cast<size_t>(b) * H;
    const bool v = a.valid ? a.valid[b] != 0 : true;
    if (!v) {  // masked row: the state passes through, nothing else
        for (size_t i = tid; i < HN; i += kST) {
            a.dh_in[bHN + i] = a.gh ? a.gh[bHN + i] : make_float2(0.f, 0.f);
            a.plam[bHN + i] = make_float2(0.f, 0.f);
        }
        for (int h = tid; h < H; h += kST) {
            a.du_in[bH + h] = a.gu ? a.gu[bH + h] : 0.f;
            a.du[bH + h] = 0.f;
            a.plog[bH + h] = 0.f;
            a.pD[bH + h] = 0.f;
        }
        for (int n = tid; n < N; n += kST) {
            const size_t o = static_cast<size_t>(b) * N + n;
            a.dB_in[o] = a.gB ? a.gB[o] : make_float2(0.f, 0.f);
            a.dC_in[o] = a.gC ? a.gC[o] : make_float2(0.f, 0.f);
            a.dBc[o] = a.dCc[o] = make_float2(0.f, 0.f);
        }
        if (tid == 0) {
            a.dt_in[b] = a.gt ? a.gt[b] : 0.f;
            a.dt[b] = 0.f;
            if (a.dcpi) a.dcpi[b] = 0.f;
            a.peps[b] = 0.f;
        }
        return;
    }
    const bool first = a.init_in[b] == 0;
    const float tl = a.t[b];
    const float t0 = first ? tl - a.dt_init : a.t_in[b];
    for (int n = tid; n < NP; n += kST) {
        const size_t o = static_cast<size_t>(b) * N + n;
        const float2 z = make_float2(0.f, 0.f);
        sBf[n] = n < N ? a.Bc[o] : z;
        sCf[n] = n < N ? a.Cc[o] : z;
        sB0[n] = n < N ? (first ? a.Bc[o] : a.B_in[o]) : z;
        sC0[n] = n < N ? (first ? a.Cc[o] : a.C_in[o]) : z;
    }
    __syncthreads();
    const float draw = tl - t0;
    const float delta = fmaxf(draw, 0.f);
    const float mdel = draw >= 0.f ? 1.f : 0.f;
    auto u0_of = [&](int h) { return first ? a.u[bH + h] : a.u_in[bH + h]; };

    // ---- pass 1: prediction and residual (one CTA a row) ----
    float acc1 = 0.f, acc2 = 0.f;
    for (int h0 = 0; h0 < H; h0 += HG) {
        const int h = h0 + hg;
        const bool hv = h < H;
        float yhp = 0.f, dte = 0.f, upv = 0.f;
        if (hv) {
            dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
            upv = u0_of(h);
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (hv && n < N) {
                const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                float2 dA, dB;
                zoh(lm, crecip(lm), dte, dA, dB);
                const float2 P = cmul(dA, a.h_in[bHN + static_cast<size_t>(h) * N + n]);
                const float2 q = cmul(dB, sB0[n]);
                const float2 xh = make_float2(fmaf(q.x, upv, P.x), fmaf(q.y, upv, P.y));
                yhp += cre_mul(sC0[n], xh);
            }
        }
        yhp = lane_sum<LANES>(yhp);
        if (ln == 0 && hv) {
            const float sd = sqrtf(a.var[h] + a.var_eps);
            const float obs = (a.u[bH + h] - a.mean[h]) / sd;
            const float pred = (yhp - a.mean[h]) / sd;
            const float d = obs - pred;
            sdv[h] = d;
            sob[h] = obs;
            acc1 += d * d;
            acc2 += obs * obs;
        }
    }
    acc1 = warp_sum(acc1);
    acc2 = warp_sum(acc2);
    if (lane == 0) sred2[wid] = make_float2(acc1, acc2);
    __syncthreads();
    const bool mod = a.cpi != nullptr && a.cpi_mod > 0.f;
    if (tid == 0) {
        float s1 = 0.f, s2 = 0.f;
        for (int w = 0; w < NW; ++w) {
            s1 += sred2[w].x;
            s2 += sred2[w].y;
        }
        const float num = sqrtf(s1), nobs = sqrtf(s2), den = nobs + a.eta;
        const float r = num / den;
        float epsl = first ? -1.f : a.eps, e1 = epsl, c = 0.f;
        if (mod) {
            c = fminf(fmaxf(a.cpi[b], 0.f), 1.f);
            e1 = epsl * (1.f - a.cpi_mod * c);
            epsl = fmaxf(e1, 1e-3f);
        }
        const float soft = 1.0f / (1.0f + expf(-((r - epsl) / a.Tp)));
        float g = a.gate_mode == 1 ? soft : (r > epsl ? 1.f : 0.f);
        if (a.gate_mode != 1 && a.gate && !first) g = a.gate[b];
        sv[0] = g;
        sv[1] = soft;
        sv[2] = num;
        sv[3] = nobs;
        sv[4] = den;
        sv[5] = e1;
        sv[6] = c;
    }
    __syncthreads();
    const float g = sv[0], soft = sv[1], num = sv[2], nobs = sv[3], den = sv[4];

    // ---- pass 2: the gate's adjoint ----
    float gl = 0.f;
    for (int h0 = 0; h0 < H; h0 += HG) {
        const int h = h0 + hg;
        const bool hv = h < H;
        float dte = 0.f, upv = 0.f, ul = 0.f, yb = 0.f;
        if (hv) {
            dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
            upv = u0_of(h);
            ul = a.u[bH + h];
            yb = a.gy ? a.gy[bH + h] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (hv && n < N) {
                const size_t o = bHN + static_cast<size_t>(h) * N + n;
                const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                float2 dA, dB;
                zoh(lm, crecip(lm), dte, dA, dB);
                const float2 h0v = a.h_in[o];
                const float2 P = cmul(dA, h0v);
                const float2 qp = cmul(dB, sB0[n]), qc = cmul(dB, sBf[n]);
                const float2 xh = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                const float2 hu = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                float2 ahc = cscale(conjf2(sCf[n]), yb);
                const float2 Ah = a.gh ? a.gh[o] : make_float2(0.f, 0.f);
                if (first) ahc = cadd(ahc, Ah);
                else gl += redot(Ah, make_float2(hu.x - h0v.x, hu.y - h0v.y));
                gl += redot(ahc, make_float2(hu.x - xh.x, hu.y - xh.y));
            }
        }
        if (!first && hv && ln == 0 && a.gu) gl += a.gu[bH + h] * (ul - upv);
    }
    float gbar = cta_sum(gl, sred, &sv[7]);
    if (tid == 0) {
        if (!first) {
            if (a.gt) gbar += a.gt[b] * (tl - t0);
            for (int n = 0; n < N; ++n) {
                const size_t o = static_cast<size_t>(b) * N + n;
                if (a.gB) gbar += redot(a.gB[o], make_float2(sBf[n].x - sB0[n].x, sBf[n].y - sB0[n].y));
                if (a.gC) gbar += redot(a.gC[o], make_float2(sCf[n].x - sC0[n].x, sCf[n].y - sC0[n].y));
            }
            if (a.gg) gbar += a.gg[b];
        }
        const float xbar = a.gate_mode == 2 ? 0.f : gbar * soft * (1.f - soft) / a.Tp;
        const float rbar = (a.gr ? a.gr[b] : 0.f) + xbar;
        float pe = 0.f, dc = 0.f;
        if (!first) {
            const float ebar = -xbar;
            if (mod) {
                if (sv[5] >= 1e-3f) {
                    pe = ebar * (1.f - a.cpi_mod * sv[6]);
                    const float cr = a.cpi[b];
                    if (cr >= 0.f && cr <= 1.f) dc = -ebar * a.eps * a.cpi_mod;
                }
            } else {
                pe = ebar;
            }
        }
        a.peps[b] = pe;
        if (a.dcpi) a.dcpi[b] = dc;
        const float nbar = (!first && a.gn) ? a.gn[b] : 0.f;
        sv[8] = rbar / den;                 // num's adjoint
        sv[9] = -rbar * num / (den * den);  // den's adjoint
        sv[10] = nbar / den;                // innov's num's adjoint
    }
    __syncthreads();
    {
        const float numbar = sv[8], denbar = sv[9], numnbar = sv[10];
        for (int h = tid; h < H; h += kST) {
            const float d = sdv[h], obs = sob[h];
            const float dbar = num > 0.f ? numbar * d / num : 0.f;
            const float obar = dbar + (nobs > 0.f ? denbar * obs / nobs : 0.f);
            const float pbar = -dbar - (num > 0.f ? numnbar * d / num : 0.f);
            const float sd = sqrtf(a.var[h] + a.var_eps);
            sdv[h] = obar / sd;
            sob[h] = pbar / sd;
        }
    }
    __syncthreads();

    // ---- pass 3: readout, prediction and ZOH adjoints ----
    float2 aBf[NPT], aCf[NPT], aB0[NPT], aC0[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) aBf[j] = aCf[j] = aB0[j] = aC0[j] = make_float2(0.f, 0.f);
    float dsum = 0.f;
    for (int h0 = 0; h0 < H; h0 += HG) {
        const int h = h0 + hg;
        const bool hv = h < H;
        float sc = 1.f, dte = 0.f, mdt = 0.f, upv = 0.f, ul = 0.f, yb = 0.f, yhb = 0.f;
        if (hv) {
            sc = expf(a.log_dt[h]);
            const float raw = delta * sc;
            dte = fminf(fmaxf(raw, a.dt_min), a.dt_max);
            mdt = (raw >= a.dt_min && raw <= a.dt_max) ? 1.f : 0.f;
            upv = u0_of(h);
            ul = a.u[bH + h];
            yb = a.gy ? a.gy[bH + h] : 0.f;
            yhb = sob[h];
        }
        float s_u0 = 0.f, s_ul = 0.f, s_dte = 0.f;
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (hv && n < N) {
                const size_t o = bHN + static_cast<size_t>(h) * N + n;
                const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                const float2 il = crecip(lm);
                float2 dA, dB;
                zoh(lm, il, dte, dA, dB);
                const float2 h0v = a.h_in[o];
                const float2 P = cmul(dA, h0v);
                const float2 qp = cmul(dB, sB0[n]), qc = cmul(dB, sBf[n]);
                const float2 xh = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                const float2 hu = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                const float2 hc = cadd(cscale(hu, g), cscale(xh, 1.f - g));
                const float2 Ah = a.gh ? a.gh[o] : make_float2(0.f, 0.f);
                float2 ahc = cscale(conjf2(sCf[n]), yb);
                float2 ahu, ah0;
                if (first) {
                    ahc = cadd(ahc, Ah);
                    ahu = cscale(ahc, g);
                    ah0 = make_float2(0.f, 0.f);
                } else {
                    ahu = cscale(cadd(ahc, Ah), g);
                    ah0 = cscale(Ah, 1.f - g);
                }
                const float2 axh = cadd(cscale(ahc, 1.f - g), cscale(conjf2(sC0[n]), yhb));
                aCf[j] = cadd(aCf[j], cscale(conjf2(hc), yb));
                aC0[j] = cadd(aC0[j], cscale(conjf2(xh), yhb));
                const float2 aP = cadd(axh, ahu);
                const float2 aqp = cscale(axh, upv), aqc = cscale(ahu, ul);
                s_u0 += redot(axh, qp);
                s_ul += redot(ahu, qc);
                const float2 adB = cadd(cmul(aqp, conjf2(sB0[n])), cmul(aqc, conjf2(sBf[n])));
                const float2 cdA = conjf2(dA), cdB = conjf2(dB);
                aB0[j] = cadd(aB0[j], cmul(cdB, aqp));
                aBf[j] = cadd(aBf[j], cmul(cdB, aqc));
                const float2 adA = cmul(aP, conjf2(h0v));
                a.dh_in[o] = cadd(ah0, cmul(cdA, aP));
                const float2 aE = cmul(adB, conjf2(il));
                float2 alm = cmul(make_float2(-aE.x, -aE.y), cdB);
                const float2 az = cmul(cdA, cadd(adA, aE));
                alm = cadd(alm, cscale(az, dte));
                a.plam[o] = alm;
                s_dte += az.x * lm.x + az.y * lm.y;
            }
        }
        s_u0 = lane_sum<LANES>(s_u0);
        s_ul = lane_sum<LANES>(s_ul);
        s_dte = lane_sum<LANES>(s_dte);
        if (hv && ln == 0) {
            const float drb = mdt * s_dte;
            a.plog[bH + h] = drb * delta * sc;
            dsum += drb * sc;
            const float Au = a.gu ? a.gu[bH + h] : 0.f;
            const float dul = yb * a.D[h] + (first ? Au : g * Au) + sdv[h] + s_ul;
            const float du0 = (first ? 0.f : (1.f - g) * Au) + s_u0;
            a.du[bH + h] = first ? dul + du0 : dul;
            a.du_in[bH + h] = first ? 0.f : du0;
            a.pD[bH + h] = yb * ul;
        }
    }
    // B's and C's adjoints summed over the channels (frame and predecessor)
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        float2* q[4] = {&aBf[j], &aCf[j], &aB0[j], &aC0[j]};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int o = LANES; o < 32; o <<= 1) {
                q[k]->x += __shfl_xor_sync(0xffffffffu, q[k]->x, o);
                q[k]->y += __shfl_xor_sync(0xffffffffu, q[k]->y, o);
            }
            if (lane < LANES) sacc[(k * NW + wid) * NP + ln + LANES * j] = *q[k];
        }
    }
    const float deltabar = cta_sum(dsum, sred, &sv[11]);  // its barriers also publish sacc
    for (int n = tid; n < N; n += kST) {
        float2 s4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float2 sum = make_float2(0.f, 0.f);
            for (int w = 0; w < NW; ++w) sum = cadd(sum, sacc[(k * NW + w) * NP + n]);
            s4[k] = sum;
        }
        const size_t o = static_cast<size_t>(b) * N + n;
        const float2 AB = a.gB ? a.gB[o] : make_float2(0.f, 0.f);
        const float2 AC = a.gC ? a.gC[o] : make_float2(0.f, 0.f);
        if (first) {
            a.dBc[o] = cadd(cadd(s4[0], AB), s4[2]);
            a.dCc[o] = cadd(cadd(s4[1], AC), s4[3]);
            a.dB_in[o] = a.dC_in[o] = make_float2(0.f, 0.f);
        } else {
            a.dBc[o] = cadd(s4[0], cscale(AB, g));
            a.dCc[o] = cadd(s4[1], cscale(AC, g));
            a.dB_in[o] = cadd(cscale(AB, 1.f - g), s4[2]);
            a.dC_in[o] = cadd(cscale(AC, 1.f - g), s4[3]);
        }
    }
    if (tid == 0) {
        const float At = a.gt ? a.gt[b] : 0.f;
        const float dtl = (first ? At : g * At) + mdel * deltabar;
        const float dt0 = (first ? 0.f : (1.f - g) * At) - mdel * deltabar;
        a.dt[b] = first ? dtl + dt0 : dtl;
        a.dt_in[b] = first ? 0.f : dt0;
    }
}

__global__ void stream_bwd_post(SbArgs a) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t HN = static_cast<int64_t>(a.H) * a.N;
    if (i < HN) {
        float2 s = make_float2(0.f, 0.f);
        for (int b = 0; b < a.B; ++b) s = cadd(s, a.plam[b * HN + i]);
        a.dlam[i] = s;
    }
    if (i < a.H) {
        float s1 = 0.f, s2 = 0.f;
        for (int b = 0; b < a.B; ++b) {
            s1 += a.plog[static_cast<size_t>(b) * a.H + i];
            s2 += a.pD[static_cast<size_t>(b) * a.H + i];
        }
        a.dlog[i] = s1;
        a.dD[i] = s2;
    }
    if (i == 0) {
        float s = 0.f;
        for (int b = 0; b < a.B; ++b) s += a.peps[b];
        a.deps[0] = s;
    }
}

size_t als(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

template <int LANES, int NPT>
cudaError_t launch_step_bwd(const SbArgs& a, cudaStream_t s) {
    const size_t smem = sizeof(float2) * 4 * (kST / 32) * LANES * NPT + sizeof(float) * 2 * a.H;
    cudaError_t e = cudaFuncSetAttribute(stream_step_bwd_k<LANES, NPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    stream_step_bwd_k<LANES, NPT><<<a.B, kST, smem, s>>>(a);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int64_t n = std::max<int64_t>(static_cast<int64_t>(a.H) * a.N, 1);
    stream_bwd_post<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(a);
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

namespace eacs {

size_t stream_step_bwd_workspace_size(int64_t B, int64_t H, int64_t N) {
    if (B <= 0 || H <= 0 || N <= 0) return 0;
    return als(sizeof(float2) * B * H * N) + 2 * als(sizeof(float) * B * H) + als(sizeof(float) * B);
}

int stream_step_bwd(const StreamBwdCall& c, cudaStream_t stream) {
    const char* fn = "eacs_stream_step_bwd";
    if (c.B < 0 || c.H < 0 || c.N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)c.N);
    if (c.B > (1LL << 31) - 1 || c.H > 20000)
        return fail(EACS_ERR_UNSUPPORTED, "%s: B or H too large", fn);
    if (c.gate_mode < 0 || c.gate_mode > 2) return fail(EACS_ERR_INVALID, "%s: gate_mode %d not in 0..2", fn, c.gate_mode);
    if (c.B == 0) return EACS_OK;
    if (c.H == 0 || c.N == 0) return fail(EACS_ERR_INVALID, "%s: H and N must be positive", fn);
    if (!c.lam || !c.log_dt || !c.D || !c.mean || !c.var || !c.u || !c.Bc || !c.Cc || !c.t || !c.h_in ||
        !c.t_in || !c.u_in || !c.B_in || !c.C_in || !c.init_in || !c.du || !c.dBc || !c.dCc || !c.dt ||
        !c.dh_in || !c.dt_in || !c.du_in || !c.dB_in || !c.dC_in || !c.dlam || !c.dlog || !c.dD || !c.deps)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    const size_t need = stream_step_bwd_workspace_size(c.B, c.H, c.N);
    if (!c.workspace || c.workspace_bytes < need)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, need, c.workspace_bytes);
    SbArgs a{};
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
    a.gate = c.gate;
    a.gy = c.gy;
    a.gg = c.gg;
    a.gr = c.gr;
    a.gn = c.gn;
    a.gh = static_cast<const float2*>(c.gh);
    a.gt = c.gt;
    a.gu = c.gu;
    a.gB = static_cast<const float2*>(c.gB);
    a.gC = static_cast<const float2*>(c.gC);
    a.du = c.du;
    a.dBc = static_cast<float2*>(c.dBc);
    a.dCc = static_cast<float2*>(c.dCc);
    a.dt = c.dt;
    a.dcpi = c.dcpi;
    a.dh_in = static_cast<float2*>(c.dh_in);
    a.dt_in = c.dt_in;
    a.du_in = c.du_in;
    a.dB_in = static_cast<float2*>(c.dB_in);
    a.dC_in = static_cast<float2*>(c.dC_in);
    a.dlam = static_cast<float2*>(c.dlam);
    a.dlog = c.dlog;
    a.dD = c.dD;
    a.deps = c.deps;
    char* ws = static_cast<char*>(c.workspace);
    const size_t o1 = als(sizeof(float2) * c.B * c.H * c.N), o2 = als(sizeof(float) * c.B * c.H);
    a.plam = reinterpret_cast<float2*>(ws);
    a.plog = reinterpret_cast<float*>(ws + o1);
    a.pD = reinterpret_cast<float*>(ws + o1 + o2);
    a.peps = reinterpret_cast<float*>(ws + o1 + 2 * o2);
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
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    cudaError_t e;
    const int64_t N = c.N;
    if (N <= 4) e = launch_step_bwd<4, 1>(a, stream);
    else if (N <= 8) e = launch_step_bwd<8, 1>(a, stream);
    else if (N <= 16) e = launch_step_bwd<16, 1>(a, stream);
    else if (N <= 32) e = launch_step_bwd<32, 1>(a, stream);
    else e = launch_step_bwd<32, 2>(a, stream);
    return cuda_check(e, fn);
}

}  // namespace eacs
