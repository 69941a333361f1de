// train.cu -- backward of the gated EACS cell (GatedEACSCellFunction) on sm_100a.
//
// Reference: cst_ssm/ops/eacs_cell_train.py:117-175 runs, per step in reverse,
// torch.autograd.grad of _step_functional (eacs_cell_train.py:15-66) with the
// forward's hard gates pinned (STE) or the soft gate.  This file evaluates the
// same vector-Jacobian product by hand (the derivation is restated in the CPU
// oracle, oracle/eacs_oracle.c, eacs_oracle_cell_bwd, and checked there
// against the reference's autograd):
//
//   per step l (reverse), chain (h, n), with hf = dA h_pi, q = dB_bar B,
//   x_hat = hf + q_pi u_pi, h_upd = hf + q_l u_l, h_cur = g h_upd + (1-g) x_hat
//     g_bar  = g_gs + sum Re(conj(a_hcur)(h_upd - x_hat)) + sum Re(conj(a_h)(h_upd - h_pi))
//              + a_t (t_l - t_pi) + sum a_u (u_l - u_pi) + sum Re(conj(a_B)(B_l - B_pi)) + ...C
//     r_bar  = g_rs + g_bar s(1-s)/T,  s = sigmoid((r - eps)/T)
//     then the residual, readout, blend, ZOH and clamp adjoints.
//
// Only g_bar couples the chains of a row within a step: every other row-level
// carry (the adjoints of t_pi, u_pi, B_pi, C_pi) is linear, so each chain (or
// channel) carries its own share and adds its share's term to the g_bar sum.
// A row is one thread-block cluster; g_bar is one float reduced per step
// through distributed shared memory: every warp sends its partial to every
// CTA with st.async, which counts the bytes on that CTA's mbarrier, and each
// CTA waits on its own barrier (no cluster-wide barrier per step).  States come from checkpoints every kK
// steps written by a gated forward pass, recomputed into shared memory one
// chunk at a time.
#include <cooperative_groups.h>

#include <algorithm>
#include <type_traits>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace cg = cooperative_groups;

namespace eacs {
namespace {

#ifndef EACS_TRAIN_KMAX
#define EACS_TRAIN_KMAX 16
#endif
constexpr int kKMax = EACS_TRAIN_KMAX;  // steps per checkpoint / recompute chunk (at most)
constexpr int kCkThreads = 128; // checkpoint kernel CTA

struct TArgs {
    const float2* lam;
    const float* log_dt;
    const void* u;
    const float2* Bc;
    const float2* Cc;
    const float* t;
    const float* D;
    const float* mean;
    const float* var;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, Tp;
    const float* gates;   // (B,L) forward gate values (hard 0/1 for STE, soft values for soft)
    const float* resid;   // (B,L)
    const float2* stats;  // (B,L) (||obs - pred||, ||obs||)
    const float* gy;      // (B,L,H)
    const float* ggs;     // (B,L) or null
    const float* grs;
    const float* gns;
    float* du;            // (B,L,H)
    float2* dBc;          // (B,L,N)
    float2* dCc;
    float* dt;            // (B,L)
    float2* dlam;         // (H,N)
    float* dlog;          // (H)
    float* dD;            // (H)
    float* deps;          // (1)
    // workspace
    float2* ck_h;         // [B][nK][H][N] state before step k*kK
    float* ck_u;          // [B][nK][H]    u_pi before step k*kK
    float4* ck_row;       // [B][nK]       (t_pi, -, -, -)
    float2* ck_bc;        // [B][nK][2][N] B_pi, C_pi before step k*kK
    float2* pB;           // [B][CL][L][N] per-CTA partials of dBc
    float2* pC;
    float* pt;            // [B][CL][L]
    float2* plam;         // [B][H][N]
    float* plog;          // [B][H]
    float* pD;            // [B][H]
    float* peps;          // [B]
    // per-frame commits (the state after every step, EACSLayer._commit_range):
    // written by the checkpoint pass when cm_h is set
    float2* cm_h;         // (B,L,H,N)
    float* cm_t;          // (B,L)
    float* cm_u;          // (B,L,H)
    float2* cm_B;         // (B,L,N)
    float2* cm_C;
    // their upstream adjoints, read by the backward when commit_grads is set
    // (any may be null = zero)
    const float2* gc_h;   // (B,L,H,N)
    const float* gc_t;    // (B,L)
    const float* gc_u;    // (B,L,H)
    const float2* gc_B;   // (B,L,N)
    const float2* gc_C;
    int B, L, H, N, nK, CL, HC;
    int K, Klog;          // steps per checkpoint / recompute chunk (K = 1 << Klog)
    int have_ckpt;        // the forward already wrote the checkpoints
    int commit_grads;     // the backward adds the commits' adjoints (extra shared memory)
    int gate_const;       // hard gates that carry no gradient (eval-mode comparison r > eps)
};

template <int LANES>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Gated forward with known gates, writing checkpoints.  Thread layout as the
// chain kernel: (hl, ln) owns chains n = ln + LANES*j of channel h.  Inputs
// (gate, t, u, B, C) are staged in shared memory 32 steps at a time,
// double-buffered: the next chunk is copied in with cp.async while the
// current one runs.
// ---------------------------------------------------------------------------
constexpr int kCkT = 32;  // steps per staged chunk (a multiple of every checkpoint interval)

template <int LANES, int NPT, typename UT>
__global__ void __launch_bounds__(kCkThreads) train_ckpt(TArgs a) {
    constexpr int HT = kCkThreads / LANES;
    constexpr int NP = LANES * NPT;
    constexpr int NBUF = NP <= 32 ? 2 : 1;
    constexpr int PAIR = sizeof(UT) == 4 ? 1 : 2;
    __shared__ float2 sB[NBUF][kCkT][NP];
    __shared__ float2 sC[NBUF][kCkT][NP];
    __shared__ __align__(16) UT su[NBUF][kCkT][HT];
    __shared__ float st[NBUF][kCkT];
    __shared__ float sg[NBUF][kCkT];
    const int tid = threadIdx.x, ln = tid % LANES, hl = tid / LANES;
    const int b = blockIdx.y, h0 = blockIdx.x * HT, h = h0 + hl;
    const bool hv = h < a.H;
    const int L = a.L, H = a.H, N = a.N;
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowL = static_cast<size_t>(b) * L;
    float2 lam[NPT], ilam[NPT], hs[NPT], Bp[NPT], Cp[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        hs[j] = make_float2(0.f, 0.f);
        Bp[j] = nv[j] ? a.Bc[rowL * N + n] : make_float2(0.f, 0.f);
        Cp[j] = nv[j] ? a.Cc[rowL * N + n] : make_float2(0.f, 0.f);
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    float u_pi = hv ? to_f32(u[rowL * H + h]) : 0.f;
    float t_pi = a.t[rowL] - a.dt_init;
    const bool row_writer = blockIdx.x == 0 && tid == 0;
    const bool bc_writer = blockIdx.x == 0 && hl == 0;  // writes B_pi, C_pi into the checkpoints
    const bool async_ok = NBUF == 2 && (PAIR == 1 || (H % 2) == 0) &&
                          (reinterpret_cast<uintptr_t>(u) & 3u) == 0 &&
                          ((reinterpret_cast<uintptr_t>(a.Bc) | reinterpret_cast<uintptr_t>(a.Cc)) & 7u) == 0 &&
                          ((reinterpret_cast<uintptr_t>(a.t) | reinterpret_cast<uintptr_t>(a.gates)) & 3u) == 0;
    auto stage = [&](int c0, int buf, bool async) {
        const int sn = min(kCkT, L - c0);
        for (int idx = tid; idx < sn * NP; idx += kCkThreads) {
            const int i = idx / NP, n = idx % NP;
            const size_t o = (rowL + c0 + i) * N + n;
            if (async) {
                cp_async8(&sB[buf][i][n], n < N ? a.Bc + o : a.Bc, n < N);
                cp_async8(&sC[buf][i][n], n < N ? a.Cc + o : a.Cc, n < N);
            } else {
                sB[buf][i][n] = n < N ? a.Bc[o] : make_float2(0.f, 0.f);
                sC[buf][i][n] = n < N ? a.Cc[o] : make_float2(0.f, 0.f);
            }
        }
        if (async) {
            for (int idx = tid; idx < sn * (HT / PAIR); idx += kCkThreads) {
                const int i = idx / (HT / PAIR), k = (idx % (HT / PAIR)) * PAIR;
                const bool ok = h0 + k < H;
                cp_async4(&su[buf][i][k], ok ? u + (rowL + c0 + i) * H + h0 + k : u, ok);
            }
            for (int i = tid; i < sn; i += kCkThreads) {
                cp_async4(&st[buf][i], a.t + rowL + c0 + i, true);
                cp_async4(&sg[buf][i], a.gates + rowL + c0 + i, true);
            }
            cp_async_commit();
        } else {
            for (int idx = tid; idx < sn * HT; idx += kCkThreads) {
                const int i = idx / HT, k = idx % HT;
                su[buf][i][k] = (h0 + k < H) ? u[(rowL + c0 + i) * H + h0 + k] : static_cast<UT>(0.f);
            }
            for (int i = tid; i < sn; i += kCkThreads) {
                st[buf][i] = a.t[rowL + c0 + i];
                sg[buf][i] = a.gates[rowL + c0 + i];
            }
        }
    };
    if (async_ok) stage(0, 0, true);
    for (int l0 = 0, chunk = 0; l0 < L; l0 += kCkT, ++chunk) {
        const int steps = min(kCkT, L - l0);
        const int buf = chunk & (NBUF - 1);
        if (async_ok) cp_async_wait_all();
        __syncthreads();
        if (!async_ok) {
            stage(l0, buf, false);
            __syncthreads();
        } else if (l0 + kCkT < L) {
            stage(l0 + kCkT, (buf ^ 1) & (NBUF - 1), true);
        }
        for (int i = 0; i < steps; ++i) {
            const int l = l0 + i;
            if ((l & (a.K - 1)) == 0) {  // K is a power of two
                const int k = l >> a.Klog;
#pragma unroll
                for (int j = 0; j < NPT; ++j)
                    if (nv[j]) a.ck_h[((static_cast<size_t>(b) * a.nK + k) * H + h) * N + ln + LANES * j] = hs[j];
                if (hv && ln == 0) a.ck_u[(static_cast<size_t>(b) * a.nK + k) * H + h] = u_pi;
                if (row_writer) a.ck_row[static_cast<size_t>(b) * a.nK + k] = make_float4(t_pi, 0.f, 0.f, 0.f);
                if (bc_writer) {
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const int n = ln + LANES * j;
                        if (n < N) {
                            const size_t o = ((static_cast<size_t>(b) * a.nK + k) * 2) * N + n;
                            a.ck_bc[o] = Bp[j];
                            a.ck_bc[o + N] = Cp[j];
                        }
                    }
                }
            }
            // one step; with G1 the gate is a hard 1 and the (1 - g) terms, which
            // are exactly zero then, are left out.  B_pi and C_pi are row values
            // that only the threads writing them into the checkpoints keep.
            auto step = [&](auto gm) {
                constexpr bool G1 = decltype(gm)::value;
                const float g = G1 ? 1.f : sg[buf][i];
                const float tl = st[buf][i];
                const float ul = to_f32(su[buf][i][hl]);
                const float dte = eff_dt(fmaxf(tl - t_pi, 0.f), scale, a.dt_min, a.dt_max);
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const float2 Bl = sB[buf][i][ln + LANES * j];
                    float2 dA, dB;
                    zoh(lam[j], ilam[j], dte, dA, dB);
                    const float2 hf = cmul(dA, hs[j]);
                    const float2 ql = cmul(dB, Bl);
                    const float2 hu = make_float2(fmaf(ql.x, ul, hf.x), fmaf(ql.y, ul, hf.y));
                    hs[j] = G1 ? hu : cadd(cscale(hu, g), cscale(hs[j], 1.f - g));
                }
                if (bc_writer) {
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const float2 Bl = sB[buf][i][ln + LANES * j];
                        const float2 Cl = sC[buf][i][ln + LANES * j];
                        Bp[j] = G1 ? Bl : cadd(cscale(Bl, g), cscale(Bp[j], 1.f - g));
                        Cp[j] = G1 ? Cl : cadd(cscale(Cl, g), cscale(Cp[j], 1.f - g));
                    }
                }
                u_pi = G1 ? ul : g * ul + (1.f - g) * u_pi;
                t_pi = G1 ? tl : g * tl + (1.f - g) * t_pi;
            };
            if (sg[buf][i] == 1.f) step(std::true_type{});
            else step(std::false_type{});
            if (a.cm_h) {  // the commits of step l: the state after it
                const size_t rl = rowL + l;
#pragma unroll
                for (int j = 0; j < NPT; ++j)
                    if (nv[j]) a.cm_h[(rl * H + h) * N + ln + LANES * j] = hs[j];
                if (hv && ln == 0) a.cm_u[rl * H + h] = u_pi;
                if (row_writer) a.cm_t[rl] = t_pi;
                if (bc_writer) {
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const int n = ln + LANES * j;
                        if (n < N) {
                            a.cm_B[rl * N + n] = Bp[j];
                            a.cm_C[rl * N + n] = Cp[j];
                        }
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// cluster helpers (distributed shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Backward: one cluster of CL CTAs per row, CTA c owns channels
// [c*HC, (c+1)*HC); thread (hl, ln) owns chains n = ln + LANES*j.
// ---------------------------------------------------------------------------
template <int LANES, int NPT, typename UT, int MAXT = 512, bool CG = false>
__global__ void __launch_bounds__(MAXT) train_bwd(TArgs a) {
    constexpr int NP = LANES * NPT;
    extern __shared__ __align__(16) unsigned char smem[];
    const int T = blockDim.x;
    const int NW = T / 32;
    const int HC = a.HC;
    const int kK = a.K;
    // shared layout (see smem_bytes)
    float2* sh = reinterpret_cast<float2*>(smem);                 // [kK][NPT][T] h_pi
    float2* sdA = sh + kK * T * NPT;                              // [kK][NPT][T] dA
    float2* sdB = sdA + kK * T * NPT;                             // [kK][NPT][T] dB_bar
    float2* sBpi = sdB + kK * T * NPT;                            // [kK][NP]
    float2* sCpi = sBpi + kK * NP;
    float2* sBl = sCpi + kK * NP;
    float2* sCl = sBl + kK * NP;
    float2* soB = sCl + kK * NP;                                  // [kK][NW][NP]
    float2* soC = soB + kK * NW * NP;
    float4* srow = reinterpret_cast<float4*>(soC + kK * NW * NP); // [kK] 1/den, num/den^2, 1/num, 1/nobs
    uint64_t* rbar = reinterpret_cast<uint64_t*>(srow + kK);      // [2] reduction mbarriers
    float* slots = reinterpret_cast<float*>(rbar + 2);            // [2][CL*NW] partials of g_bar
    float* f = slots + 2 * 16 * 32;
    float* supi = f;  f += kK * HC;                               // [kK][HC]
    float* sul = f;   f += kK * HC;
    float* sgy = f;   f += kK * HC;
    float* stl = f;   f += kK;
    float* stpi = f;  f += kK;
    float* sgt = f;   f += kK;
    float* sslp = f;  f += kK;                                    // sigmoid slope / T
    float* sgg = f;   f += kK;                                    // g_gs
    float* sgr = f;   f += kK;                                    // g_rs
    float* sgn = f;   f += kK;                                    // g_ns
    float* sot = f;   f += kK * NW;                               // [kK][NW]
    // commit adjoints (commit_grads only): u_pi's and t_pi's per step, B_pi's
    // and C_pi's per step, and a two-step ring of h_pi's prefetched with cp.async
    constexpr bool cm = CG;
    float* sgcu = f;  f += cm ? kK * HC : 0;                      // [kK][HC]
    float* sgct = f;  f += cm ? kK : 0;                           // [kK]
    f += (reinterpret_cast<uintptr_t>(f) & 7u) ? 1 : 0;
    float2* sgcB = reinterpret_cast<float2*>(f);                  // [kK][NP]
    float2* sgcC = sgcB + (cm ? kK * NP : 0);
    float2* sring = sgcC + (cm ? kK * NP : 0);                    // [2][NPT][T]

    cg::cluster_group cluster = cg::this_cluster();
    const int crank = static_cast<int>(cluster.block_rank());
    const int CL = a.CL;
    const int tid = threadIdx.x, ln = tid % LANES, hl = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const int b = blockIdx.y;
    const int h = crank * HC + hl;
    const bool hv = hl < HC && h < a.H;
    const bool row_owner = hl == 0;  // tracks the row-level B_pi, C_pi in the recompute
    const int L = a.L, H = a.H, N = a.N;
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowL = static_cast<size_t>(b) * L;

    float2 lam[NPT], ilam[NPT], ah[NPT], vB[NPT], vC[NPT], glam[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        ah[j] = vB[j] = vC[j] = glam[j] = make_float2(0.f, 0.f);
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float rsd = hv ? 1.0f / sqrtf(a.var[h] + a.var_eps) : 1.f;
    const float mu = hv ? a.mean[h] : 0.f;
    const float Dh = hv ? a.D[h] : 0.f;
    float vu = 0.f, vt = 0.f, glog = 0.f, gD = 0.f, geps = 0.f;
    if (tid == 0) {
        mbar_init(&rbar[0], 1);
        mbar_init(&rbar[1], 1);
        fence_mbar_init();
    }
    // every CTA of the cluster is running, with its barriers initialised,
    // before any remote store
    cluster_sync_all();
    const int nslot = CL * NW;                 // one partial per (source CTA, warp)
    uint32_t rslot[2] = {0u, 0u}, rbarr[2] = {0u, 0u};
    if (lane < CL) {                           // lane c sends to CTA c
        rslot[0] = mapa_u32(&slots[crank * NW + wid], lane);
        rslot[1] = mapa_u32(&slots[16 * 32 + crank * NW + wid], lane);
        rbarr[0] = mapa_u32(&rbar[0], lane);
        rbarr[1] = mapa_u32(&rbar[1], lane);
    }
    int nred = 0;                              // reductions done so far
    bool failed = false;
    // the adjoint of h_pi's commit at step l into ring slot l & 1 (zero for
    // padded chains)
    const bool cmh = cm && a.gc_h != nullptr;
    auto prefetch_gch = [&](const int l) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            cp_async8(&sring[((l & 1) * NPT + j) * T + tid],
                      nv[j] ? a.gc_h + ((rowL + l) * H + h) * N + n : a.gc_h, nv[j]);
        }
        cp_async_commit();
    };
    if (cmh) prefetch_gch(L - 1);

    for (int k = a.nK - 1; k >= 0; --k) {
        const int l0 = k * kK;
        const int steps = min(kK, L - l0);
        __syncthreads();
        // ---- stage per-step inputs of the chunk ----
        for (int idx = tid; idx < steps * NP; idx += T) {
            const int i = idx / NP, n = idx % NP;
            const size_t o = (rowL + l0 + i) * N + n;
            sBl[i * NP + n] = n < N ? a.Bc[o] : make_float2(0.f, 0.f);
            sCl[i * NP + n] = n < N ? a.Cc[o] : make_float2(0.f, 0.f);
        }
        for (int idx = tid; idx < steps * HC; idx += T) {
            const int i = idx / HC, c = idx % HC, hh = crank * HC + c;
            const bool ok = hh < H;
            sul[i * HC + c] = ok ? to_f32(u[(rowL + l0 + i) * H + hh]) : 0.f;
            sgy[i * HC + c] = ok ? a.gy[(rowL + l0 + i) * H + hh] : 0.f;
        }
        for (int i = tid; i < steps; i += T) {
            const size_t o = rowL + l0 + i;
            stl[i] = a.t[o];
            sgt[i] = a.gates[o];
            const float soft = 1.0f / (1.0f + expf(-((a.resid[o] - a.eps) / a.Tp)));
            sslp[i] = a.gate_const ? 0.f : soft * (1.f - soft) / a.Tp;
            const float2 st = a.stats[o];
            const float num = st.x, nobs = st.y, den = nobs + a.eta;
            const float rden = 1.0f / den;
            srow[i] = make_float4(rden, num * rden * rden, num > 0.f ? 1.0f / num : 0.f,
                                  nobs > 0.f ? 1.0f / nobs : 0.f);
            sgg[i] = a.ggs ? a.ggs[o] : 0.f;
            sgr[i] = a.grs ? a.grs[o] : 0.f;
            sgn[i] = a.gns ? a.gns[o] : 0.f;
            if (cm) sgct[i] = a.gc_t ? a.gc_t[o] : 0.f;
        }
        if (cm) {
            for (int idx = tid; idx < steps * HC; idx += T) {
                const int i = idx / HC, c = idx % HC, hh = crank * HC + c;
                sgcu[i * HC + c] = (a.gc_u && hh < H) ? a.gc_u[(rowL + l0 + i) * H + hh] : 0.f;
            }
            for (int idx = tid; idx < steps * NP; idx += T) {
                const int i = idx / NP, n = idx % NP;
                const size_t o = (rowL + l0 + i) * N + n;
                sgcB[i * NP + n] = (a.gc_B && n < N) ? a.gc_B[o] : make_float2(0.f, 0.f);
                sgcC[i * NP + n] = (a.gc_C && n < N) ? a.gc_C[o] : make_float2(0.f, 0.f);
            }
        }
        // ---- forward recompute of the chunk from its checkpoint ----
        float2 hs[NPT], Bp[NPT], Cp[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            const size_t o = ((static_cast<size_t>(b) * a.nK + k) * H + (hv ? h : 0)) * N + (n < N ? n : 0);
            hs[j] = nv[j] ? a.ck_h[o] : make_float2(0.f, 0.f);
            Bp[j] = Cp[j] = make_float2(0.f, 0.f);
            if (row_owner && n < N) {
                const size_t ob = ((static_cast<size_t>(b) * a.nK + k) * 2) * N + n;
                Bp[j] = a.ck_bc[ob];
                Cp[j] = a.ck_bc[ob + N];
            }
        }
        float u_pi = hv ? a.ck_u[(static_cast<size_t>(b) * a.nK + k) * H + h] : 0.f;
        float t_pi = a.ck_row[static_cast<size_t>(b) * a.nK + k].x;
        __syncthreads();
        // one step; with G1 the gate is a hard 1 and the (1 - g) terms, which
        // are exactly zero then, are left out
        auto forward_step = [&](auto gm, const int i) {
            constexpr bool G1 = decltype(gm)::value;
            const float g = G1 ? 1.f : sgt[i];
            const float tl = stl[i];
            const float ul = hv ? sul[i * HC + hl] : 0.f;
            if (hv && ln == 0) supi[i * HC + hl] = u_pi;
            if (tid == 0) stpi[i] = t_pi;
            const float dte = eff_dt(fmaxf(tl - t_pi, 0.f), scale, a.dt_min, a.dt_max);
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                const size_t so = (static_cast<size_t>(i) * NPT + j) * T + tid;
                sh[so] = hs[j];
                const float2 Bl = sBl[i * NP + n];
                float2 dA, dB;
                zoh(lam[j], ilam[j], dte, dA, dB);
                sdA[so] = dA;
                sdB[so] = dB;
                const float2 hf = cmul(dA, hs[j]);
                const float2 ql = cmul(dB, Bl);
                const float2 hu = make_float2(fmaf(ql.x, ul, hf.x), fmaf(ql.y, ul, hf.y));
                hs[j] = G1 ? hu : cadd(cscale(hu, g), cscale(hs[j], 1.f - g));
            }
            if (row_owner) {  // warp 0 only: row-level B_pi, C_pi before each step
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const int n = ln + LANES * j;
                    sBpi[i * NP + n] = Bp[j];
                    sCpi[i * NP + n] = Cp[j];
                    const float2 Bl = sBl[i * NP + n], Cl = sCl[i * NP + n];
                    Bp[j] = G1 ? Bl : cadd(cscale(Bl, g), cscale(Bp[j], 1.f - g));
                    Cp[j] = G1 ? Cl : cadd(cscale(Cl, g), cscale(Cp[j], 1.f - g));
                }
            }
            u_pi = G1 ? ul : g * ul + (1.f - g) * u_pi;
            t_pi = G1 ? tl : g * tl + (1.f - g) * t_pi;
        };
        for (int i = 0; i < steps; ++i) {
            if (sgt[i] == 1.f) forward_step(std::true_type{}, i);
            else forward_step(std::false_type{}, i);
        }
        __syncthreads();

        // ---- reverse over the chunk ----
        auto reverse_step = [&](auto gm, const int i) {
            constexpr bool G1 = decltype(gm)::value;
            const int l = l0 + i;
            const float g = G1 ? 1.f : sgt[i];
            const float tl = stl[i], tpi = stpi[i];
            const float ul = hv ? sul[i * HC + hl] : 0.f;
            const float upi = hv ? supi[i * HC + hl] : 0.f;
            const float yb = hv ? sgy[i * HC + hl] : 0.f;
            if (cm) {
                // the commits of step l are the state after it: their upstream
                // adjoints join the carried ones (u_pi's and t_pi's are kept
                // per channel on every lane, B_pi's and C_pi's as shares summed
                // over the row's channels, so channel 0 takes those)
                if (cmh) {
                    cp_async_wait_all();
                    if (l > 0) prefetch_gch(l - 1);
#pragma unroll
                    for (int j = 0; j < NPT; ++j) ah[j] = cadd(ah[j], sring[((l & 1) * NPT + j) * T + tid]);
                }
                if (hv) vu += sgcu[i * HC + hl];
                if (crank == 0 && hl == 0) {
                    vt += sgct[i];
#pragma unroll
                    for (int j = 0; j < NPT; ++j) {
                        const int n = ln + LANES * j;
                        vB[j] = cadd(vB[j], sgcB[i * NP + n]);
                        vC[j] = cadd(vC[j], sgcC[i * NP + n]);
                    }
                }
            }
            const float draw = tl - tpi;
            const float delta = fmaxf(draw, 0.f);
            const float mdel = draw >= 0.f ? 1.f : 0.f;
            const float dte_raw = delta * scale;
            const float dte = fminf(fmaxf(dte_raw, a.dt_min), a.dt_max);
            const float mdt = (dte_raw >= a.dt_min && dte_raw <= a.dt_max) ? 1.f : 0.f;
            float2 hp[NPT], dA[NPT], dB[NPT], xh[NPT], hu[NPT], qp[NPT], ql[NPT];
            float yhp = 0.f, gl = 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                const size_t so = (static_cast<size_t>(i) * NPT + j) * T + tid;
                hp[j] = sh[so];
                dA[j] = sdA[so];
                dB[j] = sdB[so];
                const float2 Bl = sBl[i * NP + n], Bpi = sBpi[i * NP + n];
                const float2 Cl = sCl[i * NP + n], Cpi = sCpi[i * NP + n];
                const float2 hf = cmul(dA[j], hp[j]);
                qp[j] = cmul(dB[j], Bpi);
                ql[j] = cmul(dB[j], Bl);
                xh[j] = make_float2(fmaf(qp[j].x, upi, hf.x), fmaf(qp[j].y, upi, hf.y));
                hu[j] = make_float2(fmaf(ql[j].x, ul, hf.x), fmaf(ql[j].y, ul, hf.y));
                yhp += cre_mul(Cpi, xh[j]);
                // local share of g_bar
                const float2 ahc = make_float2(yb * Cl.x, -yb * Cl.y);  // yb conj(C_l)
                gl += ahc.x * (hu[j].x - xh[j].x) + ahc.y * (hu[j].y - xh[j].y);
                gl += ah[j].x * (hu[j].x - hp[j].x) + ah[j].y * (hu[j].y - hp[j].y);
                gl += vB[j].x * (Bl.x - Bpi.x) + vB[j].y * (Bl.y - Bpi.y);
                gl += vC[j].x * (Cl.x - Cpi.x) + vC[j].y * (Cl.y - Cpi.y);
            }
            const float yhat = group_sum<LANES>(yhp);
            const float obs = (ul - mu) * rsd;
            const float pred = (yhat - mu) * rsd;
            const float dv = obs - pred;
            if (ln == 0 && hv) gl += vu * (ul - upi) + vt * (tl - tpi);
            const float slope = sslp[i];  // row-uniform
            float gbar = sgg[i];
            if (slope != 0.f && !failed) {
                // warp partial -> every CTA's slot for (this CTA, this warp),
                // counted on that CTA's barrier; then wait for all CL*NW partials
                gl = warp_sum(gl);
                const int par = nred & 1;
                const uint32_t phase = (nred >> 1) & 1;
                if (tid == 0) mbar_expect_tx(&rbar[par], static_cast<uint32_t>(nslot) * 4u);
                if (lane < CL)  // addresses by select: a dynamic index would use local memory
                    st_async_f32(par ? rslot[1] : rslot[0], gl, par ? rbarr[1] : rbarr[0]);
                if (!mbar_wait_row(&rbar[par], phase)) failed = true;
                const float* sl = slots + par * 16 * 32;
                float tot = 0.f;
                for (int q = lane; q < nslot; q += 32) tot += sl[q];
                tot = warp_sum(tot);
                gbar += tot;
                ++nred;
            }
            const float xbar = gbar * slope;  // already divided by T
            const float rbar = sgr[i] + xbar;
            if (crank == 0 && tid == 0) geps -= xbar;
            const float4 rw = srow[i];  // 1/den, num/den^2, 1/num, 1/nobs
            const float numbar = rbar * rw.x;
            const float denbar = -rbar * rw.y;
            const float numtbar = sgn[i] * rw.x;
            const float dbar = numbar * dv * rw.z;
            const float obar = dbar + denbar * obs * rw.w;
            const float pbar = -dbar - numtbar * dv * rw.z;
            const float yhbar = pbar * rsd;
            float s_u_pi = 0.f, s_u_l = 0.f, s_dte = 0.f;
            float part[4 * NPT];  // (dBc.re, dBc.im, dCc.re, dCc.im) x chain, summed over channels below
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                const float2 Cl = sCl[i * NP + n], Bl = sBl[i * NP + n];
                const float2 Bpi = sBpi[i * NP + n], Cpi = sCpi[i * NP + n];
                const float2 ahc = make_float2(yb * Cl.x, -yb * Cl.y);
                // x_hat and h_upd adjoints
                float2 axh, ahu;
                if constexpr (G1) {
                    axh = make_float2(yhbar * Cpi.x, -yhbar * Cpi.y);
                    ahu = cadd(ahc, ah[j]);
                } else {
                    axh = make_float2((1.f - g) * ahc.x + yhbar * Cpi.x, (1.f - g) * ahc.y - yhbar * Cpi.y);
                    ahu = make_float2(g * (ahc.x + ah[j].x), g * (ahc.y + ah[j].y));
                }
                const float2 ahf = cadd(axh, ahu);
                s_u_pi += axh.x * qp[j].x + axh.y * qp[j].y;
                s_u_l += ahu.x * ql[j].x + ahu.y * ql[j].y;
                const float2 aqp = cscale(axh, upi), aql = cscale(ahu, ul);
                const float2 adB = cadd(cmul(aqp, make_float2(Bpi.x, -Bpi.y)),
                                        cmul(aql, make_float2(Bl.x, -Bl.y)));
                const float2 cdB = make_float2(dB[j].x, -dB[j].y);
                float2 outB, outC;
                if constexpr (G1) {
                    outB = cadd(vB[j], cmul(cdB, aql));
                    vB[j] = cmul(cdB, aqp);
                    outC = cadd(vC[j], make_float2(yb * hu[j].x, -yb * hu[j].y));
                } else {
                    const float2 hc = cadd(cscale(hu[j], g), cscale(xh[j], 1.f - g));
                    outB = cadd(cscale(vB[j], g), cmul(cdB, aql));
                    vB[j] = cadd(cscale(vB[j], 1.f - g), cmul(cdB, aqp));
                    outC = cadd(cscale(vC[j], g), make_float2(yb * hc.x, -yb * hc.y));
                }
                const float2 vCn = make_float2(yhbar * xh[j].x, -yhbar * xh[j].y);
                vC[j] = G1 ? vCn : cadd(cscale(vC[j], 1.f - g), vCn);
                // state adjoint for the previous step
                const float2 cdA = make_float2(dA[j].x, -dA[j].y);
                const float2 adA = cmul(make_float2(hp[j].x, -hp[j].y), ahf);
                ah[j] = G1 ? cmul(cdA, ahf) : cadd(cscale(ah[j], 1.f - g), cmul(cdA, ahf));
                // dB_bar = expm1(z) / lam: the adjoint of expm1(z) is adB conj(1/lam)
                // and lam's share through 1/lam is -adB conj(dB_bar / lam)
                const float2 aE = cmul(adB, make_float2(ilam[j].x, -ilam[j].y));
                float2 alm = cmul(make_float2(-aE.x, -aE.y), cdB);  // -adB conj(ilam) conj(dB_bar)
                const float2 az = cmul(cdA, cadd(adA, aE));
                alm = cadd(alm, cscale(az, dte));
                s_dte += az.x * lam[j].x + az.y * lam[j].y;
                if (nv[j]) glam[j] = cadd(glam[j], alm);
                part[j] = nv[j] ? outB.x : 0.f;
                part[NPT + j] = nv[j] ? outB.y : 0.f;
                part[2 * NPT + j] = nv[j] ? outC.x : 0.f;
                part[3 * NPT + j] = nv[j] ? outC.y : 0.f;
            }
            // per-(step, n) partials over this warp's channel groups: a
            // transposed butterfly leaves each lane kRem of the 4*NPT sums
            using FS = FoldShape<4 * NPT, 16, LANES>;
            Fold<4 * NPT, 16, LANES>::run(part, lane);
            if (FS::writer(lane)) {
                const int q0 = FS::held(lane);
#pragma unroll
                for (int r = 0; r < FS::kRem; ++r) {
                    const int q = q0 + r, c = q / NPT, n = ln + LANES * (q % NPT);
                    float* dst = reinterpret_cast<float*>(c < 2 ? soB : soC);
                    dst[((i * NW + wid) * NP + n) * 2 + (c & 1)] = part[r];
                }
            }
            s_u_pi = group_sum<LANES>(s_u_pi);
            s_u_l = group_sum<LANES>(s_u_l);
            s_dte = group_sum<LANES>(s_dte);
            float out_t = 0.f;
            if (hv) {
                const float dub = yb * Dh + obar * rsd + (G1 ? vu : g * vu) + s_u_l;
                vu = G1 ? s_u_pi : (1.f - g) * vu + s_u_pi;
                const float drb = mdt * s_dte;
                const float dlt = drb * scale;  // this channel's share of delta_bar
                glog += drb * delta * scale;
                gD += yb * ul;
                out_t = (G1 ? vt : g * vt) + mdel * dlt;
                vt = G1 ? -mdel * dlt : (1.f - g) * vt - mdel * dlt;
                if (ln == 0) a.du[(rowL + l) * H + h] = dub;
            }
            float ot = (ln == 0) ? out_t : 0.f;
            ot = warp_sum(ot);
            if (lane == 0) sot[i * NW + wid] = ot;
        };
        for (int i = steps - 1; i >= 0; --i) {
            if (sgt[i] == 1.f) reverse_step(std::true_type{}, i);
            else reverse_step(std::false_type{}, i);
        }
        // ---- chunk end: per-CTA partials of dBc, dCc, dt ----
        __syncthreads();
        for (int idx = tid; idx < steps * NP; idx += T) {
            const int i = idx / NP, n = idx % NP;
            if (n >= N) continue;
            float2 sb = make_float2(0.f, 0.f), sc = make_float2(0.f, 0.f);
            for (int w = 0; w < NW; ++w) {
                sb = cadd(sb, soB[(i * NW + w) * NP + n]);
                sc = cadd(sc, soC[(i * NW + w) * NP + n]);
            }
            const size_t o = ((static_cast<size_t>(b) * CL + crank) * L + l0 + i) * N + n;
            a.pB[o] = sb;
            a.pC[o] = sc;
        }
        for (int i = tid; i < steps; i += T) {
            float s = 0.f;
            for (int w = 0; w < NW; ++w) s += sot[i * NW + w];
            a.pt[(static_cast<size_t>(b) * CL + crank) * L + l0 + i] = s;
        }
    }
    // ---- initial state (t_0 - dt_init, u_0, B_0, C_0) ----
    __syncthreads();
    if (hv && ln == 0) a.du[rowL * H + h] += vu;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        float2 ob = nv[j] ? vB[j] : make_float2(0.f, 0.f);
        float2 oc = nv[j] ? vC[j] : make_float2(0.f, 0.f);
#pragma unroll
        for (int o = LANES; o < 32; o <<= 1) {
            ob.x += __shfl_xor_sync(0xffffffffu, ob.x, o);
            ob.y += __shfl_xor_sync(0xffffffffu, ob.y, o);
            oc.x += __shfl_xor_sync(0xffffffffu, oc.x, o);
            oc.y += __shfl_xor_sync(0xffffffffu, oc.y, o);
        }
        if (lane < LANES) {
            soB[wid * NP + n] = ob;
            soC[wid * NP + n] = oc;
        }
    }
    float ot = (hv && ln == 0) ? vt : 0.f;
    ot = warp_sum(ot);
    if (lane == 0) sot[wid] = ot;
    __syncthreads();
    for (int n = tid; n < N; n += T) {
        float2 sb = make_float2(0.f, 0.f), sc = make_float2(0.f, 0.f);
        for (int w = 0; w < NW; ++w) {
            sb = cadd(sb, soB[w * NP + n]);
            sc = cadd(sc, soC[w * NP + n]);
        }
        const size_t o = ((static_cast<size_t>(b) * CL + crank) * L) * N + n;
        a.pB[o] = cadd(a.pB[o], sb);
        a.pC[o] = cadd(a.pC[o], sc);
    }
    if (tid == 0) {
        float s = 0.f;
        for (int w = 0; w < NW; ++w) s += sot[w];
        a.pt[(static_cast<size_t>(b) * CL + crank) * L] += s;
    }
    // ---- per-row parameter partials ----
#pragma unroll
    for (int j = 0; j < NPT; ++j)
        if (nv[j]) a.plam[(static_cast<size_t>(b) * H + h) * N + ln + LANES * j] = glam[j];
    if (hv && ln == 0) {
        a.plog[static_cast<size_t>(b) * H + h] = glog;
        a.pD[static_cast<size_t>(b) * H + h] = gD;
    }
    if (crank == 0 && tid == 0) a.peps[b] = geps;
    cluster_sync_all();  // no CTA leaves while a peer may still write its slots
}

// ---------------------------------------------------------------------------
// post pass: sum per-CTA and per-row partials
// ---------------------------------------------------------------------------
__global__ void train_post_rows(TArgs a) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t BLN = static_cast<int64_t>(a.B) * a.L * a.N;
    if (idx < BLN) {
        const int64_t b = idx / (static_cast<int64_t>(a.L) * a.N);
        const int64_t ln = idx % (static_cast<int64_t>(a.L) * a.N);
        float2 sb = make_float2(0.f, 0.f), sc = make_float2(0.f, 0.f);
        for (int c = 0; c < a.CL; ++c) {
            const size_t o = (static_cast<size_t>(b) * a.CL + c) * a.L * a.N + ln;
            sb = cadd(sb, a.pB[o]);
            sc = cadd(sc, a.pC[o]);
        }
        a.dBc[idx] = sb;
        a.dCc[idx] = sc;
    }
    const int64_t BL = static_cast<int64_t>(a.B) * a.L;
    if (idx < BL) {
        const int64_t b = idx / a.L, l = idx % a.L;
        float s = 0.f;
        for (int c = 0; c < a.CL; ++c) s += a.pt[(static_cast<size_t>(b) * a.CL + c) * a.L + l];
        a.dt[idx] = s;
    }
}

__global__ void train_post_params(TArgs a) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t HN = static_cast<int64_t>(a.H) * a.N;
    if (idx < HN) {
        float2 s = make_float2(0.f, 0.f);
        for (int b = 0; b < a.B; ++b) s = cadd(s, a.plam[static_cast<size_t>(b) * HN + idx]);
        a.dlam[idx] = s;
    }
    if (idx < a.H) {
        float s1 = 0.f, s2 = 0.f;
        for (int b = 0; b < a.B; ++b) {
            s1 += a.plog[static_cast<size_t>(b) * a.H + idx];
            s2 += a.pD[static_cast<size_t>(b) * a.H + idx];
        }
        a.dlog[idx] = s1;
        a.dD[idx] = s2;
    }
    if (idx == 0) {
        float s = 0.f;
        for (int b = 0; b < a.B; ++b) s += a.peps[b];
        a.deps[0] = s;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
#ifndef EACS_TRAIN_NPT
#define EACS_TRAIN_NPT 4
#endif
int lanes_train(int N, int* lanes, int* npt) {
    if (EACS_TRAIN_NPT == 4 && N > 8) {
        // four chains a thread: half the threads per channel, so a row fits
        // in a cluster of 8 CTAs and a batch of rows runs in one wave
        if (N <= 16) { *lanes = 4; *npt = 4; }
        else if (N <= 32) { *lanes = 8; *npt = 4; }
        else if (N <= 64) { *lanes = 16; *npt = 4; }
        else return 0;
        return 1;
    }
    if (N <= 8) { *lanes = 4; *npt = 2; }
    else if (N <= 16) { *lanes = 8; *npt = 2; }
    else if (N <= 32) { *lanes = 16; *npt = 2; }
    else if (N <= 64) { *lanes = 32; *npt = 2; }
    else return 0;
    return 1;
}

// Cluster size and channels per CTA: the smallest power-of-two cluster (up to
// 16) whose CTAs hold at most 512 threads (train_bwd needs ~118 registers a
// thread, so 512 threads is the most one SM can hold).  With at most
// kFewRows rows (data-parallel training with one or a few videos per GPU) the
// rows use 16-CTA clusters: the GPU has room for them, and a row's per-step
// work is spread over twice the SMs.
#ifndef EACS_TRAIN_FEW_ROWS
#define EACS_TRAIN_FEW_ROWS 4
#endif
constexpr int kFewRows = EACS_TRAIN_FEW_ROWS;
bool train_shape(int64_t H, int lanes, int64_t B, int* CL, int* HC, int* T) {
    const int first = B <= kFewRows ? 16 : 1;
    for (int cl = first; cl <= 16; cl *= 2) {
        const int64_t hc = (H + cl - 1) / cl;
        const int64_t t = ((hc * lanes + 31) / 32) * 32;
        if (t <= 512) {
            *CL = cl;
            *HC = static_cast<int>(hc);
            *T = static_cast<int>(t);
            return true;
        }
    }
    return false;
}

size_t smem_bytes(int T, int NPT, int NP, int HC, int kK, bool commits) {
    const int NW = T / 32;
    size_t s = 0;
    s += sizeof(float2) * kK * T * NPT * 3;   // h_pi, dA, dB_bar
    s += sizeof(float2) * kK * NP * 4;        // B_pi, C_pi, B_l, C_l
    s += sizeof(float2) * kK * NW * NP * 2;   // dBc, dCc partials
    s += sizeof(float4) * kK + 16;            // row constants, 2 mbarriers
    s += sizeof(float) * 2 * 16 * 32;         // reduction slots
    s += sizeof(float) * (kK * HC * 3 + kK * 7 + kK * NW);
    if (commits) {                            // commit adjoints: u_pi, t_pi, B_pi, C_pi, h_pi ring
        s += sizeof(float) * (kK * HC + kK + 1);
        s += sizeof(float2) * (kK * NP * 2 + 2 * NPT * T);
    }
    return s;
}

size_t al(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Chunk length: the largest power of two up to kKMax whose shared-memory
// footprint fits in 200 KiB.
int chunk_len(int T, int NPT, int NP, int HC, bool commits) {
    for (int k = kKMax; k >= 1; k /= 2)
        if (smem_bytes(T, NPT, NP, HC, k, commits) <= 200u * 1024u) return k;
    return 0;
}

struct TWs {
    size_t ck_h, ck_u, ck_row, ck_bc, pB, pC, pt, plam, plog, pD, peps, total;
};
TWs tws(int64_t B, int64_t L, int64_t H, int64_t N, int CL, int kK) {
    TWs w{};
    const int64_t nK = (L + kK - 1) / kK;
    size_t o = 0;
    w.ck_h = o; o += al(sizeof(float2) * B * nK * H * N);
    w.ck_u = o; o += al(sizeof(float) * B * nK * H);
    w.ck_row = o; o += al(sizeof(float4) * B * nK);
    w.ck_bc = o; o += al(sizeof(float2) * B * nK * 2 * N);
    w.pB = o; o += al(sizeof(float2) * B * CL * L * N);
    w.pC = o; o += al(sizeof(float2) * B * CL * L * N);
    w.pt = o; o += al(sizeof(float) * B * CL * L);
    w.plam = o; o += al(sizeof(float2) * B * H * N);
    w.plog = o; o += al(sizeof(float) * B * H);
    w.pD = o; o += al(sizeof(float) * B * H);
    w.peps = o; o += al(sizeof(float) * B);
    w.total = o;
    return w;
}

// The checkpoint pass is an independent chain per (h, n): it keeps two
// chains a thread (the most threads per row) whatever the backward's layout.
template <typename UT>
cudaError_t launch_ckpt(TArgs& a, cudaStream_t s) {
    const int N = a.N;
    const int lanes = N <= 8 ? 4 : N <= 16 ? 8 : N <= 32 ? 16 : 32;
    const dim3 grid((a.H + kCkThreads / lanes - 1) / (kCkThreads / lanes), a.B);
    if (lanes == 4) train_ckpt<4, 2, UT><<<grid, kCkThreads, 0, s>>>(a);
    else if (lanes == 8) train_ckpt<8, 2, UT><<<grid, kCkThreads, 0, s>>>(a);
    else if (lanes == 16) train_ckpt<16, 2, UT><<<grid, kCkThreads, 0, s>>>(a);
    else train_ckpt<32, 2, UT><<<grid, kCkThreads, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
}

template <int LANES, int NPT, typename UT, bool CG>
cudaError_t launch_train(TArgs& a, int T, cudaStream_t s) {
    constexpr int NP = LANES * NPT;
    if (!a.have_ckpt) {
        cudaError_t e = launch_ckpt<UT>(a, s);
        if (e != cudaSuccess) return e;
    }
    const size_t smem = smem_bytes(T, NPT, NP, a.HC, a.K, a.commit_grads != 0);
    // CTAs of at most 384 threads (config 3: 96 channels x 4 lanes) may use up to
    // 168 registers a thread; the 512-thread bound (128) made the kernel spill
    auto kern = T <= 384 ? train_bwd<LANES, NPT, UT, 384, CG> : train_bwd<LANES, NPT, UT, 512, CG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    if (a.CL > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.CL, a.B);
    cfg.blockDim = dim3(T);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    mark_start(s);
    e = cudaLaunchKernelEx(&cfg, kern, a);
    mark_stop(s);
    note_launch();
    if (e != cudaSuccess) return e;
    const int64_t n1 = std::max<int64_t>(static_cast<int64_t>(a.B) * a.L * a.N, static_cast<int64_t>(a.B) * a.L);
    train_post_rows<<<static_cast<unsigned>((n1 + 255) / 256), 256, 0, s>>>(a);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int64_t n2 = std::max<int64_t>(static_cast<int64_t>(a.H) * a.N, 1);
    train_post_params<<<static_cast<unsigned>((n2 + 255) / 256), 256, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
}

// the (lanes, chains a thread) pairs lanes_train can return, and no others
template <typename UT, bool CG>
cudaError_t train_by_n(TArgs& a, int T, cudaStream_t s) {
    int lanes, npt;
    lanes_train(a.N, &lanes, &npt);
#if EACS_TRAIN_NPT == 4
    if (npt == 4) {
        if (lanes == 4) return launch_train<4, 4, UT, CG>(a, T, s);
        if (lanes == 8) return launch_train<8, 4, UT, CG>(a, T, s);
        return launch_train<16, 4, UT, CG>(a, T, s);
    }
    return launch_train<4, 2, UT, CG>(a, T, s);
#else
    if (lanes == 4) return launch_train<4, 2, UT, CG>(a, T, s);
    if (lanes == 8) return launch_train<8, 2, UT, CG>(a, T, s);
    if (lanes == 16) return launch_train<16, 2, UT, CG>(a, T, s);
    return launch_train<32, 2, UT, CG>(a, T, s);
#endif
}

template <typename UT>
cudaError_t train_by_n(TArgs& a, int T, cudaStream_t s) {
    return a.commit_grads ? train_by_n<UT, true>(a, T, s) : train_by_n<UT, false>(a, T, s);
}

// Shapes of the backward for (B, L, H, N): lanes and chains a thread, cluster
// size, channels a CTA, threads a CTA and the checkpoint interval (which the
// commit-adjoint variant may shorten: its extra shared memory counts).
struct Layout {
    int lanes, npt, CL, HC, T, K;
};
// With fn null nothing is reported, only the status returned.
int train_layout(int64_t B, int64_t L, int64_t H, int64_t N, bool commits, const char* fn, Layout* o) {
#define EACS_LAYOUT_FAIL(code, ...) return fn ? fail(code, __VA_ARGS__) : (code)
    if (B < 0 || L < 0 || H < 0 || N < 0) EACS_LAYOUT_FAIL(EACS_ERR_INVALID, "%s: negative size", fn);
    if (N <= 0 || !lanes_train(static_cast<int>(N), &o->lanes, &o->npt))
        EACS_LAYOUT_FAIL(EACS_ERR_UNSUPPORTED, "%s: N=%lld outside 1..64", fn, (long long)N);
    if (H <= 0 || !train_shape(H, o->lanes, B, &o->CL, &o->HC, &o->T))
        EACS_LAYOUT_FAIL(EACS_ERR_UNSUPPORTED, "%s: H=%lld needs more than 16 CTAs of 512 threads per row", fn,
                         (long long)H);
    if (B > 65535 || L > (1LL << 30)) EACS_LAYOUT_FAIL(EACS_ERR_UNSUPPORTED, "%s: B or L too large", fn);
    o->K = chunk_len(o->T, o->npt, o->lanes * o->npt, o->HC, commits);
    if (o->K == 0)
        EACS_LAYOUT_FAIL(EACS_ERR_UNSUPPORTED, "%s: shared memory too small for H=%lld", fn, (long long)H);
#undef EACS_LAYOUT_FAIL
    return EACS_OK;
}

size_t layout_bytes(int64_t B, int64_t L, int64_t H, int64_t N, bool commits) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0) return 0;
    Layout o{};
    if (train_layout(B, L, H, N, commits, nullptr, &o) != EACS_OK) return 0;
    return tws(B, L, H, N, o.CL, o.K).total;
}

// Fills the fields of `a` every pass shares: inputs, workspace, sizes.
void fill_common(TArgs& a, const TrainBwdCall& c, const Layout& o, const TWs& w) {
    a.lam = static_cast<const float2*>(c.lam);
    a.log_dt = c.log_dt;
    a.u = c.u;
    a.Bc = static_cast<const float2*>(c.Bc);
    a.Cc = static_cast<const float2*>(c.Cc);
    a.t = c.t;
    a.D = c.D;
    a.mean = c.mean;
    a.var = c.var;
    a.eps = c.eps;
    a.eta = c.eta;
    a.var_eps = c.var_eps;
    a.dt_init = c.dt_init;
    a.dt_min = c.dt_min;
    a.dt_max = c.dt_max;
    a.Tp = c.temperature > 1e-4f ? c.temperature : 1e-4f;
    a.gates = c.gates;
    char* ws = static_cast<char*>(c.workspace);
    a.ck_h = reinterpret_cast<float2*>(ws + w.ck_h);
    a.ck_u = reinterpret_cast<float*>(ws + w.ck_u);
    a.ck_row = reinterpret_cast<float4*>(ws + w.ck_row);
    a.ck_bc = reinterpret_cast<float2*>(ws + w.ck_bc);
    a.pB = reinterpret_cast<float2*>(ws + w.pB);
    a.pC = reinterpret_cast<float2*>(ws + w.pC);
    a.pt = reinterpret_cast<float*>(ws + w.pt);
    a.plam = reinterpret_cast<float2*>(ws + w.plam);
    a.plog = reinterpret_cast<float*>(ws + w.plog);
    a.pD = reinterpret_cast<float*>(ws + w.pD);
    a.peps = reinterpret_cast<float*>(ws + w.peps);
    a.B = static_cast<int>(c.B);
    a.L = static_cast<int>(c.L);
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    a.K = o.K;
    a.nK = static_cast<int>((c.L + o.K - 1) / o.K);
    a.CL = o.CL;
    a.HC = o.HC;
    a.Klog = 0;
    while ((1 << a.Klog) < a.K) ++a.Klog;
}

}  // namespace

size_t train_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return layout_bytes(B, L, H, N, false);
}

size_t train_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return layout_bytes(B, L, H, N, true);
}

int train_ckpt_layout(int64_t B, int64_t L, int64_t H, int64_t N, void* workspace, size_t workspace_bytes,
                      CellCall* c) {
    const char* fn = "eacs_cell_train_fwd_ckpt";
    Layout o{};
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0)
        return fail(EACS_ERR_UNSUPPORTED, "%s: no training backward for B=%lld L=%lld H=%lld N=%lld", fn,
                    (long long)B, (long long)L, (long long)H, (long long)N);
    const int rc = train_layout(B, L, H, N, false, fn, &o);
    if (rc) return rc;
    const TWs w = tws(B, L, H, N, o.CL, o.K);
    if (!workspace || workspace_bytes < w.total)
        return fail(EACS_ERR_WORKSPACE, "%s: backward workspace of %zu bytes needed, %zu given", fn, w.total,
                    workspace_bytes);
    char* ws = static_cast<char*>(workspace);
    c->ck_h = ws + w.ck_h;
    c->ck_u = reinterpret_cast<float*>(ws + w.ck_u);
    c->ck_row = ws + w.ck_row;
    c->ck_bc = ws + w.ck_bc;
    c->ck_K = o.K;
    c->ck_nK = static_cast<int>((L + o.K - 1) / o.K);
    return EACS_OK;
}

int train_commits_replay(const TrainBwdCall& c, const CommitOut& out, cudaStream_t stream) {
    const char* fn = "eacs_cell_train_commits_fwd";
    if (c.B == 0 || c.L == 0 || c.H == 0) return EACS_OK;
    Layout o{};
    const int rc = train_layout(c.B, c.L, c.H, c.N, true, fn, &o);
    if (rc) return rc;
    if (c.u_dtype != EACS_DTYPE_F32 && c.u_dtype != EACS_DTYPE_F16 && c.u_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, c.u_dtype);
    if (!c.lam || !c.log_dt || !c.u || !c.Bc || !c.Cc || !c.t || !c.gates || !out.h || !out.t || !out.u ||
        !out.B || !out.C)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    const TWs w = tws(c.B, c.L, c.H, c.N, o.CL, o.K);
    if (!c.workspace || c.workspace_bytes < w.total)
        return fail(EACS_ERR_WORKSPACE, "%s: backward workspace of %zu bytes needed, %zu given", fn, w.total,
                    c.workspace_bytes);
    TArgs a{};
    fill_common(a, c, o, w);
    a.cm_h = static_cast<float2*>(out.h);
    a.cm_t = out.t;
    a.cm_u = out.u;
    a.cm_B = static_cast<float2*>(out.B);
    a.cm_C = static_cast<float2*>(out.C);
    cudaError_t e;
    if (c.u_dtype == EACS_DTYPE_F16) e = launch_ckpt<__half>(a, stream);
    else if (c.u_dtype == EACS_DTYPE_BF16) e = launch_ckpt<__nv_bfloat16>(a, stream);
    else e = launch_ckpt<float>(a, stream);
    return cuda_check(e, fn);
}

int train_bwd(const TrainBwdCall& c, cudaStream_t stream) {
    const char* fn = c.commits ? "eacs_cell_train_commits_bwd"
                   : c.have_ckpt ? "eacs_cell_train_bwd_ckpt" : "eacs_cell_train_bwd";
    if (c.B < 0 || c.L < 0 || c.H < 0 || c.N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.B == 0 || c.L == 0 || c.H == 0) return EACS_OK;
    Layout o{};
    const int rc = train_layout(c.B, c.L, c.H, c.N, c.commits, fn, &o);
    if (rc) return rc;
    if (c.u_dtype != EACS_DTYPE_F32 && c.u_dtype != EACS_DTYPE_F16 && c.u_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, c.u_dtype);
    if (!c.lam || !c.log_dt || !c.u || !c.Bc || !c.Cc || !c.t || !c.D || !c.mean || !c.var || !c.gates ||
        !c.resid || !c.stats || !c.gy || !c.du || !c.dBc || !c.dCc || !c.dt || !c.dlam || !c.dlog ||
        !c.dD || !c.deps)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    const TWs w = tws(c.B, c.L, c.H, c.N, o.CL, o.K);
    if (!c.workspace || c.workspace_bytes < w.total)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, w.total,
                    c.workspace_bytes);
    TArgs a{};
    fill_common(a, c, o, w);
    a.resid = c.resid;
    a.stats = static_cast<const float2*>(c.stats);
    a.gy = c.gy;
    a.ggs = c.ggs;
    a.grs = c.grs;
    a.gns = c.gns;
    a.du = c.du;
    a.dBc = static_cast<float2*>(c.dBc);
    a.dCc = static_cast<float2*>(c.dCc);
    a.dt = c.dt;
    a.dlam = static_cast<float2*>(c.dlam);
    a.dlog = c.dlog;
    a.dD = c.dD;
    a.deps = c.deps;
    a.have_ckpt = (c.have_ckpt || c.commits) ? 1 : 0;
    a.commit_grads = c.commits ? 1 : 0;
    a.gate_const = c.gate_const ? 1 : 0;
    a.gc_h = static_cast<const float2*>(c.gc_h);
    a.gc_t = c.gc_t;
    a.gc_u = c.gc_u;
    a.gc_B = static_cast<const float2*>(c.gc_B);
    a.gc_C = static_cast<const float2*>(c.gc_C);
    cudaError_t e;
    if (c.u_dtype == EACS_DTYPE_F16) e = train_by_n<__half>(a, o.T, stream);
    else if (c.u_dtype == EACS_DTYPE_BF16) e = train_by_n<__nv_bfloat16>(a, o.T, stream);
    else e = train_by_n<float>(a, o.T, stream);
    return cuda_check(e, fn);
}

cudaError_t train_read_status(int* out, cudaStream_t stream) { return read_clear_status(out, stream); }

}  // namespace eacs
