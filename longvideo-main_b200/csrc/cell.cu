// cell.cu -- gated EACS cell and fused ungated continuous SSM (sm_100a).
//
// Semantics: cst_ssm/modules/eacs.py:78-173 (eacs_step / scan_range with
// robust_guard), cst_ssm/ops/csrc/eacs_cell_cuda.cu:36-168 (the inference
// kernel this replaces), cst_ssm/ops/eacs_cell_train.py:15-66 (soft gate) and
// cst_ssm/modules/continuous_ssm.py:44-55 (ungated layer core).
//
// Gated forward = speculate, verify, repair:
//  1. cell_chain<SPEC>: assume every frame commits.  Then t_pi = t_{l-1},
//     u_pi = u_{l-1}, B_pi = B_{l-1}, C_pi = C_{l-1}, h_pi = h_{l-1} and the
//     gated cell is a linear recurrence, run with one thread per (h, n) chain
//     (state in registers, all of L, no (B,L,H,N) tensor anywhere).  Each step
//     also forms the prediction x_hat, y_hat and the residual partial sums
//     sum_h ((u-mu)/s - (y_hat-mu)/s)^2, sum_h ((u-mu)/s)^2 per h-tile.
//  2. cell_resid: r_l per (b, l) from the partials (fixed summation order).
//  3. cell_gates: per row, the robust_guard spike counter as a max-scan,
//     gates g_l = r_l > eps_l and the first skipped step l*.  Everything
//     before l* is exact; rows with no skip are done.
//  4. cell_chain<REPLAY>: for rows with a skip, the committed state h_{l*-1}.
//  5. cell_repair: for those rows, the exact sequential gated cell from l*
//     (one CTA per row, one block reduction per step).
// Frames with every step committing (update rate 1.0, the common case on
// N(0,1) features) cost one pass of step 1.
#include <algorithm>
#include <mutex>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

#ifndef EACS_CHAIN_THREADS
#define EACS_CHAIN_THREADS 128
#endif
#ifndef EACS_CHAIN_U
#define EACS_CHAIN_U 8
#endif
constexpr int kThreads = EACS_CHAIN_THREADS;  // chain kernel CTA
constexpr int kMinBlocks = 768 / kThreads;    // keep 24 warps per SM resident
// Wide speculative pass: one CTA of 11 warps per SM.  Four-warp CTAs leave
// SMs unevenly loaded when a launch is a little over two CTAs per SM (B=8,
// H=768: 384 CTAs on 148 SMs, so 88 SMs run 12 warps and 60 run 8); with
// 44-channel tiles the same rows are 144 CTAs, every SM runs at most 11 warps.
constexpr int kWideThreads = 352;
constexpr int kT = 32;                         // steps per staged chunk
constexpr int kRepair = 1024;  // repair kernel CTA

// SPEC_COMMITS: SPEC + commit_h; SPEC_CKPT: SPEC + the training backward's checkpoints
enum Mode { SPEC = 0, UNGATED = 1, REPLAY = 2, SPEC_COMMITS = 3, SPEC_CKPT = 4 };

struct Args {
    const float2* lam;
    const float* log_dt;
    const void* u;
    const float2* Bc;
    const float2* Cc;
    const float* t;
    const float* D;
    const float* mean;
    const float* var;
    float eps, eta, var_eps, dt_init, dt_min, dt_max;
    int robust, robust_k;
    float spike_ratio, eps_lo;
    int gate_mode;
    float Tp;
    float* y;
    float* gate;
    float* resid;
    float2* stats; // [B][L] (||obs - pred||, ||obs||) when non-null (training forward)
    float2* part;  // [B][ntiles][L] (sum d^2, sum obs^2)
    int4* row;     // [B] {l*, bits(spike after l*-1), bits(r_{l*-1}), 0}
    float2* hpi;   // [B][H][N] committed state for the repair pass
    float* upi;    // [B][H]
    float2* ck;    // UNGATED, optional: [B][nK][H][N] state before step k*kSsmCk
    // optional per-frame commits (hard gate): committed state after each step
    float2* commit_h;  // (B,L,H,N)
    float* commit_t;   // (B,L)
    float* commit_u;   // (B,L,H)
    float2* commit_B;  // (B,L,N)
    float2* commit_C;
    int* cidx;         // [B][L] last committed step <= l (-1: the initial state)
    // optional row state carried between time chunks (gated modes): the
    // committed state before this call's first step and after its last one
    const float2* cin_h;   // (B,H,N)
    const float* cin_u;    // (B,H)
    const float2* cin_B;   // (B,N)
    const float2* cin_C;
    const float4* cin_row; // (B) t_pi, spike count, r of the previous step, -
    float2* cout_h;
    float* cout_u;
    float2* cout_B;
    float2* cout_C;
    float4* cout_row;
    // optional training checkpoints (hard or soft gate): the committed state
    // before every gK-th step, in the training backward's layout
    float2* gck_h;   // [B][gnK][H][N]
    float* gck_u;    // [B][gnK][H]
    float4* gck_row; // [B][gnK] (t_pi, -, -, -)
    float2* gck_bc;  // [B][gnK][2][N] (B_pi, C_pi)
    int gK, gnK, gKlog;  // gK = 1 << gKlog
    int B, L, H, N, ntiles, nK;
    int wide;     // SPEC: 44-channel tiles of kWideThreads threads (wide_tiles)
    int chains4;  // SPEC: four chains a thread, 32-channel tiles (side_by_side_tiles)
};

// Checkpoint k = l / gK of row b from a thread owning chains n = ln + LANES*j
// of channel h: its states, its channel's u_pi; B_pi / C_pi and t_pi by the
// threads the caller names (one per row for t_pi, one channel's for B, C).
template <int LANES, int NPT>
__device__ __forceinline__ void write_gck(const Args& a, int b, int k, int h, int ln, const bool (&nv)[NPT],
                                          const float2 (&hs)[NPT], bool chan_writer, float u_pi, bool bc_writer,
                                          const float2 (&Bp)[NPT], const float2 (&Cp)[NPT], bool row_writer,
                                          float t_pi) {
    const size_t rk = static_cast<size_t>(b) * a.gnK + k;
#pragma unroll
    for (int j = 0; j < NPT; ++j)
        if (nv[j]) a.gck_h[(rk * a.H + h) * a.N + ln + LANES * j] = hs[j];
    if (chan_writer) a.gck_u[rk * a.H + h] = u_pi;
    if (bc_writer) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (n < a.N) {
                a.gck_bc[rk * 2 * a.N + n] = Bp[j];
                a.gck_bc[(rk * 2 + 1) * a.N + n] = Cp[j];
            }
        }
    }
    if (row_writer) a.gck_row[rk] = make_float4(t_pi, 0.f, 0.f, 0.f);
}

// ---------------------------------------------------------------------------
// Transposed shuffle butterfly over the LANES lanes of a channel group.  A lane
// enters with V partial sums; at each of the first log2(min(V, LANES)) levels
// it keeps half of its values and trades the other half with its partner, so V
// sums cost V-1 shuffles instead of V*log2(LANES).  Afterwards lane ln holds
// the full sums of original indices held_index(ln) .. + V_REM-1; lanes that
// differ only in the bits of the plain levels hold the same sums.
// ---------------------------------------------------------------------------
template <int V, int O>
struct Bfly {
    static __device__ __forceinline__ void run(float* v, int ln) {
        if constexpr (O == 0) {
            return;
        } else if constexpr (V == 1) {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
            Bfly<1, O / 2>::run(v, ln);
        } else {
            const bool up = (ln & O) != 0;
#pragma unroll
            for (int k = 0; k < V / 2; ++k) {
                const float send = up ? v[k] : v[k + V / 2];
                const float keep = up ? v[k + V / 2] : v[k];
                v[k] = keep + __shfl_xor_sync(0xffffffffu, send, O);
            }
            Bfly<V / 2, O / 2>::run(v, ln);
        }
    }
};

template <int V, int LANES>
struct BflyShape {
    static constexpr int levels(int v, int o) { return (o == 0 || v == 1) ? 0 : 1 + levels(v / 2, o / 2); }
    static constexpr int kHalve = levels(V, LANES / 2);
    static constexpr int kRem = V >> kHalve;                  // sums held per lane
    static constexpr int kPlainMask = (LANES >> kHalve) - 1;  // bits of the plain levels
    static __device__ __forceinline__ int held_index(int ln) {
        int idx = 0;
#pragma unroll
        for (int j = 0; j < kHalve; ++j)
            if (ln & (LANES >> (j + 1))) idx += V >> (j + 1);
        return idx;
    }
};

// ---------------------------------------------------------------------------
// 1 / 4: chain kernel.  Thread (hl, ln) of a CTA owns chains n = ln + LANES*j
// (j < NPT) of channel h = tile*HT + hl.  Steps run in groups of U: the U
// discretisations are independent (the state enters only through two complex
// FMAs per step), and the 2U readout sums of a group (y and y_hat) share one
// transposed butterfly, after which the per-channel residual work of the U
// steps is spread over the group's lanes instead of repeated by every lane.
// ---------------------------------------------------------------------------
template <int LANES, int NPT, int MODE, typename UT, int CT = kThreads>
__global__ void __launch_bounds__(CT, (CT != kThreads ? 1 : NPT == 1 ? kMinBlocks : kMinBlocks * 2 / 3))
    cell_chain(Args a) {
    constexpr int HT = CT / LANES;
    constexpr int NP = LANES * NPT;
    constexpr int NW = CT / 32;
    constexpr int U = EACS_CHAIN_U;
    constexpr bool kSpec = MODE == SPEC || MODE == SPEC_COMMITS || MODE == SPEC_CKPT;  // speculative gated pass
    constexpr int NV = kSpec ? 2 * U : U;  // readout sums per group
    using Shape = BflyShape<NV, LANES>;
    static_assert(kT % U == 0, "chunk must hold whole step groups");
    static_assert(kT % kSsmCk == 0 && kSsmCk % U == 0, "checkpoints fall on step-group starts");
    // chunk inputs, double-buffered: chunk c+1 is copied in (cp.async) while
    // chunk c runs
    constexpr int NBUF = NP <= 32 ? 2 : 1;  // N > 32: one buffer (48 KB of static shared memory)
    // (B, C) of a step and chain side by side: one 16-byte load per chain
    __shared__ float4 sBC[NBUF][kT][NP];
    __shared__ __align__(16) UT su[NBUF][kT][HT];
    __shared__ float st[NBUF][kT];
    // readouts and residual partials of a chunk, written out after the next
    // chunk's first barrier (one barrier per chunk), so double-buffered
    __shared__ float sy[2][kT][HT];
    __shared__ float2 sred[2][kT][NW];

    const int tid = threadIdx.x;
    const int ln = tid % LANES;
    const int hl = tid / LANES;
    const int tile = blockIdx.x;
    const int b = blockIdx.y;
    const int h0 = tile * HT;
    const int h = h0 + hl;
    const bool hv = h < a.H;
    const int L = a.L, H = a.H, N = a.N;

    int lstop = L;
    if (MODE == REPLAY) {
        lstop = a.row[b].x;
        if (lstop >= L) return;  // row verified: nothing to repair
    }

    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowLH = static_cast<size_t>(b) * L;

    // Wp: B_pi u_pi / lam, the input term of the prediction (gated passes)
    float2 lam[NPT], ilam[NPT], hs[NPT], Bp[NPT], Cp[NPT], Wp[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        hs[j] = make_float2(0.f, 0.f);
        Wp[j] = make_float2(0.f, 0.f);
        Bp[j] = nv[j] ? a.Bc[rowLH * N + n] : make_float2(0.f, 0.f);
        Cp[j] = nv[j] ? a.Cc[rowLH * N + n] : make_float2(0.f, 0.f);
        if (MODE != UNGATED && a.cin_h != nullptr && nv[j]) {  // resumed row
            hs[j] = a.cin_h[(static_cast<size_t>(b) * H + h) * N + n];
            Bp[j] = a.cin_B[static_cast<size_t>(b) * N + n];
            Cp[j] = a.cin_C[static_cast<size_t>(b) * N + n];
        }
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    // 1/sqrt(var + var_eps): the residual standardises with a multiply
    // (within one rounding of the reference's division)
    const float rsd = hv ? 1.0f / sqrtf(a.var[h] + a.var_eps) : 1.f;
    const float mu = hv ? a.mean[h] : 0.f;
    const float Dh = hv ? a.D[h] : 0.f;
    float u_prev = hv ? to_f32(u[rowLH * H + h]) : 0.f;
    const float t0 = a.t[rowLH];
    float t_prev = t0 - a.dt_init;
    if (MODE != UNGATED && a.cin_h != nullptr) {
        if (hv) u_prev = a.cin_u[static_cast<size_t>(b) * H + h];
        t_prev = a.cin_row[b].x;
    }
    if (kSpec) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) Wp[j] = cscale(cmul(Bp[j], ilam[j]), u_prev);
    }
    float dt0 = 0.f;  // ungated: dt_0 = dt_1 (continuous_ssm.py:45-48)
    if (MODE == UNGATED && L > 1) dt0 = fmaxf(a.t[rowLH + 1] - t0, 0.f);
    const int held = Shape::held_index(ln);
    const bool writer = (ln & Shape::kPlainMask) == 0;

    // Stage chunk [c0, c0 + kT) into buffer `buf`.  Padded chains (n >= N)
    // and channels past H read zeros: with lam = -1 and B = C = 0 their
    // state stays 0 and they add exact zeros, without a branch.  The
    // asynchronous form copies u in 4-byte units (pairs of 16-bit values),
    // so it needs H even for half / bfloat16 u.
    constexpr int PAIR = sizeof(UT) == 4 ? 1 : 2;
    const bool async_ok = NBUF == 2 && (PAIR == 1 || (H % 2) == 0) && (reinterpret_cast<uintptr_t>(u) & 3u) == 0 &&
                          ((reinterpret_cast<uintptr_t>(a.Bc) | reinterpret_cast<uintptr_t>(a.Cc)) & 7u) == 0 &&
                          (reinterpret_cast<uintptr_t>(a.t) & 3u) == 0;
    auto stage = [&](int c0, int buf, bool async) {
        const int sn = min(kT, lstop - c0);
        for (int idx = tid; idx < sn * NP; idx += CT) {
            const int i = idx / NP, n = idx % NP;  // NP is a power of two
            const size_t o = (rowLH + c0 + i) * N + n;
            float2* d = reinterpret_cast<float2*>(&sBC[buf][i][n]);
            if (async) {
                cp_async8(d, n < N ? a.Bc + o : a.Bc, n < N);
                cp_async8(d + 1, n < N ? a.Cc + o : a.Cc, n < N);
            } else {
                d[0] = n < N ? a.Bc[o] : make_float2(0.f, 0.f);
                d[1] = n < N ? a.Cc[o] : make_float2(0.f, 0.f);
            }
        }
        if (async) {
            for (int idx = tid; idx < sn * (HT / PAIR); idx += CT) {
                const int i = idx / (HT / PAIR), k = (idx % (HT / PAIR)) * PAIR;
                const bool ok = h0 + k < H;  // a pair is both in or both past H (H, h0 even)
                cp_async4(&su[buf][i][k], ok ? u + (rowLH + c0 + i) * H + h0 + k : u, ok);
            }
            for (int i = tid; i < sn; i += CT) cp_async4(&st[buf][i], a.t + rowLH + c0 + i, true);
            cp_async_commit();
        } else {
            for (int idx = tid; idx < sn * HT; idx += CT) {
                const int i = idx / HT, k = idx % HT;
                su[buf][i][k] = (h0 + k < H) ? u[(rowLH + c0 + i) * H + h0 + k] : static_cast<UT>(0.f);
            }
            for (int i = tid; i < sn; i += CT) st[buf][i] = a.t[rowLH + c0 + i];
        }
    };
    if (async_ok && lstop > 0) stage(0, 0, true);
    // y and the residual partials of the chunk at f0 from slot fb
    auto flush = [&](int f0, int fsteps, int fb) {
        for (int idx = tid; idx < fsteps * HT; idx += CT) {
            const int i = idx / HT, k = idx % HT;
            if (h0 + k < H) a.y[(rowLH + f0 + i) * H + h0 + k] = sy[fb][i][k];
        }
        if (kSpec) {
            for (int i = tid; i < fsteps; i += CT) {
                float s1 = 0.f, s2 = 0.f;
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    s1 += sred[fb][i][w].x;
                    s2 += sred[fb][i][w].y;
                }
                a.part[(static_cast<size_t>(b) * a.ntiles + tile) * L + f0 + i] = make_float2(s1, s2);
            }
        }
    };

    for (int l0 = 0, chunk = 0; l0 < lstop; l0 += kT, ++chunk) {
        const int steps = min(kT, lstop - l0);
        const int buf = chunk & (NBUF - 1);
        const int ob = chunk & 1;           // output slot of this chunk
        if (async_ok) cp_async_wait_all();  // this thread's copies of chunk `chunk`
        __syncthreads();                    // everyone's, and the previous chunk is done
        if (MODE != REPLAY && chunk > 0) flush(l0 - kT, kT, ob ^ 1);
        if (!async_ok) {
            stage(l0, buf, false);
            __syncthreads();
        } else if (l0 + kT < lstop) {
            stage(l0 + kT, (buf ^ 1) & (NBUF - 1), true);
        }

        for (int i0 = 0; i0 < steps; i0 += U) {
            if (MODE == UNGATED && a.ck != nullptr && ((l0 + i0) % kSsmCk) == 0) {
                // training forward: checkpoint of the state before step l0 + i0
                const size_t ko = (static_cast<size_t>(b) * a.nK + (l0 + i0) / kSsmCk) * H + h;
#pragma unroll
                for (int j = 0; j < NPT; ++j)
                    if (nv[j]) a.ck[ko * N + ln + LANES * j] = hs[j];
            }
            float vals[NV];
            // With one lane per step of a group (LANES == U), lane ln of each
            // channel group forms the effective step of step i0 + ln (it
            // depends on the row's times and the channel's scale only) and the
            // group's lanes read it by shuffle, instead of every lane forming
            // all U of them.
            constexpr bool kLaneDt = LANES == U && NPT == 2 && MODE != REPLAY && MODE != SPEC_COMMITS;
            float dte_own = 0.f;
            if constexpr (kLaneDt) {
                const int i = i0 + ln;
                const float tl = st[buf][i];
                const float tp = ln == 0 ? t_prev : st[buf][i - 1];
                float delta;
                if (MODE == UNGATED)
                    delta = (l0 + i == 0) ? dt0 : fmaxf(tl - tp, 0.f);
                else
                    delta = fmaxf(tl - tp, 0.f);
                dte_own = eff_dt(delta, scale, a.dt_min, a.dt_max);
            }
#pragma unroll
            for (int uu = 0; uu < U; ++uu) {
                const int i = i0 + uu;
                // Steps past the end of the last chunk only matter to REPLAY,
                // whose final state is kept; elsewhere they compute values that
                // are never stored (each butterfly sum stays within its step).
                const bool act = MODE == REPLAY ? i < steps : true;
                const float ul = act ? to_f32(su[buf][i][hl]) : 0.f;
                float dte, tl = 0.f;
                if constexpr (kLaneDt) {
                    dte = __shfl_sync(0xffffffffu, dte_own, (tid & 31 & ~(LANES - 1)) | uu);
                } else {
                    tl = act ? st[buf][i] : t_prev;
                    float delta;
                    if (MODE == UNGATED)
                        delta = (l0 + i == 0) ? dt0 : fmaxf(tl - t_prev, 0.f);
                    else
                        delta = fmaxf(tl - t_prev, 0.f);
                    dte = eff_dt(delta, scale, a.dt_min, a.dt_max);
                }
                if (MODE == SPEC_CKPT && i < steps && ((l0 + i) & (a.gK - 1)) == 0) {
                    // the state before step l under the all-commit assumption (rows
                    // that skip get theirs from l* on rewritten by the repair pass)
                    const float t_pi = (kLaneDt && uu > 0) ? st[buf][i - 1] : t_prev;
                    write_gck<LANES, NPT>(a, b, (l0 + i) >> a.gKlog, h, ln, nv, hs, hv && ln == 0, u_prev,
                                          tile == 0 && hl == 0, Bp, Cp, tile == 0 && tid == 0, t_pi);
                }
                float yp = 0.f, yhp = 0.f;
                // Branch-free: channels past H stage u = 0 and padded chains
                // stage B = C = 0, so both keep a zero state and add zeros.
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const int n = ln + LANES * j;
                    const float4 bc = sBC[buf][i][n];
                    const float2 Bl = make_float2(bc.x, bc.y);
                    float2 dA, P, hn, W;
                    if (MODE == UNGATED) {
                        float2 dB;
                        zoh(lam[j], ilam[j], dte, dA, dB);
                        P = cmul(dA, hs[j]);
                        const float2 qc = cmul(dB, Bl);
                        hn = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                    } else {
                        // dB_bar B u = expm1(z) W with W = B u / lam; step l's W is also
                        // the input term of step l+1's prediction (carried in Wp)
                        float2 E;
                        zoh_e(lam[j], dte, dA, E);
                        P = cmul(dA, hs[j]);
                        W = cscale(cmul(Bl, ilam[j]), ul);
                        hn = cfma(E, W, P);
                        if (kSpec) {
                            const float2 xh = cfma(E, Wp[j], P);
                            yhp += cre_mul(Cp[j], xh);
                            Wp[j] = W;
                            if (MODE == SPEC_CKPT) Bp[j] = Bl;  // B_pi for the checkpoints
                        }
                    }
                    if (MODE == REPLAY)
                        hs[j] = act ? hn : hs[j];
                    else
                        hs[j] = hn;
                    // commits: under the all-commit assumption h_pi after step l is h_l;
                    // rows that skip get their steps from l* on rewritten by the repair
                    if (MODE == SPEC_COMMITS && nv[j] && i < steps)
                        a.commit_h[((rowLH + l0 + i) * H + h) * N + n] = hn;
                    if (MODE != REPLAY) {
                        const float2 Cl = make_float2(bc.z, bc.w);
                        yp += cre_mul(Cl, hs[j]);
                        if (kSpec) Cp[j] = Cl;
                    }
                }
                vals[uu] = yp;
                if (kSpec) vals[U + uu] = yhp;
                if (act) {
                    u_prev = ul;
                    if constexpr (!kLaneDt) t_prev = tl;
                }
            }
            if constexpr (kLaneDt) t_prev = st[buf][i0 + U - 1];
            if (MODE == REPLAY) continue;
            Bfly<NV, LANES / 2>::run(vals, ln);
            float r1[Shape::kRem], r2[Shape::kRem];
#pragma unroll
            for (int k = 0; k < Shape::kRem; ++k) {
                r1[k] = 0.f;
                r2[k] = 0.f;
                const int orig = held + k;
                const int i = i0 + (orig % U);
                if (orig < U) {  // output readout of step i
                    if (writer && hv && i < steps) sy[ob][i][hl] = vals[k] + Dh * to_f32(su[buf][i][hl]);
                } else if (kSpec && writer && hv && i < steps) {  // prediction of step i
                    const float ul = to_f32(su[buf][i][hl]);
                    const float obs = (ul - mu) * rsd;
                    const float pred = (vals[k] - mu) * rsd;
                    const float d = obs - pred;
                    r1[k] = d * d;
                    r2[k] = obs * obs;
                }
            }
            if (kSpec) {
                // sum over the channel groups of the warp (lanes with equal ln hold the same step)
#pragma unroll
                for (int o = LANES; o < 32; o <<= 1) {
#pragma unroll
                    for (int k = 0; k < Shape::kRem; ++k) {
                        r1[k] += __shfl_xor_sync(0xffffffffu, r1[k], o);
                        r2[k] += __shfl_xor_sync(0xffffffffu, r2[k], o);
                    }
                }
                if ((tid & 31) < LANES && writer) {
#pragma unroll
                    for (int k = 0; k < Shape::kRem; ++k) {
                        const int orig = held + k;
                        const int i = i0 + (orig % U);
                        if (orig >= U && i < steps) sred[ob][i][tid >> 5] = make_float2(r1[k], r2[k]);
                    }
                }
            }
        }
    }
    if (MODE != REPLAY && lstop > 0) {  // the last chunk
        __syncthreads();
        const int last = (lstop - 1) / kT;
        flush(last * kT, lstop - last * kT, last & 1);
    }
    if (MODE == REPLAY) {
#pragma unroll
        for (int j = 0; j < NPT; ++j)
            if (nv[j]) a.hpi[(static_cast<size_t>(b) * H + h) * N + ln + LANES * j] = hs[j];
    }
    if (kSpec && a.cout_h != nullptr) {
        // state after the last step if every step committed (the repair pass
        // rewrites it for rows that skip); the caller keeps L a multiple of U
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (nv[j]) a.cout_h[(static_cast<size_t>(b) * H + h) * N + n] = hs[j];
            if (tile == 0 && hl == 0 && n < N) {  // B_pi, C_pi: the last step's
                a.cout_B[static_cast<size_t>(b) * N + n] = a.Bc[(rowLH + L - 1) * N + n];
                a.cout_C[static_cast<size_t>(b) * N + n] = Cp[j];
            }
        }
        if (hv && ln == 0) a.cout_u[static_cast<size_t>(b) * H + h] = u_prev;
    }
}

// ---------------------------------------------------------------------------
// 2: residual per (b, l) from the h-tile partials.
// ---------------------------------------------------------------------------
__global__ void cell_resid(Args a) {
    const int b = blockIdx.y;
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= a.L) return;
    float s1 = 0.f, s2 = 0.f;
    const float2* p = a.part + static_cast<size_t>(b) * a.ntiles * a.L + l;
    for (int k = 0; k < a.ntiles; ++k) {
        const float2 v = p[static_cast<size_t>(k) * a.L];
        s1 += v.x;
        s2 += v.y;
    }
    const float num = sqrtf(s1), nobs = sqrtf(s2);
    a.resid[static_cast<size_t>(b) * a.L + l] = num / (nobs + a.eta);
    if (a.stats) a.stats[static_cast<size_t>(b) * a.L + l] = make_float2(num, nobs);
}

// ---------------------------------------------------------------------------
// 3: gates, robust_guard and the first skipped step, one CTA per row.
// spike after step l is l - R_l with R_l the last step <= l that was not a
// spike (r_l > r_{l-1} * spike_ratio), so it is a max-scan over the tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) cell_gates(Args a) {
    __shared__ int swarp[32];
    __shared__ float slast_r;
    __shared__ int slast_R;
    __shared__ int sfirst;
    const int b = blockIdx.x;
    const int tid = threadIdx.x;
    const int lane = tid & 31, wid = tid >> 5;
    const size_t rb = static_cast<size_t>(b) * a.L;
    // R_{l0-1} (last step that was not a spike; the spike count after step
    // l is l - R_l) and r_{l0-1}; a resumed row starts from its carried count
    const bool resumed = a.cin_row != nullptr;
    const float4 cin = resumed ? a.cin_row[b] : make_float4(0.f, 0.f, 0.f, 0.f);
    int carry_R = resumed ? -1 - static_cast<int>(cin.y) : -1;
    float carry_r = cin.z;
    int lstar = a.L;
    int4 rowv = make_int4(a.L, 0, 0, 0);
    for (int l0 = 0; l0 < a.L; l0 += 1024) {
        const int l = l0 + tid;
        const bool valid = l < a.L;
        const float r = valid ? a.resid[rb + l] : 0.f;
        // previous residual
        float rprev = __shfl_up_sync(0xffffffffu, r, 1);
        __shared__ float sbound[32];
        if (lane == 31) sbound[wid] = r;
        __syncthreads();
        if (lane == 0) rprev = (wid == 0) ? carry_r : sbound[wid - 1];
        const bool f = valid && (l >= 1 || resumed) && (r > rprev * a.spike_ratio);
        // inclusive max-scan of key = f ? -1 : l  (R_l), with the tile carry
        int key = f ? -1 : (valid ? l : -1);
        int x = key;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x = max(x, y);
        }
        if (lane == 31) swarp[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int w = swarp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w = max(w, y);
            }
            swarp[lane] = w;
        }
        __syncthreads();
        const int pre_w = wid > 0 ? swarp[wid - 1] : -1;
        const int incl = max(max(x, pre_w), carry_R);          // R_l
        int excl = __shfl_up_sync(0xffffffffu, incl, 1);       // R_{l-1}
        if (lane == 0) excl = max(pre_w, carry_R);
        if (wid == 0 && lane == 0) excl = carry_R;
        const float spike_prev = static_cast<float>((l - 1) - excl);
        float eps_l = a.eps;
        if (a.robust && spike_prev >= static_cast<float>(a.robust_k)) eps_l = a.eps_lo;
        const bool g = r > eps_l;
        if (valid) a.gate[rb + l] = g ? 1.f : 0.f;
        // first skipped step in this tile
        if (tid == 0) sfirst = 0x7fffffff;
        __syncthreads();
        if (valid && !g) atomicMin(&sfirst, l);
        if (l == min(a.L, l0 + 1024) - 1) {  // last step of the tile
            slast_r = r;
            slast_R = incl;
        }
        __syncthreads();
        const int first = sfirst;
        if (first != 0x7fffffff) {
            if (l == first) {
                rowv.x = first;
                rowv.y = __float_as_int(spike_prev);
                rowv.z = __float_as_int(rprev);
                a.row[b] = rowv;
            }
            lstar = first;
            break;
        }
        carry_r = slast_r;
        carry_R = slast_R;
        __syncthreads();
    }
    if (lstar == a.L && tid == 0) {
        a.row[b] = rowv;
        if (a.cout_row != nullptr) {  // every step committed: t_pi is the last step's time
            a.cout_row[b] = make_float4(a.t[rb + a.L - 1], static_cast<float>((a.L - 1) - carry_R),
                                        carry_r, 0.f);
        }
    }
}

// ---------------------------------------------------------------------------
// 5: exact sequential gated cell from l* (one CTA per row).
// ---------------------------------------------------------------------------
template <int LANES, int NPT, typename UT>
__global__ void __launch_bounds__(kRepair) cell_repair(Args a) {
    constexpr int HG = kRepair / LANES;  // channel groups per pass
    constexpr int NP = LANES * NPT;
    __shared__ float2 sBpi[NP];
    __shared__ float2 sCpi[NP];
    __shared__ float2 sred[32];
    __shared__ float sg;

    const int b = blockIdx.x;
    const int L = a.L, H = a.H, N = a.N;
    const int4 rowv = a.row[b];
    const int lstar = rowv.x;
    if (lstar >= L) return;
    const int tid = threadIdx.x;
    const int ln = tid % LANES, hg = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowLH = static_cast<size_t>(b) * L;
    const int lp = lstar > 0 ? lstar - 1 : 0;
    float2* hpi = a.hpi + static_cast<size_t>(b) * H * N;
    float* upi = a.upi + static_cast<size_t>(b) * H;

    // every step before l* committed: the predecessor is step l* - 1, or at
    // l* = 0 the carried state of a resumed row (else step 0's inputs)
    const bool resumed = a.cin_row != nullptr;
    const bool from_carry = lstar == 0 && resumed;
    for (int n = tid; n < N; n += kRepair) {
        sBpi[n] = from_carry ? a.cin_B[static_cast<size_t>(b) * N + n] : a.Bc[(rowLH + lp) * N + n];
        sCpi[n] = from_carry ? a.cin_C[static_cast<size_t>(b) * N + n] : a.Cc[(rowLH + lp) * N + n];
    }
    for (int hh = tid; hh < H; hh += kRepair)
        upi[hh] = from_carry ? a.cin_u[static_cast<size_t>(b) * H + hh] : to_f32(u[(rowLH + lp) * H + hh]);
    float t_pi = lstar > 0 ? a.t[rowLH + lp] : (resumed ? a.cin_row[b].x : a.t[rowLH] - a.dt_init);
    float spike = __int_as_float(rowv.y);
    float prev_r = __int_as_float(rowv.z);
    __syncthreads();

    for (int l = lstar; l < L; ++l) {
        const float tl = a.t[rowLH + l];
        const float delta = fmaxf(tl - t_pi, 0.f);
        // phase A: prediction and residual
        float acc1 = 0.f, acc2 = 0.f;
        for (int h0 = 0; h0 < H; h0 += HG) {
            const int h = h0 + hg;
            const bool hv = h < H;
            float yhp = 0.f;
            float dte = 0.f, upv = 0.f;
            if (hv) {
                dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
                upv = upi[h];
            }
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                if (hv && n < N) {
                    const float2 lm = a.lam[static_cast<size_t>(h) * N + n];
                    float2 dA, dB;
                    zoh(lm, crecip(lm), dte, dA, dB);
                    const float2 P = cmul(dA, hpi[static_cast<size_t>(h) * N + n]);
                    const float2 q = cmul(dB, sBpi[n]);
                    const float2 xh = make_float2(fmaf(q.x, upv, P.x), fmaf(q.y, upv, P.y));
                    yhp += cre_mul(sCpi[n], xh);
                }
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yhp += __shfl_xor_sync(0xffffffffu, yhp, o);
            if (ln == 0 && hv) {
                const float sd = sqrtf(a.var[h] + a.var_eps);
                const float ul = to_f32(u[(rowLH + l) * H + h]);
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
            for (int w = 0; w < kRepair / 32; ++w) {
                s1 += sred[w].x;
                s2 += sred[w].y;
            }
            const float r = sqrtf(s1) / (sqrtf(s2) + a.eta);
            if (a.stats) a.stats[rowLH + l] = make_float2(sqrtf(s1), sqrtf(s2));
            float g;
            if (a.gate_mode == 1) {
                g = 1.0f / (1.0f + expf(-((r - a.eps) / a.Tp)));
            } else {
                float eps_l = a.eps;
                if (a.robust && spike >= static_cast<float>(a.robust_k)) eps_l = a.eps_lo;
                g = r > eps_l ? 1.f : 0.f;
            }
            if (a.robust && (l > 0 || resumed)) spike = (r > prev_r * a.spike_ratio) ? spike + 1.f : 0.f;
            prev_r = r;
            a.gate[rowLH + l] = g;
            a.resid[rowLH + l] = r;
            sg = g;
        }
        __syncthreads();
        const float g = sg;
        const bool soft = a.gate_mode == 1;
        const bool fire = soft || g > 0.5f;
        // phase C: update / select / readout / commit h_pi, u_pi
        for (int h0 = 0; h0 < H; h0 += HG) {
            const int h = h0 + hg;
            const bool hv = h < H;
            float yp = 0.f, dte = 0.f, upv = 0.f, ul = 0.f;
            if (hv) {
                dte = eff_dt(delta, expf(a.log_dt[h]), a.dt_min, a.dt_max);
                upv = upi[h];
                ul = to_f32(u[(rowLH + l) * H + h]);
            }
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                if (hv && n < N) {
                    const size_t o = static_cast<size_t>(h) * N + n;
                    const float2 lm = a.lam[o];
                    float2 dA, dB;
                    zoh(lm, crecip(lm), dte, dA, dB);
                    const float2 hp = hpi[o];
                    const float2 P = cmul(dA, hp);
                    const float2 Cl = a.Cc[(rowLH + l) * N + n];
                    float2 hc, hn = hp;
                    if (fire) {
                        const float2 qc = cmul(dB, a.Bc[(rowLH + l) * N + n]);
                        const float2 hu = make_float2(fmaf(qc.x, ul, P.x), fmaf(qc.y, ul, P.y));
                        if (soft) {
                            const float2 qp = cmul(dB, sBpi[n]);
                            const float2 xh = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                            const float2 gu = cscale(hu, g);
                            hc = cadd(gu, cscale(xh, 1.f - g));
                            hn = cadd(gu, cscale(hp, 1.f - g));
                        } else {
                            hc = hu;
                            hn = hu;
                        }
                        hpi[o] = hn;
                    } else {
                        const float2 qp = cmul(dB, sBpi[n]);
                        hc = make_float2(fmaf(qp.x, upv, P.x), fmaf(qp.y, upv, P.y));
                    }
                    if (a.commit_h != nullptr) a.commit_h[((rowLH + l) * H + h) * N + n] = hn;
                    yp += cre_mul(Cl, hc);
                }
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
            if (ln == 0 && hv) {
                a.y[(rowLH + l) * H + h] = yp + a.D[h] * ul;
                if (soft) upi[h] = g * ul + (1.f - g) * upv;
                else if (fire) upi[h] = ul;
            }
        }
        __syncthreads();
        if (soft) {
            for (int n = tid; n < N; n += kRepair) {
                const float2 Bl = a.Bc[(rowLH + l) * N + n], Cl = a.Cc[(rowLH + l) * N + n];
                sBpi[n] = cadd(cscale(Bl, g), cscale(sBpi[n], 1.f - g));
                sCpi[n] = cadd(cscale(Cl, g), cscale(sCpi[n], 1.f - g));
            }
            t_pi = g * tl + (1.f - g) * t_pi;
        } else if (fire) {
            for (int n = tid; n < N; n += kRepair) {
                sBpi[n] = a.Bc[(rowLH + l) * N + n];
                sCpi[n] = a.Cc[(rowLH + l) * N + n];
            }
            t_pi = tl;
        }
        __syncthreads();
    }
    if (a.cout_h != nullptr) {  // the row's state after its last step
        for (int i = tid; i < H * N; i += kRepair) a.cout_h[static_cast<size_t>(b) * H * N + i] = hpi[i];
        for (int hh = tid; hh < H; hh += kRepair) a.cout_u[static_cast<size_t>(b) * H + hh] = upi[hh];
        for (int n = tid; n < N; n += kRepair) {
            a.cout_B[static_cast<size_t>(b) * N + n] = sBpi[n];
            a.cout_C[static_cast<size_t>(b) * N + n] = sCpi[n];
        }
        if (tid == 0) a.cout_row[b] = make_float4(t_pi, spike, prev_r, 0.f);
    }
}

// ---------------------------------------------------------------------------
// 5' (cluster): the exact sequential gated cell from l*, one thread-block
// cluster of CL CTAs per row.  CTA c owns channels [c*HC, (c+1)*HC); thread
// (hl, ln) owns chains n = ln + LANES*j (j < NPT) and keeps their committed
// state, B_pi, C_pi and its channel's u_pi in registers.  Per step: one ZOH
// per chain (shared by the prediction and the update), the prediction's
// residual sums reduced over the row through distributed shared memory --
// every warp sends its two partial sums to every CTA with st.async, counted
// on that CTA's mbarrier (double-buffered slots, bounded wait) -- then the
// gate, the update and the readout.  Every CTA sums the slots in the same
// order, so all of them take the same gate decision.
// ---------------------------------------------------------------------------
constexpr int kRcMaxThreads = 512;
constexpr int kRcMaxCL = 16;

__device__ __forceinline__ void rc_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

constexpr int kRcT = 32;  // steps per staged input chunk of the cluster repair pass

// Dynamic shared memory of cell_repair_cluster: two input buffers of kRcT
// steps, each B_l and C_l (NP complex), t_l and the CTA's HC channels of u_l.
template <typename UT>
__host__ __device__ constexpr size_t rc_buf_bytes(int NP, int HC) {
    return ((static_cast<size_t>(kRcT) * NP * 2 * sizeof(float2) + kRcT * sizeof(float) +
             static_cast<size_t>(kRcT) * ((HC + 1) & ~1) * sizeof(UT)) + 15) & ~static_cast<size_t>(15);
}

template <int LANES, int NPT, typename UT, int MAXT = kRcMaxThreads>
__global__ void __launch_bounds__(MAXT) cell_repair_cluster(Args a, int CL, int HC) {
    constexpr int NP = LANES * NPT;
    __shared__ uint64_t rbar[2];
    __shared__ float2 slots[2][kRcMaxCL * (kRcMaxThreads / 32)];
    extern __shared__ __align__(16) unsigned char rc_smem[];
    const int b = blockIdx.y;
    const int crank = blockIdx.x;  // the cluster spans the CL CTAs of a row
    const int L = a.L, H = a.H, N = a.N;
    const int4 rowv = a.row[b];
    const int lstar = rowv.x;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int NW = blockDim.x >> 5;
    const int ln = tid % LANES, hl = tid / LANES;
    const int h = crank * HC + hl;
    const bool hv = hl < HC && h < H;
    if (tid == 0) {
        mbar_init(&rbar[0], 1);
        mbar_init(&rbar[1], 1);
        fence_mbar_init();
    }
    rc_cluster_sync();  // barriers initialised everywhere before any remote store
    if (lstar >= L) {   // row verified by the speculative pass (uniform over the cluster)
        rc_cluster_sync();
        return;
    }
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowLH = static_cast<size_t>(b) * L;
    const int lp = lstar > 0 ? lstar - 1 : 0;
    const bool resumed = a.cin_row != nullptr;

    float2 lam[NPT], ilam[NPT], hs[NPT], Bp[NPT], Cp[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        const size_t o = static_cast<size_t>(hv ? h : 0) * N + (n < N ? n : 0);
        lam[j] = nv[j] ? a.lam[o] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        hs[j] = nv[j] ? a.hpi[static_cast<size_t>(b) * H * N + o] : make_float2(0.f, 0.f);
        // every step before l* committed: the predecessor is step l* - 1, or at
        // l* = 0 the carried state of a resumed row (else step 0's inputs)
        Bp[j] = (n < N) ? a.Bc[(rowLH + lp) * N + n] : make_float2(0.f, 0.f);
        Cp[j] = (n < N) ? a.Cc[(rowLH + lp) * N + n] : make_float2(0.f, 0.f);
        if (lstar == 0 && resumed && n < N) {
            Bp[j] = a.cin_B[static_cast<size_t>(b) * N + n];
            Cp[j] = a.cin_C[static_cast<size_t>(b) * N + n];
        }
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float rsd = hv ? 1.0f / sqrtf(a.var[h] + a.var_eps) : 1.f;
    const float mu = hv ? a.mean[h] : 0.f;
    const float Dh = hv ? a.D[h] : 0.f;
    float u_pi = hv ? to_f32(u[(rowLH + lp) * H + h]) : 0.f;
    float t_pi = lstar > 0 ? a.t[rowLH + lp] : a.t[rowLH] - a.dt_init;
    if (lstar == 0 && resumed) {
        if (hv) u_pi = a.cin_u[static_cast<size_t>(b) * H + h];
        t_pi = a.cin_row[b].x;
    }
    float spike = __int_as_float(rowv.y);
    float prev_r = __int_as_float(rowv.z);
    const bool soft = a.gate_mode == 1;
    const int nslot = CL * NW;
    uint32_t rslot[2] = {0u, 0u}, rbarr[2] = {0u, 0u};
    if (lane < CL) {  // lane c sends to CTA c
        rslot[0] = mapa_u32(&slots[0][crank * NW + wid], lane);
        rslot[1] = mapa_u32(&slots[1][crank * NW + wid], lane);
        rbarr[0] = mapa_u32(&rbar[0], lane);
        rbarr[1] = mapa_u32(&rbar[1], lane);
    }
    bool failed = false;

    // Inputs of kRcT steps at a time in shared memory, the next chunk copied
    // in with cp.async while this one runs (zero-filled past N and H).
    const int HC2 = (HC + 1) & ~1;
    const size_t buf_bytes = rc_buf_bytes<UT>(NP, HC);
    auto sBl = [&](int buf, int i) { return reinterpret_cast<float2*>(rc_smem + buf * buf_bytes) + i * NP; };
    auto sCl = [&](int buf, int i) { return reinterpret_cast<float2*>(rc_smem + buf * buf_bytes) + (kRcT + i) * NP; };
    auto stl = [&](int buf) { return reinterpret_cast<float*>(rc_smem + buf * buf_bytes + 2 * kRcT * NP * sizeof(float2)); };
    auto sul = [&](int buf, int i) {
        return reinterpret_cast<UT*>(rc_smem + buf * buf_bytes + 2 * kRcT * NP * sizeof(float2) + kRcT * sizeof(float)) +
               i * HC2;
    };
    const int h0 = crank * HC;
    constexpr bool kPair = sizeof(UT) == 2;
    // 4-byte copies: u in pairs of channels when it is 2 bytes wide
    const bool async_ok = (reinterpret_cast<uintptr_t>(u) & 3u) == 0 && (!kPair || ((H | h0) & 1) == 0) &&
                          ((reinterpret_cast<uintptr_t>(a.Bc) | reinterpret_cast<uintptr_t>(a.Cc)) & 7u) == 0 &&
                          (reinterpret_cast<uintptr_t>(a.t) & 3u) == 0;
    auto stage = [&](int c0, int buf) {
        const int sn = min(kRcT, L - c0);
        for (int idx = tid; idx < sn * NP; idx += blockDim.x) {
            const int i = idx / NP, n = idx % NP;
            const size_t o = (rowLH + c0 + i) * N + n;
            if (async_ok) {
                cp_async8(sBl(buf, i) + n, n < N ? a.Bc + o : a.Bc, n < N);
                cp_async8(sCl(buf, i) + n, n < N ? a.Cc + o : a.Cc, n < N);
            } else {
                sBl(buf, i)[n] = n < N ? a.Bc[o] : make_float2(0.f, 0.f);
                sCl(buf, i)[n] = n < N ? a.Cc[o] : make_float2(0.f, 0.f);
            }
        }
        constexpr int P = kPair ? 2 : 1;
        for (int idx = tid; idx < sn * (HC2 / P); idx += blockDim.x) {
            const int i = idx / (HC2 / P), c = (idx % (HC2 / P)) * P;
            const bool ok = h0 + c < H && c < HC;
            const UT* src = u + (rowLH + c0 + i) * H + h0 + c;
            if (async_ok) {
                cp_async4(sul(buf, i) + c, ok ? src : u, ok);
            } else {
#pragma unroll
                for (int e = 0; e < P; ++e)
                    sul(buf, i)[c + e] = (h0 + c + e < H && c + e < HC) ? src[e] : static_cast<UT>(0.f);
            }
        }
        for (int i = tid; i < sn; i += blockDim.x) {
            if (async_ok) cp_async4(stl(buf) + i, a.t + rowLH + c0 + i, true);
            else stl(buf)[i] = a.t[rowLH + c0 + i];
        }
        if (async_ok) cp_async_commit();
    };
    stage(lstar, 0);

    for (int c0 = lstar, chunk = 0; c0 < L; c0 += kRcT, ++chunk) {
    const int buf = chunk & 1;
    const int csteps = min(kRcT, L - c0);
    if (async_ok) cp_async_wait_all();
    __syncthreads();  // chunk c0 staged; every thread is done with the other buffer
    if (c0 + kRcT < L) stage(c0 + kRcT, buf ^ 1);
    for (int i = 0; i < csteps; ++i) {
        const int l = c0 + i;
        const float tl = stl(buf)[i];
        const float ul = hv ? to_f32(sul(buf, i)[hl]) : 0.f;
        float2 Bl[NPT], Cl[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            Bl[j] = sBl(buf, i)[ln + LANES * j];
            Cl[j] = sCl(buf, i)[ln + LANES * j];
        }
        if (a.gck_h != nullptr && (l & (a.gK - 1)) == 0)  // training checkpoint: the committed state before step l
            write_gck<LANES, NPT>(a, b, l >> a.gKlog, h, ln, nv, hs, hv && ln == 0, u_pi, crank == 0 && hl == 0, Bp,
                                  Cp, crank == 0 && tid == 0, t_pi);
        const float dte = eff_dt(fmaxf(tl - t_pi, 0.f), scale, a.dt_min, a.dt_max);
        float2 P[NPT], dB[NPT], xh[NPT];
        float yhp = 0.f;
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            float2 dA;
            zoh(lam[j], ilam[j], dte, dA, dB[j]);
            P[j] = cmul(dA, hs[j]);
            const float2 q = cmul(dB[j], Bp[j]);
            xh[j] = make_float2(fmaf(q.x, u_pi, P[j].x), fmaf(q.y, u_pi, P[j].y));
            yhp += cre_mul(Cp[j], xh[j]);
        }
#pragma unroll
        for (int o = LANES / 2; o > 0; o >>= 1) yhp += __shfl_xor_sync(0xffffffffu, yhp, o);
        float d2 = 0.f, o2 = 0.f;
        if (hv && ln == 0) {
            const float obs = (ul - mu) * rsd;
            const float dd = obs - (yhp - mu) * rsd;
            d2 = dd * dd;
            o2 = obs * obs;
        }
        d2 = warp_sum(d2);
        o2 = warp_sum(o2);
        // row sums through the cluster
        const int k = l - lstar;
        const int par = k & 1;
        const uint32_t phase = (k >> 1) & 1;
        if (!failed) {
            if (tid == 0) mbar_expect_tx(&rbar[par], static_cast<uint32_t>(nslot) * 8u);
            if (lane < CL) {
                // addresses by select: a dynamic index would keep the arrays in local memory
                const uint32_t rs = par ? rslot[1] : rslot[0], rb = par ? rbarr[1] : rbarr[0];
                st_async_f32(rs, d2, rb);
                st_async_f32(rs + 4u, o2, rb);
            }
            if (!mbar_wait_row(&rbar[par], phase)) failed = true;
        }
        float s1 = 0.f, s2 = 0.f;
        for (int q = lane; q < nslot; q += 32) {
            const float2 v = slots[par][q];
            s1 += v.x;
            s2 += v.y;
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        const float num = sqrtf(s1), nobs = sqrtf(s2);
        const float r = num / (nobs + a.eta);
        float g;
        if (soft) {
            g = 1.0f / (1.0f + expf(-((r - a.eps) / a.Tp)));
        } else {
            float eps_l = a.eps;
            if (a.robust && spike >= static_cast<float>(a.robust_k)) eps_l = a.eps_lo;
            g = r > eps_l ? 1.f : 0.f;
        }
        if (a.robust) {
            if (l > 0 || resumed) spike = (r > prev_r * a.spike_ratio) ? spike + 1.f : 0.f;
            prev_r = r;
        } else {
            prev_r = r;
        }
        if (crank == 0 && tid == 0) {
            a.gate[rowLH + l] = g;
            a.resid[rowLH + l] = r;
            if (a.stats) a.stats[rowLH + l] = make_float2(num, nobs);
        }
        // update, readout, commit
        float yp = 0.f;
        const bool fire = soft || g > 0.5f;
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            float2 hc = xh[j];
            if (fire) {
                const float2 qc = cmul(dB[j], Bl[j]);
                const float2 hu = make_float2(fmaf(qc.x, ul, P[j].x), fmaf(qc.y, ul, P[j].y));
                if (soft) {
                    const float2 gu = cscale(hu, g);
                    hc = cadd(gu, cscale(xh[j], 1.f - g));
                    hs[j] = cadd(gu, cscale(hs[j], 1.f - g));
                } else {
                    hc = hu;
                    hs[j] = hu;
                }
            }
            yp += cre_mul(Cl[j], hc);
            if (a.commit_h != nullptr && nv[j])
                a.commit_h[((rowLH + l) * H + h) * N + ln + LANES * j] = hs[j];
        }
#pragma unroll
        for (int o = LANES / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
        if (hv && ln == 0) a.y[(rowLH + l) * H + h] = yp + Dh * ul;
        if (soft) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                Bp[j] = cadd(cscale(Bl[j], g), cscale(Bp[j], 1.f - g));
                Cp[j] = cadd(cscale(Cl[j], g), cscale(Cp[j], 1.f - g));
            }
            u_pi = g * ul + (1.f - g) * u_pi;
            t_pi = g * tl + (1.f - g) * t_pi;
        } else if (fire) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                Bp[j] = Bl[j];
                Cp[j] = Cl[j];
            }
            u_pi = ul;
            t_pi = tl;
        }
    }
    }
    if (a.cout_h != nullptr) {  // the row's state after its last step
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (nv[j]) a.cout_h[(static_cast<size_t>(b) * H + h) * N + n] = hs[j];
            if (crank == 0 && hl == 0 && n < N) {
                a.cout_B[static_cast<size_t>(b) * N + n] = Bp[j];
                a.cout_C[static_cast<size_t>(b) * N + n] = Cp[j];
            }
        }
        if (hv && ln == 0) a.cout_u[static_cast<size_t>(b) * H + h] = u_pi;
        if (crank == 0 && tid == 0) a.cout_row[b] = make_float4(t_pi, spike, prev_r, 0.f);
    }
    rc_cluster_sync();  // no CTA leaves while a peer may still write its slots
}

// Cluster shape of the repair pass for (H, N) over B rows: LANES x NPT chains
// per channel and CL CTAs per row with at most kRcMaxThreads threads each; 0
// when the shape does not fit (the one-CTA repair pass handles it).  CL is
// the smallest of 8, 10, .., EACS_RC_MAXCL that fits.  (A repair step is
// bound by its dependent instruction chain and the cluster exchange, not by
// the SM count: 12- and 16-CTA rows at config 1's shape measured no faster,
// and with one CTA per SM slower, since fewer such clusters are resident.)
#ifndef EACS_RC_MAXCL
#define EACS_RC_MAXCL 16
#endif
struct RcShape {
    int lanes, npt, cl, hc, threads;
};
RcShape rc_shape(int H, int N, int B) {
    (void)B;
    RcShape r{0, 0, 0, 0, 0};
    if (N <= 4) { r.lanes = 4; r.npt = 1; }
    else if (N <= 8) { r.lanes = 4; r.npt = 2; }
    else if (N <= 16) { r.lanes = 4; r.npt = 4; }
    else if (N <= 32) { r.lanes = 8; r.npt = 4; }
    else if (N <= 64) { r.lanes = 16; r.npt = 4; }
    else return r;
    int best = 0;
    for (int cl = 8; cl <= kRcMaxCL && cl <= EACS_RC_MAXCL && best == 0; cl += 2) {
        const int hc = (H + cl - 1) / cl;
        if (((hc * r.lanes + 31) / 32) * 32 <= kRcMaxThreads) best = cl;
    }
    if (best == 0) return r;
    r.cl = best;
    r.hc = (H + best - 1) / best;
    r.threads = ((r.hc * r.lanes + 31) / 32) * 32;
    return r;
}

template <int LANES, int NPT, typename UT>
cudaError_t launch_repair_cluster(const Args& a, const RcShape& rs, cudaStream_t s) {
    // CTAs of at most 384 threads (config 1: 96 channels x 4 lanes) may use up
    // to 168 registers a thread instead of the 512-thread bound's 128
    auto kern = rs.threads <= 384 ? cell_repair_cluster<LANES, NPT, UT, 384> : cell_repair_cluster<LANES, NPT, UT>;
    cudaError_t e;
    if (rs.cl > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    const size_t smem = 2 * rc_buf_bytes<UT>(LANES * NPT, rs.hc);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rs.cl, a.B);
    cfg.blockDim = dim3(rs.threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = rs.cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a, rs.cl, rs.hc);
    note_launch();
    return e;
}

// ---------------------------------------------------------------------------
// 5b: windowed speculative repair (hard gate, no commit or checkpoint
// recording).  From l* on, a row's gates are decided a window of up to
// kWinMax steps per cluster exchange instead of one step per exchange.  A
// window runs under one hypothesis: every step commits (after a committed
// step) or every step skips (after a skipped one).  Under "commit" the
// committed state of step k is step k-1's update (a linear chain, as in the
// speculative pass); under "skip" it stays the window's starting state, so
// the window's predictions are independent of one another.  Every step
// forms its prediction x_hat, its update h_upd = dA h_pi + E W_l and both
// candidate outputs Re C_l x_hat and Re C_l h_upd; one exchange then gives
// each CTA the residual sums of all the window's steps.  The gates are taken
// in order and the window is accepted up to and including the first step
// whose gate differs from the hypothesis: that step's prediction came from
// the exact committed state, so it is exact whichever way its gate went.
// The committed state then moves to the update of the last committed step
// (each step's update is kept in shared memory for this), and the next
// window runs under the hypothesis that the last accepted step's gate makes
// true.  Window lengths follow the run lengths seen for each hypothesis.
// ---------------------------------------------------------------------------
constexpr int kWinMax = 8;

template <typename UT>
__host__ __device__ constexpr size_t win_smem_bytes(int NP, int NPT, int T, int HC) {
    return 2 * rc_buf_bytes<UT>(NP, HC) +                                   // staged inputs
           static_cast<size_t>(kWinMax + 1) * NPT * T * sizeof(float2) +     // updates (+ start state)
           static_cast<size_t>(kWinMax) * HC * 2 * sizeof(float) +           // candidate outputs
           static_cast<size_t>(kWinMax) * (T / 32) * sizeof(float2);         // warp residual sums
}

template <int LANES, int NPT, typename UT, int MAXT = kRcMaxThreads>
__global__ void __launch_bounds__(MAXT) cell_repair_window(Args a, int CL, int HC) {
    constexpr int NP = LANES * NPT;
    constexpr int V = 3 * kWinMax;  // per step: y_hat (prediction), y if skipped, y if committed
    using Shape = BflyShape<V, LANES>;
    __shared__ uint64_t rbar[2];
    __shared__ float2 slots[2][kRcMaxCL][kWinMax];  // (sum d^2, sum obs^2) per source CTA and step
    __shared__ float2 wslots[2][kRcMaxCL * (kRcMaxThreads / 32)];  // single steps: per source warp
    extern __shared__ __align__(16) unsigned char rc_smem[];
    const int b = blockIdx.y;
    const int crank = blockIdx.x;
    const int L = a.L, H = a.H, N = a.N;
    const int4 rowv = a.row[b];
    const int lstar = rowv.x;
    const int tid = threadIdx.x;
    const int T = blockDim.x, NW = T >> 5;
    const int ln = tid % LANES, hl = tid / LANES;
    const int h0 = crank * HC;
    const int h = h0 + hl;
    const bool hv = hl < HC && h < H;
    if (tid == 0) {
        mbar_init(&rbar[0], 1);
        mbar_init(&rbar[1], 1);
        fence_mbar_init();
    }
    rc_cluster_sync();  // barriers initialised everywhere before any remote store
    if (lstar >= L) {
        rc_cluster_sync();
        return;
    }
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowLH = static_cast<size_t>(b) * L;
    const int lp = lstar > 0 ? lstar - 1 : 0;
    const bool resumed = a.cin_row != nullptr;
    const bool from_carry = lstar == 0 && resumed;

    float2 lam[NPT], ilam[NPT], hs[NPT], Cp[NPT], Wc[NPT];
    bool nv[NPT];
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float rsd = hv ? 1.0f / sqrtf(a.var[h] + a.var_eps) : 1.f;
    const float mu = hv ? a.mean[h] : 0.f;
    // committed inputs (u_pi, B_pi, C_pi) of step lc, or with lc < 0 those the
    // row held before l*: step l* - 1's, a resumed row's carried ones, or step 0's
    auto committed_inputs = [&](int lc, float& upi, float2 (&Bq)[NPT], float2 (&Cq)[NPT]) {
        const int ls = lc >= 0 ? lc : lp;
        upi = hv ? to_f32(u[(rowLH + ls) * H + h]) : 0.f;
        if (lc < 0 && from_carry && hv) upi = a.cin_u[static_cast<size_t>(b) * H + h];
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            Bq[j] = n < N ? a.Bc[(rowLH + ls) * N + n] : make_float2(0.f, 0.f);
            Cq[j] = n < N ? a.Cc[(rowLH + ls) * N + n] : make_float2(0.f, 0.f);
            if (lc < 0 && from_carry && n < N) {
                Bq[j] = a.cin_B[static_cast<size_t>(b) * N + n];
                Cq[j] = a.cin_C[static_cast<size_t>(b) * N + n];
            }
        }
    };
    float u_pi;
    {
        float2 Bq[NPT];
        committed_inputs(-1, u_pi, Bq, Cp);
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            nv[j] = hv && n < N;
            const size_t o = static_cast<size_t>(hv ? h : 0) * N + (n < N ? n : 0);
            lam[j] = nv[j] ? a.lam[o] : make_float2(-1.f, 0.f);
            ilam[j] = crecip(lam[j]);
            hs[j] = nv[j] ? a.hpi[static_cast<size_t>(b) * H * N + o] : make_float2(0.f, 0.f);
            Wc[j] = cscale(cmul(Bq[j], ilam[j]), u_pi);
        }
    }
    float t_pi = lstar > 0 ? a.t[rowLH + lp] : a.t[rowLH] - a.dt_init;
    if (from_carry) t_pi = a.cin_row[b].x;
    float spike = __int_as_float(rowv.y);
    float prev_r = __int_as_float(rowv.z);
    int lc = -1;  // last committed step since l* (-1: none yet)

    // shared memory: staged inputs (kRcT steps per buffer, two buffers), the
    // window's updates [k][j][thread] and the start state, candidate outputs,
    // per-warp residual sums
    const int HC2 = (HC + 1) & ~1;
    const size_t buf_bytes = rc_buf_bytes<UT>(NP, HC);
    auto sBl = [&](int buf, int i) { return reinterpret_cast<float2*>(rc_smem + buf * buf_bytes) + i * NP; };
    auto sCl = [&](int buf, int i) { return reinterpret_cast<float2*>(rc_smem + buf * buf_bytes) + (kRcT + i) * NP; };
    auto stl = [&](int buf) { return reinterpret_cast<float*>(rc_smem + buf * buf_bytes + 2 * kRcT * NP * sizeof(float2)); };
    auto sul = [&](int buf, int i) {
        return reinterpret_cast<UT*>(rc_smem + buf * buf_bytes + 2 * kRcT * NP * sizeof(float2) + kRcT * sizeof(float)) +
               i * HC2;
    };
    float2* hist = reinterpret_cast<float2*>(rc_smem + 2 * buf_bytes);
    float* ycand = reinterpret_cast<float*>(hist + static_cast<size_t>(kWinMax + 1) * NPT * T);
    float2* wsum = reinterpret_cast<float2*>(ycand + static_cast<size_t>(kWinMax) * HC * 2);

    constexpr bool kPair = sizeof(UT) == 2;
    const bool async_ok = (reinterpret_cast<uintptr_t>(u) & 3u) == 0 && (!kPair || ((H | h0) & 1) == 0) &&
                          ((reinterpret_cast<uintptr_t>(a.Bc) | reinterpret_cast<uintptr_t>(a.Cc)) & 7u) == 0 &&
                          (reinterpret_cast<uintptr_t>(a.t) & 3u) == 0;
    // chunk c holds steps [l* + c kRcT, l* + (c+1) kRcT) in buffer c & 1
    auto stage = [&](int c) {
        const int c0 = lstar + c * kRcT, buf = c & 1;
        const int sn = min(kRcT, L - c0);
        for (int idx = tid; idx < sn * NP; idx += T) {
            const int i = idx / NP, n = idx % NP;
            const size_t o = (rowLH + c0 + i) * N + n;
            if (async_ok) {
                cp_async8(sBl(buf, i) + n, n < N ? a.Bc + o : a.Bc, n < N);
                cp_async8(sCl(buf, i) + n, n < N ? a.Cc + o : a.Cc, n < N);
            } else {
                sBl(buf, i)[n] = n < N ? a.Bc[o] : make_float2(0.f, 0.f);
                sCl(buf, i)[n] = n < N ? a.Cc[o] : make_float2(0.f, 0.f);
            }
        }
        constexpr int P = kPair ? 2 : 1;
        for (int idx = tid; idx < sn * (HC2 / P); idx += T) {
            const int i = idx / (HC2 / P), c2 = (idx % (HC2 / P)) * P;
            const bool ok = h0 + c2 < H && c2 < HC;
            const UT* src = u + (rowLH + c0 + i) * H + h0 + c2;
            if (async_ok) {
                cp_async4(sul(buf, i) + c2, ok ? src : u, ok);
            } else {
#pragma unroll
                for (int e = 0; e < P; ++e)
                    sul(buf, i)[c2 + e] = (h0 + c2 + e < H && c2 + e < HC) ? src[e] : static_cast<UT>(0.f);
            }
        }
        for (int i = tid; i < sn; i += T) {
            if (async_ok) cp_async4(stl(buf) + i, a.t + rowLH + c0 + i, true);
            else stl(buf)[i] = a.t[rowLH + c0 + i];
        }
        if (async_ok) cp_async_commit();
    };
    int issued = 0, ready = 0;  // chunks issued / known complete (uniform over the CTA)
    const int nchunks = (L - lstar + kRcT - 1) / kRcT;

    float run_skip = 2.f, run_commit = 2.f;  // run lengths seen for each hypothesis
    int run = 0;                    // accepted steps of the current hypothesis so far
    bool cr = false;                // l* skips: the first window assumes skips
    int wlen = kWinMax;
    bool failed = false;
    for (int l0 = lstar, w = 0; l0 < L; ++w) {
        const int Wn = min(wlen, L - l0);
        const int r0 = l0 - lstar;
        const int cA = r0 / kRcT, cB = (r0 + Wn - 1) / kRcT;
        while (issued <= cB) stage(issued++);
        if (ready <= cB) {
            if (async_ok) cp_async_wait_all();
            __syncthreads();
            ready = issued;
        }
        if (cA == cB && issued == cB + 1 && issued < nchunks) stage(issued++);  // the next chunk

        if (Wn == 1) {
            // ---- one step (short runs): every warp sends its own partial sums
            // straight to every CTA, and no shared-memory staging of results ----
            const int buf = (r0 / kRcT) & 1, i = r0 % kRcT;
            const float tl = stl(buf)[i];
            const float ul = hv ? to_f32(sul(buf, i)[hl]) : 0.f;
            const float dte = eff_dt(fmaxf(tl - t_pi, 0.f), scale, a.dt_min, a.dt_max);
            float2 P[NPT], E[NPT], xh[NPT];
            float yhp = 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                float2 dA;
                zoh_e(lam[j], dte, dA, E[j]);
                P[j] = cmul(dA, hs[j]);
                xh[j] = cfma(E[j], Wc[j], P[j]);
                yhp += cre_mul(Cp[j], xh[j]);
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yhp += __shfl_xor_sync(0xffffffffu, yhp, o);
            float d2 = 0.f, o2 = 0.f;
            if (hv && ln == 0) {
                const float obs = (ul - mu) * rsd;
                const float dd = obs - (yhp - mu) * rsd;
                d2 = dd * dd;
                o2 = obs * obs;
            }
            d2 = warp_sum(d2);
            o2 = warp_sum(o2);
            const int par = w & 1;
            const uint32_t phase = (w >> 1) & 1;
            const int nslot = CL * NW;
            if (!failed) {
                if (tid == 0) mbar_expect_tx(&rbar[par], static_cast<uint32_t>(nslot) * 8u);
                if ((tid & 31) < CL) {  // lane c sends to CTA c
                    const uint32_t rs = mapa_u32(&wslots[par][crank * NW + (tid >> 5)], tid & 31);
                    const uint32_t rb = mapa_u32(&rbar[par], tid & 31);
                    st_async_f32(rs, d2, rb);
                    st_async_f32(rs + 4u, o2, rb);
                }
                if (!mbar_wait_row(&rbar[par], phase)) failed = true;
            }
            float s1 = 0.f, s2 = 0.f;
            for (int q = tid & 31; q < nslot; q += 32) {
                const float2 v = wslots[par][q];
                s1 += v.x;
                s2 += v.y;
            }
            s1 = warp_sum(s1);
            s2 = warp_sum(s2);
            const float num = sqrtf(s1), nobs = sqrtf(s2);
            const float r = num / (nobs + a.eta);
            float eps_l = a.eps;
            if (a.robust && spike >= static_cast<float>(a.robust_k)) eps_l = a.eps_lo;
            const bool g = r > eps_l;
            if (a.robust && (l0 > 0 || resumed)) spike = (r > prev_r * a.spike_ratio) ? spike + 1.f : 0.f;
            prev_r = r;
            if (crank == 0 && tid == 0) {
                a.gate[rowLH + l0] = g ? 1.f : 0.f;
                a.resid[rowLH + l0] = r;
                if (a.stats) a.stats[rowLH + l0] = make_float2(num, nobs);
            }
            float yp = 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const float2 Cl = sCl(buf, i)[ln + LANES * j];
                float2 hc = xh[j];
                if (g) {
                    const float2 Wk = cscale(cmul(sBl(buf, i)[ln + LANES * j], ilam[j]), ul);
                    hc = cfma(E[j], Wk, P[j]);
                    hs[j] = hc;
                    Wc[j] = Wk;
                    Cp[j] = Cl;
                }
                yp += cre_mul(Cl, hc);
            }
#pragma unroll
            for (int o = LANES / 2; o > 0; o >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
            if (hv && ln == 0) a.y[(rowLH + l0) * H + h] = yp + a.D[h] * ul;
            if (g) {
                t_pi = tl;
                u_pi = ul;
                lc = l0;
            }
            if (g != cr) {
                float& est = cr ? run_commit : run_skip;
                est = 0.5f * est + 0.5f * static_cast<float>(run);
                run = 1;
                cr = g;
            } else {
                ++run;
            }
            const float m = fmaxf(cr ? run_commit : run_skip, static_cast<float>(run));
            wlen = m < 5.f ? 1 : min(kWinMax, max(2, __float2int_rn(sqrtf(1.3f * m))));
            ++l0;
            continue;
        }

        // ---- the window under the hypothesis ----
        if (cr) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) hist[(static_cast<size_t>(kWinMax) * NPT + j) * T + tid] = hs[j];
        }
        float vals[V];
        float tp = t_pi;
#pragma unroll
        for (int k = 0; k < kWinMax; ++k) {
            vals[k] = vals[kWinMax + k] = vals[2 * kWinMax + k] = 0.f;
            if (k < Wn) {
                const int r = r0 + k, buf = (r / kRcT) & 1, i = r % kRcT;
                const float tl = stl(buf)[i];
                const float ul = hv ? to_f32(sul(buf, i)[hl]) : 0.f;
                const float dte = eff_dt(fmaxf(tl - tp, 0.f), scale, a.dt_min, a.dt_max);
                float yh = 0.f, ys = 0.f, yc = 0.f;
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const float2 Bl = sBl(buf, i)[ln + LANES * j];
                    const float2 Cl = sCl(buf, i)[ln + LANES * j];
                    float2 dA, E;
                    zoh_e(lam[j], dte, dA, E);
                    const float2 P = cmul(dA, hs[j]);
                    const float2 xh = cfma(E, Wc[j], P);
                    const float2 Wk = cscale(cmul(Bl, ilam[j]), ul);
                    const float2 hk = cfma(E, Wk, P);
                    yh += cre_mul(Cp[j], xh);
                    ys += cre_mul(Cl, xh);
                    yc += cre_mul(Cl, hk);
                    hist[(static_cast<size_t>(k) * NPT + j) * T + tid] = hk;
                    if (cr) {  // the next step's committed state is this step's update
                        hs[j] = hk;
                        Wc[j] = Wk;
                        Cp[j] = Cl;
                    }
                }
                if (cr) tp = tl;
                vals[k] = yh;
                vals[kWinMax + k] = ys;
                vals[2 * kWinMax + k] = yc;
            }
        }
        Bfly<V, LANES / 2>::run(vals, ln);
        // residual terms of the predictions; candidate outputs to shared memory
        float dd[Shape::kRem], oo[Shape::kRem];
        const int held = Shape::held_index(ln);
#pragma unroll
        for (int q = 0; q < Shape::kRem; ++q) {
            const int orig = held + q, k = orig % kWinMax, kind = orig / kWinMax;
            dd[q] = 0.f;
            oo[q] = 0.f;
            if (hv && k < Wn) {
                if (kind == 0) {
                    const int r = r0 + k;
                    const float ul = to_f32(sul((r / kRcT) & 1, r % kRcT)[hl]);
                    const float obs = (ul - mu) * rsd;
                    const float d = obs - (vals[q] - mu) * rsd;
                    dd[q] = d * d;
                    oo[q] = obs * obs;
                } else if ((ln & Shape::kPlainMask) == 0) {
                    ycand[(k * HC + hl) * 2 + (kind - 1)] = vals[q];
                }
            }
        }
#pragma unroll
        for (int o = LANES; o < 32; o <<= 1) {
#pragma unroll
            for (int q = 0; q < Shape::kRem; ++q) {
                dd[q] += __shfl_xor_sync(0xffffffffu, dd[q], o);
                oo[q] += __shfl_xor_sync(0xffffffffu, oo[q], o);
            }
        }
        if ((tid & 31) < LANES && (ln & Shape::kPlainMask) == 0) {
#pragma unroll
            for (int q = 0; q < Shape::kRem; ++q) {
                const int orig = held + q;
                if (orig < Wn) wsum[orig * NW + (tid >> 5)] = make_float2(dd[q], oo[q]);
            }
        }
        __syncthreads();
        // ---- one exchange: this CTA's sums of the window's steps to every CTA ----
        const int par = w & 1;
        const uint32_t phase = (w >> 1) & 1;
        if (!failed) {
            if (tid == 0) mbar_expect_tx(&rbar[par], static_cast<uint32_t>(CL * Wn) * 8u);
            if (tid < Wn) {
                float s1 = 0.f, s2 = 0.f;
                for (int q = 0; q < NW; ++q) {
                    const float2 v = wsum[tid * NW + q];
                    s1 += v.x;
                    s2 += v.y;
                }
                for (int c = 0; c < CL; ++c) {
                    const uint32_t rs = mapa_u32(&slots[par][crank][tid], c), rb = mapa_u32(&rbar[par], c);
                    st_async_f32(rs, s1, rb);
                    st_async_f32(rs + 4u, s2, rb);
                }
            }
            if (!mbar_wait_row(&rbar[par], phase)) failed = true;
        }
        // ---- gates in order, up to the first step against the hypothesis ----
        int A = Wn;
        unsigned gmask = 0u;
        bool deviated = false;
        for (int k = 0; k < Wn; ++k) {
            float s1 = 0.f, s2 = 0.f;
            for (int c = 0; c < CL; ++c) {
                const float2 v = slots[par][c][k];
                s1 += v.x;
                s2 += v.y;
            }
            const float num = sqrtf(s1), nobs = sqrtf(s2);
            const float r = num / (nobs + a.eta);
            const int l = l0 + k;
            float eps_l = a.eps;
            if (a.robust && spike >= static_cast<float>(a.robust_k)) eps_l = a.eps_lo;
            const bool g = r > eps_l;
            if (a.robust && (l > 0 || resumed)) spike = (r > prev_r * a.spike_ratio) ? spike + 1.f : 0.f;
            prev_r = r;
            if (crank == 0 && tid == 0) {
                a.gate[rowLH + l] = g ? 1.f : 0.f;
                a.resid[rowLH + l] = r;
                if (a.stats) a.stats[rowLH + l] = make_float2(num, nobs);
            }
            if (g) gmask |= 1u << k;
            if (g != cr) {
                A = k + 1;
                deviated = true;
                break;
            }
        }
        // ---- outputs of the accepted steps ----
        for (int idx = tid; idx < A * HC; idx += T) {
            const int k = idx / HC, c = idx % HC;
            const int hh = h0 + c;
            if (hh < H) {
                const int r = r0 + k;
                const float ul = to_f32(sul((r / kRcT) & 1, r % kRcT)[c]);
                a.y[(rowLH + l0 + k) * H + hh] = ycand[(k * HC + c) * 2 + ((gmask >> k) & 1u)] + a.D[hh] * ul;
            }
        }
        // ---- the committed state after the window ----
        const bool last_g = (gmask >> (A - 1)) & 1u;
        const int kc = last_g ? A - 1 : (cr ? A - 2 : -1);
        if (kc >= 0) {
            const int r = r0 + kc, buf = (r / kRcT) & 1, i = r % kRcT;
            t_pi = stl(buf)[i];
            u_pi = hv ? to_f32(sul(buf, i)[hl]) : 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                hs[j] = hist[(static_cast<size_t>(kc) * NPT + j) * T + tid];
                Cp[j] = sCl(buf, i)[ln + LANES * j];
                Wc[j] = cscale(cmul(sBl(buf, i)[ln + LANES * j], ilam[j]), u_pi);
            }
            lc = l0 + kc;
        } else if (cr) {  // "commit" window whose first step skipped: back to its start state
            float2 Bq[NPT];
            committed_inputs(lc, u_pi, Bq, Cp);
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                hs[j] = hist[(static_cast<size_t>(kWinMax) * NPT + j) * T + tid];
                Wc[j] = cscale(cmul(Bq[j], ilam[j]), u_pi);
            }
        }
        // ---- next hypothesis and window length ----
        if (deviated) {
            float& est = cr ? run_commit : run_skip;
            est = 0.5f * est + 0.5f * static_cast<float>(run + A - 1);
            run = 1;
            cr = !cr;
        } else {
            run += A;
        }
        // Window length: a window of W steps costs about W steps of compute
        // plus one exchange and accepts (1 - q^W) / (1 - q) steps on average
        // when the hypothesis holds step to step with probability q = 1 - 1/m
        // (m the mean run length); with the exchange worth ~0.7 step of
        // compute (measured at config 1), W ~ sqrt(1.3 m) minimises the cost
        // per accepted step, and below m = 5 single steps (the lean path) win.
        const float m = fmaxf(cr ? run_commit : run_skip, static_cast<float>(run));
        wlen = m < 5.f ? 1 : min(kWinMax, max(2, __float2int_rn(sqrtf(1.3f * m))));
        l0 += A;
        __syncthreads();  // the window's shared memory is reused by the next one
    }
    if (a.cout_h != nullptr) {  // the row's state after its last step
        float2 Bq[NPT], Cq[NPT];
        float uq;
        committed_inputs(lc, uq, Bq, Cq);
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            if (nv[j]) a.cout_h[(static_cast<size_t>(b) * H + h) * N + n] = hs[j];
            if (crank == 0 && hl == 0 && n < N) {
                a.cout_B[static_cast<size_t>(b) * N + n] = Bq[j];
                a.cout_C[static_cast<size_t>(b) * N + n] = Cq[j];
            }
        }
        if (hv && ln == 0) a.cout_u[static_cast<size_t>(b) * H + h] = u_pi;
        if (crank == 0 && tid == 0) a.cout_row[b] = make_float4(t_pi, spike, prev_r, 0.f);
    }
    rc_cluster_sync();  // no CTA leaves while a peer may still write its slots
}

template <int LANES, int NPT, typename UT>
cudaError_t launch_repair_window(const Args& a, const RcShape& rs, cudaStream_t s) {
    auto kern = rs.threads <= 384 ? cell_repair_window<LANES, NPT, UT, 384> : cell_repair_window<LANES, NPT, UT>;
    cudaError_t e;
    if (rs.cl > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    const size_t smem = win_smem_bytes<UT>(LANES * NPT, NPT, rs.threads, rs.hc);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rs.cl, a.B);
    cfg.blockDim = dim3(rs.threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = rs.cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a, rs.cl, rs.hc);
    note_launch();
    return e;
}

// ---------------------------------------------------------------------------
// 6 (commits): per row, the last committed step c(l) <= l as a max-scan of
// (g_l > 0.5 ? l : -1), and t_pi after each step; then u_pi, B_pi, C_pi are
// the inputs at max(c(l), 0) (the initial state holds step 0's u, B, C and
// t_0 - dt_init), gathered one (b, l) per CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) commit_index(Args a) {
    __shared__ int swarp[32];
    __shared__ int scarry;
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const size_t rb = static_cast<size_t>(b) * a.L;
    const float t_init = a.t[rb] - a.dt_init;
    if (tid == 0) scarry = -1;
    for (int l0 = 0; l0 < a.L; l0 += 1024) {
        const int l = l0 + tid;
        const bool valid = l < a.L;
        int x = (valid && a.gate[rb + l] > 0.5f) ? l : -1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x = max(x, y);
        }
        if (lane == 31) swarp[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int w = swarp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w = max(w, y);
            }
            swarp[lane] = w;
        }
        __syncthreads();
        const int c = max(max(x, wid > 0 ? swarp[wid - 1] : -1), scarry);
        if (valid) {
            a.cidx[rb + l] = c;
            a.commit_t[rb + l] = c < 0 ? t_init : a.t[rb + c];
        }
        __syncthreads();
        if (tid == 1023) scarry = c;
        __syncthreads();
    }
}

template <typename UT>
__global__ void commit_gather(Args a) {
    const int l = blockIdx.x, b = blockIdx.y;
    const size_t row = static_cast<size_t>(b) * a.L + l;
    const int c = max(a.cidx[row], 0);
    const size_t src = static_cast<size_t>(b) * a.L + c;
    const UT* u = static_cast<const UT*>(a.u);
    for (int h = threadIdx.x; h < a.H; h += blockDim.x) a.commit_u[row * a.H + h] = to_f32(u[src * a.H + h]);
    for (int n = threadIdx.x; n < a.N; n += blockDim.x) {
        a.commit_B[row * a.N + n] = a.Bc[src * a.N + n];
        a.commit_C[row * a.N + n] = a.Cc[src * a.N + n];
    }
}

// ---------------------------------------------------------------------------
// zoh_kernels (discretization.py:20-36) on its own: dt (M,H) -> dA, dB_bar
// (M,H,N).  One thread per output element.
// ---------------------------------------------------------------------------
__global__ void zoh_kernels_k(const float2* __restrict__ lam, const float* __restrict__ dt,
                              float2* __restrict__ dA, float2* __restrict__ dB, int64_t M, int H,
                              int N) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t HN = static_cast<int64_t>(H) * N;
    if (idx >= M * HN) return;
    const int64_t m = idx / HN;
    const int64_t hn = idx - m * HN;
    const int hh = static_cast<int>(hn / N);
    const float2 lm = lam[hn];
    float2 a_, b_;
    zoh(lm, crecip(lm), dt[m * H + hh], a_, b_);
    dA[idx] = a_;
    dB[idx] = b_;
}

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
#ifndef EACS_CHAIN_NPT
#define EACS_CHAIN_NPT 2
#endif
int lanes_for(int N, int* lanes, int* npt) {
    if (EACS_CHAIN_NPT == 4) {
        if (N <= 16) { *lanes = 4; *npt = 4; }
        else if (N <= 32) { *lanes = 8; *npt = 4; }
        else if (N <= 64) { *lanes = 16; *npt = 4; }
        else return 0;
        return 1;
    }
    if (EACS_CHAIN_NPT == 2) {
        // two chains a thread up to N = 16 (H=768 N=16: 309 Gupd/s, against 275 with
        // one and 226 with four); four for N <= 32 (H=2048 N=32: 412 against 396 with two)
        if (N <= 8) { *lanes = 4; *npt = 2; }
        else if (N <= 16) { *lanes = 8; *npt = 2; }
        else if (N <= 32) { *lanes = 8; *npt = 4; }
        else if (N <= 64) { *lanes = 32; *npt = 2; }
        else return 0;
        return 1;
    }
    if (N <= 4) { *lanes = 4; *npt = 1; }
    else if (N <= 8) { *lanes = 8; *npt = 1; }
    else if (N <= 16) { *lanes = 16; *npt = 1; }
    else if (N <= 32) { *lanes = 32; *npt = 1; }
    else if (N <= 64) { *lanes = 32; *npt = 2; }
    else return 0;
    return 1;
}

template <int LANES, int NPT, int MODE, typename UT, int CT = kThreads>
cudaError_t launch_chain(const Args& a, cudaStream_t s) {
    dim3 grid(a.ntiles, a.B);
    if (MODE != REPLAY) mark_start(s);
    cell_chain<LANES, NPT, MODE, UT, CT><<<grid, CT, 0, s>>>(a);
    if (MODE != REPLAY) mark_stop(s);
    note_launch();
    return cudaGetLastError();
}

template <int MODE, typename UT>
cudaError_t chain_by_n(const Args& a, cudaStream_t s) {
    int lanes, npt;
    lanes_for(a.N, &lanes, &npt);
    if constexpr (MODE == SPEC) {
        if (a.wide && lanes == 8 && npt == 2) return launch_chain<8, 2, MODE, UT, kWideThreads>(a, s);
        if (a.chains4 && lanes == 8 && npt == 2) return launch_chain<4, 4, MODE, UT>(a, s);
    }
#if EACS_CHAIN_NPT == 4
    if (lanes == 4) return launch_chain<4, 4, MODE, UT>(a, s);
    if (lanes == 8) return launch_chain<8, 4, MODE, UT>(a, s);
    return launch_chain<16, 4, MODE, UT>(a, s);
#elif EACS_CHAIN_NPT == 2
    if (lanes == 4) return launch_chain<4, 2, MODE, UT>(a, s);
    if (lanes == 8 && npt == 2) return launch_chain<8, 2, MODE, UT>(a, s);
    if (lanes == 8) return launch_chain<8, 4, MODE, UT>(a, s);
    return launch_chain<32, 2, MODE, UT>(a, s);
#else
    if (lanes == 4) return launch_chain<4, 1, MODE, UT>(a, s);
    if (lanes == 8) return launch_chain<8, 1, MODE, UT>(a, s);
    if (lanes == 16) return launch_chain<16, 1, MODE, UT>(a, s);
    if (npt == 1) return launch_chain<32, 1, MODE, UT>(a, s);
    return launch_chain<32, 2, MODE, UT>(a, s);
#endif
}

template <int MODE>
cudaError_t chain_dispatch(const Args& a, int dtype, cudaStream_t s) {
    if (dtype == EACS_DTYPE_F16) return chain_by_n<MODE, __half>(a, s);
    if (dtype == EACS_DTYPE_BF16) return chain_by_n<MODE, __nv_bfloat16>(a, s);
    return chain_by_n<MODE, float>(a, s);
}

template <typename UT>
cudaError_t repair_by_n(const Args& a, cudaStream_t s) {
    const RcShape rs = rc_shape(a.H, a.N, a.B);
#ifndef EACS_REPAIR_WINDOW
#define EACS_REPAIR_WINDOW 1
#endif
    if (EACS_REPAIR_WINDOW && rs.cl > 0 && rs.lanes <= 8 && a.gate_mode == 0 && a.commit_h == nullptr &&
        a.gck_h == nullptr &&
        win_smem_bytes<UT>(rs.lanes * rs.npt, rs.npt, rs.threads, rs.hc) <= 200u * 1024u) {
        // hard gate without per-step recording: the windowed speculative repair
        if (rs.lanes == 4 && rs.npt == 1) return launch_repair_window<4, 1, UT>(a, rs, s);
        if (rs.lanes == 4 && rs.npt == 2) return launch_repair_window<4, 2, UT>(a, rs, s);
        if (rs.lanes == 4) return launch_repair_window<4, 4, UT>(a, rs, s);
        return launch_repair_window<8, 4, UT>(a, rs, s);
    }
    if (rs.cl > 0) {
        if (rs.lanes == 4 && rs.npt == 1) return launch_repair_cluster<4, 1, UT>(a, rs, s);
        if (rs.lanes == 4 && rs.npt == 2) return launch_repair_cluster<4, 2, UT>(a, rs, s);
        if (rs.lanes == 4) return launch_repair_cluster<4, 4, UT>(a, rs, s);
        if (rs.lanes == 8) return launch_repair_cluster<8, 4, UT>(a, rs, s);
        return launch_repair_cluster<16, 4, UT>(a, rs, s);
    }
    int lanes, npt;
    lanes_for(a.N, &lanes, &npt);
    while (npt > 1 && lanes < 32) {  // the repair pass keeps one chain per lane
        lanes *= 2;
        npt /= 2;
    }
    if (lanes == 4) cell_repair<4, 1, UT><<<a.B, kRepair, 0, s>>>(a);
    else if (lanes == 8) cell_repair<8, 1, UT><<<a.B, kRepair, 0, s>>>(a);
    else if (lanes == 16) cell_repair<16, 1, UT><<<a.B, kRepair, 0, s>>>(a);
    else if (npt == 1) cell_repair<32, 1, UT><<<a.B, kRepair, 0, s>>>(a);
    else cell_repair<32, 2, UT><<<a.B, kRepair, 0, s>>>(a);
    note_launch();
    return cudaGetLastError();
}

cudaError_t repair_dispatch(const Args& a, int dtype, cudaStream_t s) {
    if (dtype == EACS_DTYPE_F16) return repair_by_n<__half>(a, s);
    if (dtype == EACS_DTYPE_BF16) return repair_by_n<__nv_bfloat16>(a, s);
    return repair_by_n<float>(a, s);
}

int tiles_for(int H, int N) {
    int lanes, npt;
    lanes_for(N, &lanes, &npt);
    const int HT = kThreads / lanes;
    return (H + HT - 1) / HT;
}

int sm_count() {
    static int cache[64];  // per device; a repeated query writes the same value
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        cache[dev] = n;
    }
    return cache[dev];
}

// Tiles of the wide speculative pass, or 0 where the four-warp layout is as
// good: the wide one runs when its B x tiles CTAs fit one per SM and the
// four-warp CTAs would put three or more on some SM (12+ warps against 11).
// Its tiles never outnumber tiles_for's, so the workspace sized by that holds
// its partial sums.
int wide_tiles(int B, int H, int N) {
    int lanes, npt;
    lanes_for(N, &lanes, &npt);
    if (lanes != 8 || npt != 2) return 0;
    const int sms = sm_count();
    if (sms <= 0) return 0;
    const int64_t nt = (H + kWideThreads / 8 - 1) / (kWideThreads / 8);
    const int64_t narrow = static_cast<int64_t>(B) * tiles_for(H, N);
    if (static_cast<int64_t>(B) * nt > sms || narrow <= 2LL * sms) return 0;
    return static_cast<int>(nt);
}

// Tiles of the four-chains-a-thread speculative pass for k cells of this
// shape run side by side, or 0: it runs when the k cells' four-warp CTAs of
// two chains a thread are more than the SMs hold at once (four each at 128
// registers), so a thin second wave would follow, and the four-chain CTAs
// (half as many) fit in one.  A lone cell keeps its own layout: halving its
// CTAs would leave SMs idle.
int side_by_side_tiles(int k, int B, int H, int N) {
    int lanes, npt;
    lanes_for(N, &lanes, &npt);
    if (k <= 1 || lanes != 8 || npt != 2) return 0;
    const int sms = sm_count();
    if (sms <= 0) return 0;
    const int64_t t4 = (H + kThreads / 4 - 1) / (kThreads / 4);
    const int64_t cap = 4LL * sms;
    const int64_t two = static_cast<int64_t>(k) * B * tiles_for(H, N);
    const int64_t four = static_cast<int64_t>(k) * B * t4;
    if (two <= cap || four > cap) return 0;
    return static_cast<int>(t4);
}

size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct WsLayout {
    size_t part, row, hpi, upi, total, cidx, total_commits;
};
WsLayout ws_layout(int64_t B, int64_t L, int64_t H, int64_t N) {
    WsLayout w;
    const int64_t nt = tiles_for(static_cast<int>(H), static_cast<int>(N));
    w.part = 0;
    w.row = w.part + align_up(static_cast<size_t>(B * nt * L) * sizeof(float2));
    w.hpi = w.row + align_up(static_cast<size_t>(B) * sizeof(int4));
    w.upi = w.hpi + align_up(static_cast<size_t>(B * H * N) * sizeof(float2));
    w.total = w.upi + align_up(static_cast<size_t>(B * H) * sizeof(float));
    // commit recording also keeps the last committed step per (b, l)
    w.cidx = w.total;
    w.total_commits = w.cidx + align_up(static_cast<size_t>(B * L) * sizeof(int));
    return w;
}

int check_shape(const char* fn, int64_t B, int64_t L, int64_t H, int64_t N, int dtype) {
    if (B < 0 || L < 0 || H < 0 || N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)N);
    if (B > 65535) return fail(EACS_ERR_UNSUPPORTED, "%s: B=%lld > 65535", fn, (long long)B);
    if (L > (1LL << 30) || H > (1LL << 24)) return fail(EACS_ERR_UNSUPPORTED, "%s: L or H too large", fn);
    if (dtype != EACS_DTYPE_F32 && dtype != EACS_DTYPE_F16 && dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, dtype);
    return EACS_OK;
}

}  // namespace

size_t cell_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0 || N > 64) return 0;
    return ws_layout(B, L, H, N).total;
}

bool cell_resumable(int64_t H, int64_t N) {
    // both repair passes (cluster and one-CTA) take and return a carried state
    return H > 0 && N > 0 && N <= 64 && H <= (1LL << 24);
}

size_t cell_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0 || N > 64) return 0;
    return ws_layout(B, L, H, N).total_commits;
}

int cell_fwd(const CellCall& c, cudaStream_t stream) {
    const bool commits = c.commit_h != nullptr;
    const char* fn = commits ? "eacs_cell_commits" : "eacs_cell_fwd";
    int rc = check_shape(fn, c.B, c.L, c.H, c.N, c.u_dtype);
    if (rc) return rc;
    if (c.B == 0 || c.L == 0 || c.H == 0) return EACS_OK;
    if (c.N == 0) return fail(EACS_ERR_INVALID, "%s: N must be positive", fn);
    if (!c.lam || !c.log_dt || !c.u || !c.Bc || !c.Cc || !c.t || !c.D || !c.mean || !c.var ||
        !c.y || !c.gate || !c.resid)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (c.gate_mode != 0 && c.gate_mode != 1)
        return fail(EACS_ERR_INVALID, "%s: gate_mode must be 0 (hard) or 1 (soft)", fn);
    if (c.gate_mode == 1 && c.robust)
        return fail(EACS_ERR_INVALID, "%s: robust_guard applies to the hard gate only", fn);
    if (commits && (!c.commit_t || !c.commit_u || !c.commit_B || !c.commit_C))
        return fail(EACS_ERR_INVALID, "%s: null commit output", fn);
    if (commits && c.gate_mode != 0)
        return fail(EACS_ERR_INVALID, "%s: commits are recorded for the hard gate only", fn);
    const bool ckpt = c.ck_h != nullptr;
    if (ckpt && (!c.ck_u || !c.ck_row || !c.ck_bc || c.ck_K <= 0 || (c.ck_K & (c.ck_K - 1)) || c.ck_nK <= 0))
        return fail(EACS_ERR_INVALID, "%s: incomplete checkpoint layout (K a power of two)", fn);
    if (ckpt && (commits || rc_shape(static_cast<int>(c.H), static_cast<int>(c.N), static_cast<int>(c.B)).cl == 0))
        return fail(EACS_ERR_UNSUPPORTED, "%s: checkpoints need the cluster repair shape and no commits", fn);
    const bool carry = c.cin_h != nullptr || c.cout_h != nullptr;
    if (carry && !cell_resumable(c.H, c.N))
        return fail(EACS_ERR_UNSUPPORTED, "%s: H=%lld N=%lld rows cannot be resumed", fn, (long long)c.H,
                    (long long)c.N);
    if (c.cout_h != nullptr && (c.L % EACS_CHAIN_U) != 0)
        return fail(EACS_ERR_INVALID, "%s: a chunk with a carried-out state needs L %% %d == 0", fn,
                    EACS_CHAIN_U);
    const WsLayout w = ws_layout(c.B, c.L, c.H, c.N);
    const size_t need = commits ? w.total_commits : w.total;
    if (!c.workspace || c.workspace_bytes < need)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, need,
                    c.workspace_bytes);
    Args a{};
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
    a.robust = c.robust ? 1 : 0;
    a.robust_k = c.robust_k;
    a.spike_ratio = c.spike_ratio;
    a.eps_lo = c.eps * c.eps_factor;
    a.gate_mode = c.gate_mode;
    a.Tp = c.temperature > 1e-4f ? c.temperature : 1e-4f;
    a.y = c.y;
    a.gate = c.gate;
    a.resid = c.resid;
    a.stats = static_cast<float2*>(c.stats);
    char* ws = static_cast<char*>(c.workspace);
    a.part = reinterpret_cast<float2*>(ws + w.part);
    a.row = reinterpret_cast<int4*>(ws + w.row);
    a.hpi = reinterpret_cast<float2*>(ws + w.hpi);
    a.upi = reinterpret_cast<float*>(ws + w.upi);
    if (commits) {
        a.commit_h = static_cast<float2*>(c.commit_h);
        a.commit_t = c.commit_t;
        a.commit_u = c.commit_u;
        a.commit_B = static_cast<float2*>(c.commit_B);
        a.commit_C = static_cast<float2*>(c.commit_C);
        a.cidx = reinterpret_cast<int*>(ws + w.cidx);
    }
    a.cin_h = static_cast<const float2*>(c.cin_h);
    a.cin_u = c.cin_u;
    a.cin_B = static_cast<const float2*>(c.cin_B);
    a.cin_C = static_cast<const float2*>(c.cin_C);
    a.cin_row = static_cast<const float4*>(c.cin_row);
    a.cout_h = static_cast<float2*>(c.cout_h);
    a.cout_u = c.cout_u;
    a.cout_B = static_cast<float2*>(c.cout_B);
    a.cout_C = static_cast<float2*>(c.cout_C);
    a.cout_row = static_cast<float4*>(c.cout_row);
    if (ckpt) {
        a.gck_h = static_cast<float2*>(c.ck_h);
        a.gck_u = c.ck_u;
        a.gck_row = static_cast<float4*>(c.ck_row);
        a.gck_bc = static_cast<float2*>(c.ck_bc);
        a.gK = c.ck_K;
        a.gnK = c.ck_nK;
        a.gKlog = 0;
        while ((1 << a.gKlog) < a.gK) ++a.gKlog;
    }
    a.B = static_cast<int>(c.B);
    a.L = static_cast<int>(c.L);
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    a.ntiles = tiles_for(a.H, a.N);

    cudaError_t e;
    if (c.gate_mode == 0) {
        if (!commits && !ckpt) {
            const int st4 = side_by_side_tiles(c.side_by_side, a.B, a.H, a.N);
            const int wt = c.side_by_side > 1 ? 0 : wide_tiles(a.B, a.H, a.N);
            if (st4 > 0) {
                a.chains4 = 1;
                a.ntiles = st4;
            } else if (wt > 0) {
                a.wide = 1;
                a.ntiles = wt;  // partial sums per row for cell_resid
            }
        }
        e = commits ? chain_dispatch<SPEC_COMMITS>(a, c.u_dtype, stream)
            : ckpt  ? chain_dispatch<SPEC_CKPT>(a, c.u_dtype, stream)
                    : chain_dispatch<SPEC>(a, c.u_dtype, stream);
        if (e != cudaSuccess) return cuda_check(e, fn);
        cell_resid<<<dim3((a.L + 255) / 256, a.B), 256, 0, stream>>>(a);
        note_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);
        cell_gates<<<a.B, 1024, 0, stream>>>(a);
        note_launch();
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);
    } else {
        // soft gate: the state is a continuous blend, so run the exact cell from l = 0
        if ((e = cudaMemsetAsync(a.row, 0, static_cast<size_t>(a.B) * sizeof(int4), stream)) != cudaSuccess)
            return cuda_check(e, fn);
    }
    a.wide = 0;  // the replay pass covers the channels in four-warp tiles
    a.chains4 = 0;
    a.ntiles = tiles_for(a.H, a.N);
    if ((e = chain_dispatch<REPLAY>(a, c.u_dtype, stream)) != cudaSuccess) return cuda_check(e, fn);
    if ((e = repair_dispatch(a, c.u_dtype, stream)) != cudaSuccess) return cuda_check(e, fn);
    if (commits) {
        commit_index<<<a.B, 1024, 0, stream>>>(a);
        const dim3 grid(a.L, a.B);
        if (c.u_dtype == EACS_DTYPE_F16) commit_gather<__half><<<grid, 256, 0, stream>>>(a);
        else if (c.u_dtype == EACS_DTYPE_BF16) commit_gather<__nv_bfloat16><<<grid, 256, 0, stream>>>(a);
        else commit_gather<float><<<grid, 256, 0, stream>>>(a);
        note_launch(2);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);
    }
    return EACS_OK;
}

size_t ssm_ckpt_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0 || N > 64) return 0;
    return static_cast<size_t>(B) * static_cast<size_t>((L + kSsmCk - 1) / kSsmCk) *
           static_cast<size_t>(H) * static_cast<size_t>(N) * sizeof(float2);
}

int ssm_fwd(const void* lam, const float* log_dt, const float* t, const void* Bc, const void* Cc,
            const void* u, int u_dtype, const float* D, float* y, int64_t B, int64_t L, int64_t H,
            int64_t N, float dt_min, float dt_max, void* ckpt, size_t ckpt_bytes,
            cudaStream_t stream) {
    const char* fn = ckpt ? "eacs_ssm_train_fwd" : "eacs_ssm_fwd";
    int rc = check_shape(fn, B, L, H, N, u_dtype);
    if (rc) return rc;
    if (B == 0 || L == 0 || H == 0) return EACS_OK;
    if (N == 0) return fail(EACS_ERR_INVALID, "%s: N must be positive", fn);
    if (!lam || !log_dt || !t || !Bc || !Cc || !u || !D || !y)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (ckpt && ckpt_bytes < ssm_ckpt_size(B, L, H, N))
        return fail(EACS_ERR_WORKSPACE, "%s: checkpoint buffer of %zu bytes needed, %zu given", fn,
                    ssm_ckpt_size(B, L, H, N), ckpt_bytes);
    Args a{};
    a.ck = static_cast<float2*>(ckpt);
    a.nK = static_cast<int>((L + kSsmCk - 1) / kSsmCk);
    a.lam = static_cast<const float2*>(lam);
    a.log_dt = log_dt;
    a.u = u;
    a.Bc = static_cast<const float2*>(Bc);
    a.Cc = static_cast<const float2*>(Cc);
    a.t = t;
    a.D = D;
    a.dt_min = dt_min;
    a.dt_max = dt_max;
    a.y = y;
    a.B = static_cast<int>(B);
    a.L = static_cast<int>(L);
    a.H = static_cast<int>(H);
    a.N = static_cast<int>(N);
    a.ntiles = tiles_for(a.H, a.N);
    cudaError_t e = chain_dispatch<UNGATED>(a, u_dtype, stream);
    return cuda_check(e, fn);
}

cudaError_t cell_read_status(int* out, cudaStream_t stream) { return read_clear_status(out, stream); }

// Failure-path check: an mbarrier (count 1) that nothing arrives at, waited on
// with the bounded waits the repair and training passes use, at a small poll
// limit.  Both waits give up, record EACS_ERR_TIMEOUT and return.
__global__ void wait_selftest_k(uint32_t polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool a = mbar_wait(&bar, 0, polls);
        const bool b = mbar_wait_row(&bar, 0, polls);
        if (a || b) set_status(EACS_ERR_INVALID);  // a phase nothing completes cannot complete
    }
}

int wait_selftest(int polls, cudaStream_t stream) {
    if (polls < 1 || polls > 65536)
        return fail(EACS_ERR_INVALID, "eacs_wait_selftest: polls %d outside 1..65536", polls);
    wait_selftest_k<<<1, 32, 0, stream>>>(static_cast<uint32_t>(polls));
    note_launch();
    return cuda_check(cudaGetLastError(), "eacs_wait_selftest");
}

int zoh_kernels(const void* lam, const float* dt, void* dA, void* dBbar, int64_t M, int64_t H,
                int64_t N, cudaStream_t stream) {
    const char* fn = "eacs_zoh_kernels";
    if (M < 0 || H < 0 || N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    const int64_t n = M * H * N;
    if (n == 0) return EACS_OK;
    if (!lam || !dt || !dA || !dBbar) return fail(EACS_ERR_INVALID, "%s: null pointer", fn);
    if (H > (1LL << 30) || N > (1LL << 30) || (n + 255) / 256 > 0x7fffffffLL)
        return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    zoh_kernels_k<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        static_cast<const float2*>(lam), dt, static_cast<float2*>(dA), static_cast<float2*>(dBbar), M,
        static_cast<int>(H), static_cast<int>(N));
    note_launch();
    return cuda_check(cudaGetLastError(), fn);
}

// ---------------------------------------------------------------------------
// Gated cell with library-owned scratch, for callers that cannot allocate
// device memory: a host that binds only this C ABI and has no device
// allocator of its own, or a process whose device memory belongs to another
// allocator (a framework's pool) where a stray cudaMalloc -- which also
// synchronises the device -- is not allowed.  The scratch is this file-scope
// array: every GPU that loads the library holds EACS_NOALLOC_SCRATCH_BYTES of
// it until the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_cell_scratch[EACS_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
}  // namespace

int cell_fwd_noalloc(const CellCall& c, cudaStream_t stream) {
    const char* fn = "eacs_cell_fwd_noalloc";
    const size_t need = cell_workspace_size(c.B, c.L, c.H, c.N);
    if (need > EACS_NOALLOC_SCRATCH_BYTES)
        return fail(EACS_ERR_WORKSPACE,
                    "%s: B=%lld L=%lld H=%lld N=%lld needs %zu bytes of scratch, more than the "
                    "%zu-byte static array; use eacs_cell_fwd with a caller workspace",
                    fn, (long long)c.B, (long long)c.L, (long long)c.H, (long long)c.N, need,
                    static_cast<size_t>(EACS_NOALLOC_SCRATCH_BYTES));
    int dev = 0;
    int rc = cuda_check(cudaGetDevice(&dev), fn);
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices) return fail(EACS_ERR_UNSUPPORTED, "%s: device %d", fn, dev);
    void* scratch = nullptr;
    {
        // Set-up, once per device with that device current: the host-side name
        // g_cell_scratch is a stand-in, not a device address.
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            rc = cuda_check(cudaGetSymbolAddress(&p, g_cell_scratch), fn);
            if (rc) return rc;
            g_scratch_addr[dev] = p;
        }
        scratch = g_scratch_addr[dev];
    }
    CellCall c2 = c;
    c2.workspace = scratch;
    c2.workspace_bytes = EACS_NOALLOC_SCRATCH_BYTES;
    return cell_fwd(c2, stream);
}

}  // namespace eacs
