// ssm_train.cu -- backward of the fused ungated continuous SSM core (sm_100a).
//
// Reference: cst_ssm/modules/continuous_ssm.py:44-55 differentiated by
// autograd through effective_dt and zoh_discretize (ops/discretization.py:
// 20-82), the scan (ops/scan.py:64-78, whose CUDA backward is
// ops/csrc/eacs_scan_cuda.cu:40-60) and the readout.  Per chain (b, h, n),
// with w_l the adjoint of h_l and z = lam*dte, dA = e^z, dB_bar = (e^z-1)/lam,
// q = dB_bar B:
//   w_l    = conj(dA_{l+1}) w_{l+1} + gy_l conj(C_l)
//   du_l   = sum_n Re(w_l conj(q_l)) + D gy_l
//   dB_l  += u_l w_l conj(dB_bar_l)                      (sum over h)
//   dC_l  += gy_l conj(h_l)                              (sum over h)
//   a_z    = w_l conj(dA_l (h_{l-1} + u_l B_l / lam))    (adjoint of z)
//   dlam  += dte a_z - conj(1/lam) u_l w_l conj(q_l)
//   ddte_l = sum_n Re(conj(a_z) lam), masked where the clamp of dt*e^log_dt
//            to [dt_min, dt_max] is active, then to log_dt and to the
//            timestamp differences (dt_l = max(t_l - t_{l-1}, 0), dt_0 = dt_1).
// The same vector-Jacobian product is written out in double precision in the
// CPU oracle (oracle/eacs_oracle.c, eacs_oracle_ssm_bwd), which is checked
// against the reference's autograd.
//
// States come from checkpoints every kSsmCk steps written by the forward
// chain kernel (eacs_ssm_train_fwd).  One CTA per (row, tile of channels)
// walks the chunks from last to first: it recomputes the chunk forward from
// its checkpoint into shared memory (h_{l-1}, dA, dB_bar per chain and step),
// then runs the chunk in reverse, while the next chunk's inputs load into
// registers.  Sums over n (du, ddte) use a transposed shuffle butterfly
// within a channel group; each chain's dB, dC terms go to its own shared
// slot and the chunk's output pass sums them over the CTA's channels, one
// partial per (row, tile, step) in the workspace.  Post kernels add the tile
// and row partials in a fixed order (deterministic).
#include <algorithm>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kBT = 128;     // backward CTA
constexpr int kK = kSsmCk;   // steps per recomputed chunk
constexpr int kU = 2;        // steps per reduction group
static_assert(kK % kU == 0, "chunk must hold whole step groups");

struct SArgs {
    const float2* lam;
    const float* log_dt;
    const float* t;
    const float2* Bc;
    const float2* Cc;
    const void* u;
    const float* D;
    const float* gy;
    const float2* ck;  // [B][nK][H][N]
    float* du;         // (B,L,H)
    float2* dBc;       // (B,L,N)
    float2* dCc;
    float* dt;         // (B,L) gradient of the timestamps
    float2* dlam;      // (H,N)
    float* dlog;       // (H)
    float* dD;         // (H)
    // workspace
    float4* part;      // [B][ntiles][L][N] (dB, dC) summed over the tile's channels
    float* pt;         // [B][ntiles][L]    d(dt_l) summed over the tile's channels
    float2* plam;      // [B][H][N]
    float* plog;       // [B][H]
    float* pD;         // [B][H]
    float dt_min, dt_max;
    int B, L, H, N, ntiles, nK;
};

template <int LANES, int NPT>
struct BwdSmem {
    static constexpr int HT = kBT / LANES;
    static constexpr int NP = LANES * NPT;
    static constexpr size_t kAB = static_cast<size_t>(kK) * NPT * kBT * sizeof(float4);
    static constexpr size_t kH = static_cast<size_t>(kK) * NPT * kBT * sizeof(float2);
    static constexpr size_t kBC = 2ull * kK * NP * sizeof(float2);
    static constexpr size_t kRow = 4ull * kK * HT * sizeof(float) + kK * sizeof(float);
    static constexpr size_t bytes = kAB + kH + kBC + kRow;
};

template <int LANES, int NPT, typename UT>
__global__ void __launch_bounds__(kBT, NPT == 1 ? 5 : 4) ssm_bwd_chain(SArgs a) {
    using SM = BwdSmem<LANES, NPT>;
    constexpr int HT = SM::HT, NP = SM::NP, U = kU;
    constexpr int VN = 2 * U;                      // per group: du and ddte of U steps (sum over n)
    constexpr int PB = (kK * NP + kBT - 1) / kBT;  // prefetched B, C entries per thread
    constexpr int PU = (kK * HT + kBT - 1) / kBT;  // prefetched u, gy entries per thread
    using SN = FoldShape<VN, LANES / 2, 1>;

    extern __shared__ __align__(16) unsigned char smem[];
    // [kK][NPT][kBT]: (dA, dB_bar) from the recompute; the reverse step
    // overwrites its own slot with (u w conj(dB_bar), gy conj(h)), which the
    // chunk's output pass then sums over the CTA's channels
    float4* sAB = reinterpret_cast<float4*>(smem);
    float2* sH = reinterpret_cast<float2*>(smem + SM::kAB);            // [kK][NPT][kBT] h_{l-1}
    float2* sB = reinterpret_cast<float2*>(smem + SM::kAB + SM::kH);   // [kK][NP]
    float2* sC = sB + kK * NP;                                         // [kK][NP]
    float* su = reinterpret_cast<float*>(sC + kK * NP);                // [kK][HT]
    float* sg = su + kK * HT;                                          // [kK][HT] gy
    float* sdu = sg + kK * HT;                                         // [kK][HT]
    float* sdt = sdu + kK * HT;                                        // [kK][HT]
    float* sdel = sdt + kK * HT;                                       // [kK] dt before the clamp

    const int tid = threadIdx.x;
    const int ln = tid % LANES, hl = tid / LANES;
    const int tile = blockIdx.x, b = blockIdx.y;
    const int h0 = tile * HT, h = h0 + hl;
    const bool hv = h < a.H;
    const int L = a.L, H = a.H, N = a.N;
    const UT* u = static_cast<const UT*>(a.u);
    const size_t rowL = static_cast<size_t>(b) * L;

    float2 lam[NPT], ilam[NPT], s[NPT], acc1[NPT], acc2[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        s[j] = acc1[j] = acc2[j] = make_float2(0.f, 0.f);
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float Dh = hv ? a.D[h] : 0.f;
    const float dt0 = L > 1 ? fmaxf(a.t[rowL + 1] - a.t[rowL], 0.f) : 0.f;
    const int heldN = SN::held(ln);
    const bool wN = SN::writer(ln);
    float glog = 0.f, gD = 0.f;

    // Registers holding the next chunk's inputs, loaded while the current
    // chunk runs; steps past L and padded chains read zeros.
    float2 pB[PB], pC[PB], pck[NPT];
    UT pu[PU];
    float pg[PU], pt1 = 0.f, pt0 = 0.f;  // raw loads; converted when staged
    const UT uzero = static_cast<UT>(0.f);
    auto prefetch = [&](int k) {
        const int l0 = k * kK;
        const int steps = min(kK, L - l0);
#pragma unroll
        for (int r = 0; r < PB; ++r) {
            const int idx = tid + r * kBT;
            const int i = idx / NP, n = idx % NP;
            const bool ok = idx < kK * NP && i < steps && n < N;
            const size_t o = (rowL + l0 + i) * N + n;
            pB[r] = ok ? a.Bc[o] : make_float2(0.f, 0.f);
            pC[r] = ok ? a.Cc[o] : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int r = 0; r < PU; ++r) {
            const int idx = tid + r * kBT;
            const int i = idx / HT, c = idx % HT;
            const bool ok = idx < kK * HT && i < steps && h0 + c < H;
            const size_t o = (rowL + l0 + i) * H + h0 + c;
            pu[r] = ok ? u[o] : uzero;
            pg[r] = ok ? a.gy[o] : 0.f;
        }
        if (tid < kK && tid < steps && l0 + tid > 0) {
            pt1 = a.t[rowL + l0 + tid];
            pt0 = a.t[rowL + l0 + tid - 1];
        }
        const size_t ko = (static_cast<size_t>(b) * a.nK + k) * H + (hv ? h : 0);
#pragma unroll
        for (int j = 0; j < NPT; ++j)
            pck[j] = nv[j] ? a.ck[ko * N + ln + LANES * j] : make_float2(0.f, 0.f);
    };
    // Chunk outputs: dB, dC summed over the CTA's channels, du, and the
    // channels' sum of d(dt_l) per step.
    auto emit = [&](int k) {
        const int l0 = k * kK;
        const int steps = min(kK, L - l0);
        for (int idx = tid; idx < steps * N; idx += kBT) {
            const int i = idx / N, n = idx % N;
            const float4* src = sAB + (i * NPT + n / LANES) * kBT + n % LANES;
            float4 acc = src[0];
#pragma unroll
            for (int c = 1; c < HT; ++c) {
                const float4 v = src[c * LANES];
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            a.part[((static_cast<size_t>(b) * a.ntiles + tile) * L + l0 + i) * N + n] = acc;
        }
        for (int idx = tid; idx < steps * HT; idx += kBT) {
            const int i = idx / HT, c = idx % HT;
            if (h0 + c < H) a.du[(rowL + l0 + i) * H + h0 + c] = sdu[idx];
        }
        if (tid < steps) {
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < HT; ++c) sum += sdt[tid * HT + c];
            a.pt[(static_cast<size_t>(b) * a.ntiles + tile) * L + l0 + tid] = sum;
        }
    };

    prefetch(a.nK - 1);
    for (int k = a.nK - 1; k >= 0; --k) {
        __syncthreads();  // the reverse pass of chunk k+1 is done everywhere
        if (k + 1 < a.nK) emit(k + 1);
        // ---- stage chunk k from the prefetch registers ----
#pragma unroll
        for (int r = 0; r < PB; ++r) {
            const int idx = tid + r * kBT;
            if (idx < kK * NP) {
                sB[idx] = pB[r];
                sC[idx] = pC[r];
            }
        }
#pragma unroll
        for (int r = 0; r < PU; ++r) {
            const int idx = tid + r * kBT;
            if (idx < kK * HT) {
                su[idx] = to_f32(pu[r]);
                sg[idx] = pg[r];
            }
        }
        if (tid < kK) {
            const int l = k * kK + tid;
            sdel[tid] = l >= L ? 0.f : (l == 0 ? dt0 : fmaxf(pt1 - pt0, 0.f));
        }
        float2 hs[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) hs[j] = pck[j];
        __syncthreads();
        if (k > 0) prefetch(k - 1);

        // ---- forward recompute of the chunk from its checkpoint ----
#pragma unroll
        for (int i = 0; i < kK; ++i) {
            const float ul = su[i * HT + hl];
            const float dte = eff_dt(sdel[i], scale, a.dt_min, a.dt_max);
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                float2 dA, dB;
                zoh(lam[j], ilam[j], dte, dA, dB);
                const int si = (i * NPT + j) * kBT + tid;
                sAB[si] = make_float4(dA.x, dA.y, dB.x, dB.y);
                sH[si] = hs[j];
                const float2 q = cmul(dB, sB[i * NP + ln + LANES * j]);
                const float2 P = cmul(dA, hs[j]);
                hs[j] = make_float2(fmaf(q.x, ul, P.x), fmaf(q.y, ul, P.y));
            }
        }

        // ---- reverse over the chunk; hs holds h of its last step ----
#pragma unroll 1
        for (int g = kK / U - 1; g >= 0; --g) {
            const int i0 = g * U;
            float vn[VN];
#pragma unroll
            for (int uu = U - 1; uu >= 0; --uu) {
                const int i = i0 + uu;
                const float ul = su[i * HT + hl];
                const float yb = sg[i * HT + hl];
                const float dte = eff_dt(sdel[i], scale, a.dt_min, a.dt_max);
                float dun = 0.f, dzn = 0.f;
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const int n = ln + LANES * j;
                    const int si = (i * NPT + j) * kBT + tid;
                    const float4 ab = sAB[si];
                    const float2 dA = make_float2(ab.x, ab.y), dB = make_float2(ab.z, ab.w);
                    const float2 hp = sH[si];
                    const float2 Bl = sB[i * NP + n], Cl = sC[i * NP + n];
                    // adjoint of h_l: carried + readout
                    const float2 w = make_float2(fmaf(yb, Cl.x, s[j].x), fmaf(-yb, Cl.y, s[j].y));
                    const float2 q = cmul(dB, Bl);
                    const float2 c = make_float2(w.x * q.x + w.y * q.y, w.y * q.x - w.x * q.y);  // w conj(q)
                    dun += c.x;
                    acc1[j] = make_float2(fmaf(ul, c.x, acc1[j].x), fmaf(ul, c.y, acc1[j].y));
                    const float2 kb = cmul(Bl, ilam[j]);
                    const float2 m = make_float2(fmaf(ul, kb.x, hp.x), fmaf(ul, kb.y, hp.y));
                    const float2 dm = cmul(dA, m);
                    const float2 az = make_float2(w.x * dm.x + w.y * dm.y, w.y * dm.x - w.x * dm.y);  // w conj(dm)
                    acc2[j] = make_float2(fmaf(dte, az.x, acc2[j].x), fmaf(dte, az.y, acc2[j].y));
                    dzn = fmaf(az.x, lam[j].x, fmaf(az.y, lam[j].y, dzn));
                    const float2 uw = cscale(w, ul);
                    // (u w conj(dB_bar), gy conj(h_l)) into this chain's slot
                    sAB[si] = make_float4(uw.x * dB.x + uw.y * dB.y, uw.y * dB.x - uw.x * dB.y,
                                          yb * hs[j].x, -yb * hs[j].y);
                    s[j] = make_float2(dA.x * w.x + dA.y * w.y, dA.x * w.y - dA.y * w.x);  // conj(dA) w
                    hs[j] = hp;
                }
                vn[uu] = dun;
                vn[U + uu] = dzn;
                gD = fmaf(yb, ul, gD);
            }
            // sums over n: du and ddte per (step, channel)
            Fold<VN, LANES / 2, 1>::run(vn, ln);
            if (wN) {
#pragma unroll
                for (int r = 0; r < SN::kRem; ++r) {
                    const int orig = heldN + r;
                    const int i = i0 + (orig % U);
                    if (orig < U) {
                        sdu[i * HT + hl] = vn[r] + Dh * sg[i * HT + hl];
                    } else {
                        const float v = sdel[i] * scale;
                        const float drb = (v >= a.dt_min && v <= a.dt_max) ? vn[r] : 0.f;
                        glog = fmaf(drb, v, glog);
                        sdt[i * HT + hl] = drb * scale;
                    }
                }
            }
        }
    }
    __syncthreads();
    emit(0);
    // ---- per-row parameter partials ----
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) glog += __shfl_xor_sync(0xffffffffu, glog, o);
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        if (!nv[j]) continue;
        // dlam = sum dte a_z - conj(1/lam) sum u w conj(q)
        const float2 cil = make_float2(ilam[j].x, -ilam[j].y);
        const float2 t1 = cmul(cil, acc1[j]);
        a.plam[(static_cast<size_t>(b) * H + h) * N + ln + LANES * j] =
            make_float2(acc2[j].x - t1.x, acc2[j].y - t1.y);
    }
    if (hv && ln == 0) {
        a.plog[static_cast<size_t>(b) * H + h] = glog;
        a.pD[static_cast<size_t>(b) * H + h] = gD;
    }
}

// dB, dC: sum of the tile partials.
__global__ void ssm_post_bc(SArgs a) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t LN = static_cast<int64_t>(a.L) * a.N;
    if (idx >= a.B * LN) return;
    const int64_t b = idx / LN, r = idx - b * LN;
    const float4* p = a.part + b * a.ntiles * LN + r;
    float4 acc = p[0];
    for (int k = 1; k < a.ntiles; ++k) {
        const float4 v = p[k * LN];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    a.dBc[idx] = make_float2(acc.x, acc.y);
    a.dCc[idx] = make_float2(acc.z, acc.w);
}

// gradient flowing into the timestamp difference d_l = t_l - t_{l-1} (l >= 1):
// the clamp_min(0) mask times the step's d(dt), plus step 0's (dt_0 = dt_1)
__device__ float diff_grad(const SArgs& a, int b, int l) {
    if (l < 1 || l >= a.L) return 0.f;
    const float* tb = a.t + static_cast<size_t>(b) * a.L;
    if (!(tb[l] - tb[l - 1] >= 0.f)) return 0.f;
    const float* p = a.pt + static_cast<size_t>(b) * a.ntiles * a.L;
    float g = 0.f;
    for (int k = 0; k < a.ntiles; ++k) g += p[static_cast<size_t>(k) * a.L + l];
    if (l == 1) {
        float g0 = 0.f;
        for (int k = 0; k < a.ntiles; ++k) g0 += p[static_cast<size_t>(k) * a.L];
        g += g0;
    }
    return g;
}

__global__ void ssm_post_dt(SArgs a) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(a.B) * a.L) return;
    const int b = static_cast<int>(idx / a.L), l = static_cast<int>(idx % a.L);
    a.dt[idx] = diff_grad(a, b, l) - diff_grad(a, b, l + 1);
}

// dlam, dlog_dt, dD: sum of the row partials.
__global__ void ssm_post_params(SArgs a) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t HN = static_cast<int64_t>(a.H) * a.N;
    if (idx < HN) {
        float2 acc = make_float2(0.f, 0.f);
        for (int b = 0; b < a.B; ++b) acc = cadd(acc, a.plam[b * HN + idx]);
        a.dlam[idx] = acc;
    }
    if (idx < a.H) {
        float s1 = 0.f, s2 = 0.f;
        for (int b = 0; b < a.B; ++b) {
            s1 += a.plog[static_cast<int64_t>(b) * a.H + idx];
            s2 += a.pD[static_cast<int64_t>(b) * a.H + idx];
        }
        a.dlog[idx] = s1;
        a.dD[idx] = s2;
    }
}

#ifndef EACS_SSMBWD_NPT
#define EACS_SSMBWD_NPT 2
#endif
// Thread layout of the backward: LANES threads per channel, NPT chains each.
void bwd_shape(int N, int* lanes, int* npt) {
    *npt = EACS_SSMBWD_NPT;
    if (EACS_SSMBWD_NPT == 1) {
        *lanes = N <= 4 ? 4 : N <= 8 ? 8 : N <= 16 ? 16 : 32;
        if (N > 32) *npt = 2;
    } else {
        *lanes = N <= 8 ? 4 : N <= 16 ? 8 : N <= 32 ? 16 : 32;
    }
}
int bwd_lanes(int N) {
    int lanes, npt;
    bwd_shape(N, &lanes, &npt);
    return lanes;
}

size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct SWs {
    size_t part, pt, plam, plog, pD, total;
};
SWs ws_layout(int64_t B, int64_t L, int64_t H, int64_t N) {
    const int64_t nt = (H + kBT / bwd_lanes(static_cast<int>(N)) - 1) / (kBT / bwd_lanes(static_cast<int>(N)));
    SWs w;
    w.part = 0;
    w.pt = w.part + align_up(static_cast<size_t>(B * nt * L * N) * sizeof(float4));
    w.plam = w.pt + align_up(static_cast<size_t>(B * nt * L) * sizeof(float));
    w.plog = w.plam + align_up(static_cast<size_t>(B * H * N) * sizeof(float2));
    w.pD = w.plog + align_up(static_cast<size_t>(B * H) * sizeof(float));
    w.total = w.pD + align_up(static_cast<size_t>(B * H) * sizeof(float));
    return w;
}

template <int LANES, int NPT, typename UT>
cudaError_t launch_bwd(const SArgs& a, cudaStream_t s) {
    const size_t smem = BwdSmem<LANES, NPT>::bytes;
    cudaError_t e = cudaFuncSetAttribute(ssm_bwd_chain<LANES, NPT, UT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    mark_start(s);
    ssm_bwd_chain<LANES, NPT, UT><<<dim3(a.ntiles, a.B), kBT, smem, s>>>(a);
    mark_stop(s);
    note_launch();
    return cudaGetLastError();
}

template <typename UT>
cudaError_t bwd_by_n(const SArgs& a, cudaStream_t s) {
    int lanes, npt;
    bwd_shape(a.N, &lanes, &npt);
#if EACS_SSMBWD_NPT == 1
    switch (lanes) {
        case 4: return launch_bwd<4, 1, UT>(a, s);
        case 8: return launch_bwd<8, 1, UT>(a, s);
        case 16: return launch_bwd<16, 1, UT>(a, s);
        default: return npt == 1 ? launch_bwd<32, 1, UT>(a, s) : launch_bwd<32, 2, UT>(a, s);
    }
#else
    switch (lanes) {
        case 4: return launch_bwd<4, 2, UT>(a, s);
        case 8: return launch_bwd<8, 2, UT>(a, s);
        case 16: return launch_bwd<16, 2, UT>(a, s);
        default: return launch_bwd<32, 2, UT>(a, s);
    }
#endif
}

}  // namespace

size_t ssm_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0 || N > 64) return 0;
    return ws_layout(B, L, H, N).total;
}

int ssm_bwd(const SsmBwdCall& c, cudaStream_t stream) {
    const char* fn = "eacs_ssm_bwd";
    if (c.B < 0 || c.L < 0 || c.H < 0 || c.N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)c.N);
    if (c.B > 65535) return fail(EACS_ERR_UNSUPPORTED, "%s: B=%lld > 65535", fn, (long long)c.B);
    if (c.L > (1LL << 30) || c.H > (1LL << 24)) return fail(EACS_ERR_UNSUPPORTED, "%s: L or H too large", fn);
    if (c.u_dtype != EACS_DTYPE_F32 && c.u_dtype != EACS_DTYPE_F16 && c.u_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, c.u_dtype);
    if (c.B == 0 || c.L == 0 || c.H == 0) return EACS_OK;
    if (c.N == 0) return fail(EACS_ERR_INVALID, "%s: N must be positive", fn);
    if (!c.lam || !c.log_dt || !c.t || !c.Bc || !c.Cc || !c.u || !c.D || !c.gy || !c.ckpt || !c.du ||
        !c.dBc || !c.dCc || !c.dt || !c.dlam || !c.dlog || !c.dD)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (c.ckpt_bytes < ssm_ckpt_size(c.B, c.L, c.H, c.N))
        return fail(EACS_ERR_WORKSPACE, "%s: checkpoint buffer of %zu bytes needed, %zu given", fn,
                    ssm_ckpt_size(c.B, c.L, c.H, c.N), c.ckpt_bytes);
    const SWs w = ws_layout(c.B, c.L, c.H, c.N);
    if (!c.workspace || c.workspace_bytes < w.total)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, w.total,
                    c.workspace_bytes);
    SArgs a{};
    a.lam = static_cast<const float2*>(c.lam);
    a.log_dt = c.log_dt;
    a.t = c.t;
    a.Bc = static_cast<const float2*>(c.Bc);
    a.Cc = static_cast<const float2*>(c.Cc);
    a.u = c.u;
    a.D = c.D;
    a.gy = c.gy;
    a.ck = static_cast<const float2*>(c.ckpt);
    a.du = c.du;
    a.dBc = static_cast<float2*>(c.dBc);
    a.dCc = static_cast<float2*>(c.dCc);
    a.dt = c.dt;
    a.dlam = static_cast<float2*>(c.dlam);
    a.dlog = c.dlog;
    a.dD = c.dD;
    char* ws = static_cast<char*>(c.workspace);
    a.part = reinterpret_cast<float4*>(ws + w.part);
    a.pt = reinterpret_cast<float*>(ws + w.pt);
    a.plam = reinterpret_cast<float2*>(ws + w.plam);
    a.plog = reinterpret_cast<float*>(ws + w.plog);
    a.pD = reinterpret_cast<float*>(ws + w.pD);
    a.dt_min = c.dt_min;
    a.dt_max = c.dt_max;
    a.B = static_cast<int>(c.B);
    a.L = static_cast<int>(c.L);
    a.H = static_cast<int>(c.H);
    a.N = static_cast<int>(c.N);
    const int HT = kBT / bwd_lanes(a.N);
    a.ntiles = (a.H + HT - 1) / HT;
    a.nK = (a.L + kK - 1) / kK;

    cudaError_t e;
    if (c.u_dtype == EACS_DTYPE_F16) e = bwd_by_n<__half>(a, stream);
    else if (c.u_dtype == EACS_DTYPE_BF16) e = bwd_by_n<__nv_bfloat16>(a, stream);
    else e = bwd_by_n<float>(a, stream);
    if (e != cudaSuccess) return cuda_check(e, fn);
    const int64_t nbc = static_cast<int64_t>(a.B) * a.L * a.N;
    ssm_post_bc<<<static_cast<unsigned>((nbc + 255) / 256), 256, 0, stream>>>(a);
    const int64_t nbl = static_cast<int64_t>(a.B) * a.L;
    ssm_post_dt<<<static_cast<unsigned>((nbl + 255) / 256), 256, 0, stream>>>(a);
    const int64_t np = std::max<int64_t>(static_cast<int64_t>(a.H) * a.N, a.H);
    ssm_post_params<<<static_cast<unsigned>((np + 255) / 256), 256, 0, stream>>>(a);
    note_launch(3);
    return cuda_check(cudaGetLastError(), fn);
}

}  // namespace eacs
