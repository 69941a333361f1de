// query.cu -- continuous-time queries over recorded commits (sm_100a).
//
// Reference: cst_ssm/modules/continuous_query.py:12-61.  segment_index finds,
// per query time t*, the last frame k with frame_t[k] <= t* (searchsorted
// right, minus one, clamped to [0, L-1]); readout_from_commits evolves that
// frame's committed state to t*:
//   delta = max(t* - t_pi, 0), dte = clamp(delta e^log_dt, dt_min, dt_max)
//   x*    = dA h_pi + dB_bar B_pi u_pi,   y = Re sum_n C_pi x* + D u_pi
// (the layer's proj_out is the caller's).  One CTA per (tile of channels, row,
// block of queries); thread (hl, ln) of a channel group owns chains
// n = ln + LANES*j; each group of U queries shares one transposed butterfly
// for its U sums over n.  HBM-bound on h_pi: 8 B per (query, h, n).
#include <algorithm>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kQT = 128;  // readout CTA
constexpr int kQB = 32;   // queries per CTA
constexpr int kQU = 4;    // queries per butterfly group

__global__ void query_index_k(const float* __restrict__ ft, const float* __restrict__ tq,
                              int* __restrict__ idx, int B, int L, int Q) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(B) * Q) return;
    const int b = static_cast<int>(i / Q);
    const float* f = ft + static_cast<size_t>(b) * L;
    const float t = tq[i];
    int lo = 0, hi = L;  // first index with f > t
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (f[mid] <= t) lo = mid + 1;
        else hi = mid;
    }
    idx[i] = min(max(lo - 1, 0), L - 1);
}

struct QArgs {
    const float2* lam;
    const float* log_dt;
    const float* D;
    const float2* ch;
    const float* ct;
    const float* cu;
    const float2* cB;
    const float2* cC;
    const float* tq;
    const int* idx;
    float* y;
    float dt_min, dt_max;
    int B, L, Q, H, N;
};

template <int LANES, int NPT>
__global__ void __launch_bounds__(kQT) query_readout_k(QArgs a) {
    constexpr int HT = kQT / LANES;
    using SN = FoldShape<kQU, LANES / 2, 1>;
    const int tid = threadIdx.x, ln = tid % LANES, hl = tid / LANES;
    const int h = blockIdx.x * HT + hl;
    const int b = blockIdx.y;
    const int q0 = blockIdx.z * kQB;
    const bool hv = h < a.H;
    const int H = a.H, N = a.N, L = a.L, Q = a.Q;
    float2 lam[NPT], ilam[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float Dh = hv ? a.D[h] : 0.f;
    const int held = SN::held(ln);
    const bool writer = SN::writer(ln);
    const int qend = min(q0 + kQB, Q);
    for (int g0 = q0; g0 < qend; g0 += kQU) {
        float v[kQU];
#pragma unroll
        for (int uu = 0; uu < kQU; ++uu) {
            const int q = min(g0 + uu, qend - 1);  // a partial group repeats its last query
            const size_t bq = static_cast<size_t>(b) * Q + q;
            // indices from the caller are clamped like segment_index's own
            const size_t row = static_cast<size_t>(b) * L + min(max(a.idx[bq], 0), L - 1);
            const float delta = fmaxf(a.tq[bq] - a.ct[row], 0.f);
            const float dte = eff_dt(delta, scale, a.dt_min, a.dt_max);
            const float upi = hv ? a.cu[row * H + h] : 0.f;
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int n = ln + LANES * j;
                if (!nv[j]) continue;
                float2 dA, dB;
                zoh(lam[j], ilam[j], dte, dA, dB);
                const float2 hp = a.ch[(row * H + h) * N + n];
                const float2 q2 = cmul(dB, a.cB[row * N + n]);
                const float2 P = cmul(dA, hp);
                const float2 xs = make_float2(fmaf(q2.x, upi, P.x), fmaf(q2.y, upi, P.y));
                acc += cre_mul(a.cC[row * N + n], xs);
            }
            v[uu] = acc;
        }
        Fold<kQU, LANES / 2, 1>::run(v, ln);
        if (writer && hv) {
#pragma unroll
            for (int r = 0; r < SN::kRem; ++r) {
                const int q = g0 + held + r;
                if (q < qend) {
                    const size_t bq = static_cast<size_t>(b) * Q + q;
                    const size_t row = static_cast<size_t>(b) * L + min(max(a.idx[bq], 0), L - 1);
                    a.y[bq * H + h] = v[r] + Dh * a.cu[row * H + h];
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Adjoint of the readout (training through continuous queries).  Given gy
// (B,Q,H) = dLoss/dy before proj_out and query indices sorted per row, every
// commit a query reads gets its adjoint:
//   ax = gy conj(C_pi)                 (x*'s)
//   gc_h += conj(dA) ax,  gc_C += gy conj(x*),  gc_B += conj(dB_bar) ax u_pi,
//   gc_u += Re(conj(ax) dB_bar B_pi) + gy D,   gc_t -= delta's adjoint,
// and lam, log_dt, D and the query time get theirs (the ZOH adjoints as in
// the cell backward).  CTA = (tile of channels, row, block of kSB frames);
// the frames' queries come from the segment offsets (one CTA owns a frame's
// h_pi adjoint, so nothing is accumulated across CTAs); sums over channels
// (B_pi, C_pi, the query times) leave as per-tile partials and are added in a
// fixed order by query_bwd_post.  Deterministic, no atomics.
// ---------------------------------------------------------------------------
constexpr int kQBT = 256;  // backward CTA
constexpr int kSB = 64;    // frames per CTA

// first query of each frame: seg[b][l] = #{q : idx[b][q] < l}, l = 0..L;
// indices out of order record EACS_ERR_INVALID in the status word
__global__ void query_seg_k(const int* __restrict__ idx, int* __restrict__ seg, int B, int L, int Q) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    auto cl = [&](int v) { return min(max(v, 0), L - 1); };
    if (i < static_cast<int64_t>(B) * (L + 1)) {
        const int b = static_cast<int>(i / (L + 1)), l = static_cast<int>(i % (L + 1));
        const int* r = idx + static_cast<size_t>(b) * Q;
        int lo = 0, hi = Q;  // first q with idx >= l
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (cl(r[mid]) < l) lo = mid + 1;
            else hi = mid;
        }
        seg[i] = lo;
    }
    if (i < static_cast<int64_t>(B) * Q && (i % Q) > 0 && cl(idx[i]) < cl(idx[i - 1])) set_status(EACS_ERR_INVALID);
}

struct QBArgs {
    const float2* lam;
    const float* log_dt;
    const float* D;
    const float2* ch;
    const float* ct;
    const float* cu;
    const float2* cB;
    const float2* cC;
    const float* tq;
    const int* seg;    // (B, L+1)
    const float* gy;   // (B,Q,H)
    float2* gch;       // (B,L,H,N)
    float* gct;        // (B,L)
    float* gcu;        // (B,L,H)
    float2* gcB;       // (B,L,N)
    float2* gcC;
    float* gtq;        // (B,Q) or null
    float2* dlam;      // (H,N)
    float* dlog;       // (H)
    float* dD;         // (H)
    float2* pB;        // [B][ntile][L][N] per-tile partials
    float2* pC;
    float* pQ;         // [B][Q][ntile*NW] per-(tile, warp) partials of the query times' adjoints
    float2* plam;      // [B*nSB][H][N]
    float* plog;       // [B*nSB][H]
    float* pD;
    float dt_min, dt_max;
    int B, L, Q, H, N, ntile, nSB;
};

template <int LANES>
__device__ __forceinline__ float lane_group_sum(float v) {
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int LANES, int NPT>
__global__ void __launch_bounds__(kQBT) query_bwd_k(QBArgs a) {
    constexpr int HT = kQBT / LANES;
    constexpr int NW = kQBT / 32;
    constexpr int NP = LANES * NPT;
    __shared__ float2 sred[2][NW][NP];
    const int tid = threadIdx.x, ln = tid % LANES, hl = tid / LANES;
    const int lane = tid & 31, wid = tid >> 5;
    const int tile = blockIdx.x, b = blockIdx.y, sb = blockIdx.z;
    const int h = tile * HT + hl;
    const bool hv = h < a.H;
    const int H = a.H, N = a.N, L = a.L, Q = a.Q;
    const int l0 = sb * kSB, l1 = min(L, l0 + kSB);
    float2 lam[NPT], ilam[NPT], glam[NPT];
    bool nv[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int n = ln + LANES * j;
        nv[j] = hv && n < N;
        lam[j] = nv[j] ? a.lam[static_cast<size_t>(h) * N + n] : make_float2(-1.f, 0.f);
        ilam[j] = crecip(lam[j]);
        glam[j] = make_float2(0.f, 0.f);
    }
    const float scale = hv ? expf(a.log_dt[h]) : 1.f;
    const float Dh = hv ? a.D[h] : 0.f;
    float glog = 0.f, gD = 0.f;
    for (int l = l0; l < l1; ++l) {
        const size_t row = static_cast<size_t>(b) * L + l;
        const int qs = a.seg[static_cast<size_t>(b) * (L + 1) + l];
        const int qe = a.seg[static_cast<size_t>(b) * (L + 1) + l + 1];
        if (qs >= qe) {  // no query reads this frame: zero adjoints (CTA-uniform)
#pragma unroll
            for (int j = 0; j < NPT; ++j)
                if (nv[j]) a.gch[(row * H + h) * N + ln + LANES * j] = make_float2(0.f, 0.f);
            if (hv && ln == 0) a.gcu[row * H + h] = 0.f;
            for (int idx = tid; idx < N; idx += kQBT) {
                const size_t o = ((static_cast<size_t>(b) * a.ntile + tile) * L + l) * N + idx;
                a.pB[o] = make_float2(0.f, 0.f);
                a.pC[o] = make_float2(0.f, 0.f);
            }
            continue;
        }
        float2 hp[NPT], Bp[NPT], Cp[NPT], aH[NPT], aB[NPT], aC[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int n = ln + LANES * j;
            hp[j] = nv[j] ? a.ch[(row * H + h) * N + n] : make_float2(0.f, 0.f);
            Bp[j] = nv[j] ? a.cB[row * N + n] : make_float2(0.f, 0.f);
            Cp[j] = nv[j] ? a.cC[row * N + n] : make_float2(0.f, 0.f);
            aH[j] = aB[j] = aC[j] = make_float2(0.f, 0.f);
        }
        const float upi = hv ? a.cu[row * H + h] : 0.f;
        const float tpi = a.ct[row];
        float uc = 0.f, ud = 0.f;
        for (int q = qs; q < qe; ++q) {
            const size_t bq = static_cast<size_t>(b) * Q + q;
            const float draw = a.tq[bq] - tpi;
            const float delta = fmaxf(draw, 0.f);
            const float mdel = draw >= 0.f ? 1.f : 0.f;
            const float dte_raw = delta * scale;
            const float dte = fminf(fmaxf(dte_raw, a.dt_min), a.dt_max);
            const float mdt = (dte_raw >= a.dt_min && dte_raw <= a.dt_max) ? 1.f : 0.f;
            const float gyv = hv ? a.gy[bq * H + h] : 0.f;
            float sdte = 0.f;
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                if (!nv[j]) continue;
                float2 dA, dB;
                zoh(lam[j], ilam[j], dte, dA, dB);
                const float2 qv = cmul(dB, Bp[j]);
                const float2 P = cmul(dA, hp[j]);
                const float2 xs = make_float2(fmaf(qv.x, upi, P.x), fmaf(qv.y, upi, P.y));
                const float2 ax = make_float2(gyv * Cp[j].x, -gyv * Cp[j].y);
                aC[j] = cadd(aC[j], make_float2(gyv * xs.x, -gyv * xs.y));
                const float2 cdA = make_float2(dA.x, -dA.y), cdB = make_float2(dB.x, -dB.y);
                aH[j] = cadd(aH[j], cmul(cdA, ax));
                uc += ax.x * qv.x + ax.y * qv.y;
                const float2 aq = cscale(ax, upi);
                aB[j] = cadd(aB[j], cmul(cdB, aq));
                const float2 adB = cmul(aq, make_float2(Bp[j].x, -Bp[j].y));
                const float2 adA = cmul(make_float2(hp[j].x, -hp[j].y), ax);
                const float2 aE = cmul(adB, make_float2(ilam[j].x, -ilam[j].y));
                float2 alm = cmul(make_float2(-aE.x, -aE.y), cdB);
                const float2 az = cmul(cdA, cadd(adA, aE));
                alm = cadd(alm, cscale(az, dte));
                glam[j] = cadd(glam[j], alm);
                sdte += az.x * lam[j].x + az.y * lam[j].y;
            }
            sdte = lane_group_sum<LANES>(sdte);
            const float drb = mdt * sdte;
            glog += drb * delta * scale;
            gD += gyv * upi;
            ud += gyv;
            // this warp's share of the query time's adjoint (one lane per channel)
            float v = (hv && ln == 0) ? mdel * drb * scale : 0.f;
            v = warp_sum(v);
            if (lane == 0) a.pQ[(bq * a.ntile + tile) * NW + wid] = v;
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j)
            if (nv[j]) a.gch[(row * H + h) * N + ln + LANES * j] = aH[j];
        uc = lane_group_sum<LANES>(uc);
        if (hv && ln == 0) a.gcu[row * H + h] = uc + Dh * ud;
        // B_pi's and C_pi's adjoints summed over the tile's channels
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
#pragma unroll
            for (int o = LANES; o < 32; o <<= 1) {
                aB[j].x += __shfl_xor_sync(0xffffffffu, aB[j].x, o);
                aB[j].y += __shfl_xor_sync(0xffffffffu, aB[j].y, o);
                aC[j].x += __shfl_xor_sync(0xffffffffu, aC[j].x, o);
                aC[j].y += __shfl_xor_sync(0xffffffffu, aC[j].y, o);
            }
            if (lane < LANES) {
                sred[0][wid][ln + LANES * j] = aB[j];
                sred[1][wid][ln + LANES * j] = aC[j];
            }
        }
        __syncthreads();
        for (int idx = tid; idx < 2 * N; idx += kQBT) {
            const int c = idx / N, n = idx % N;
            float2 sum = make_float2(0.f, 0.f);
            for (int w = 0; w < NW; ++w) sum = cadd(sum, sred[c][w][n]);
            const size_t o = ((static_cast<size_t>(b) * a.ntile + tile) * L + l) * N + n;
            (c ? a.pC : a.pB)[o] = sum;
        }
        __syncthreads();
    }
    const size_t pr = static_cast<size_t>(b) * a.nSB + sb;
#pragma unroll
    for (int j = 0; j < NPT; ++j)
        if (nv[j]) a.plam[(pr * H + h) * N + ln + LANES * j] = glam[j];
    if (hv && ln == 0) {
        a.plog[pr * H + h] = glog;
        a.pD[pr * H + h] = gD;
    }
}

// sums of the partials in a fixed order: B_pi's and C_pi's adjoints over the
// tiles, the query times' over the (tile, warp) slots, t_pi's over the
// frame's queries, the parameters' over the (row, frame block) CTAs
__global__ void query_bwd_post_k(QBArgs a, int nslot) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t BLN = static_cast<int64_t>(a.B) * a.L * a.N;
    if (i < BLN) {
        const int64_t b = i / (static_cast<int64_t>(a.L) * a.N), ln = i % (static_cast<int64_t>(a.L) * a.N);
        float2 sb = make_float2(0.f, 0.f), sc = make_float2(0.f, 0.f);
        for (int t = 0; t < a.ntile; ++t) {
            const size_t o = (static_cast<size_t>(b) * a.ntile + t) * a.L * a.N + ln;
            sb = cadd(sb, a.pB[o]);
            sc = cadd(sc, a.pC[o]);
        }
        a.gcB[i] = sb;
        a.gcC[i] = sc;
    }
    auto qsum = [&](size_t bq) {
        float s = 0.f;
        for (int k = 0; k < nslot; ++k) s += a.pQ[bq * nslot + k];
        return s;
    };
    const int64_t BL = static_cast<int64_t>(a.B) * a.L;
    if (i < BL) {
        const int64_t b = i / a.L, l = i % a.L;
        const int qs = a.seg[b * (a.L + 1) + l], qe = a.seg[b * (a.L + 1) + l + 1];
        float s = 0.f;
        for (int q = qs; q < qe; ++q) s += qsum(static_cast<size_t>(b) * a.Q + q);
        a.gct[i] = -s;
    }
    if (a.gtq && i < static_cast<int64_t>(a.B) * a.Q) a.gtq[i] = qsum(static_cast<size_t>(i));
    const int64_t HN = static_cast<int64_t>(a.H) * a.N;
    const int64_t np = static_cast<int64_t>(a.B) * a.nSB;
    if (i < HN) {
        float2 s = make_float2(0.f, 0.f);
        for (int64_t p = 0; p < np; ++p) s = cadd(s, a.plam[p * HN + i]);
        a.dlam[i] = s;
    }
    if (i < a.H) {
        float s1 = 0.f, s2 = 0.f;
        for (int64_t p = 0; p < np; ++p) {
            s1 += a.plog[p * a.H + i];
            s2 += a.pD[p * a.H + i];
        }
        a.dlog[i] = s1;
        a.dD[i] = s2;
    }
}

size_t alq(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct QBWs {
    size_t seg, pB, pC, pQ, plam, plog, pD, total;
};
QBWs qbws(int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N, int ntile, int nSB) {
    QBWs w{};
    constexpr int NW = kQBT / 32;
    size_t o = 0;
    w.seg = o; o += alq(sizeof(int) * B * (L + 1));
    w.pB = o; o += alq(sizeof(float2) * B * ntile * L * N);
    w.pC = o; o += alq(sizeof(float2) * B * ntile * L * N);
    w.pQ = o; o += alq(sizeof(float) * B * Q * ntile * NW);
    w.plam = o; o += alq(sizeof(float2) * B * nSB * H * N);
    w.plog = o; o += alq(sizeof(float) * B * nSB * H);
    w.pD = o; o += alq(sizeof(float) * B * nSB * H);
    w.total = o;
    return w;
}

int qb_lanes(int64_t N) { return N <= 8 ? 4 : N <= 16 ? 8 : N <= 32 ? 16 : 32; }

}  // namespace

int query_index(const float* frame_t, const float* t_query, int* idx, int64_t B, int64_t L,
                int64_t Q, cudaStream_t stream) {
    const char* fn = "eacs_query_index";
    if (B < 0 || L < 0 || Q < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (B == 0 || Q == 0) return EACS_OK;
    if (L == 0) return fail(EACS_ERR_INVALID, "%s: no frames", fn);
    if (!frame_t || !t_query || !idx) return fail(EACS_ERR_INVALID, "%s: null pointer", fn);
    if (L > (1LL << 30) || B * Q > (1LL << 38)) return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    const int64_t n = B * Q;
    query_index_k<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        frame_t, t_query, idx, static_cast<int>(B), static_cast<int>(L), static_cast<int>(Q));
    note_launch();
    return cuda_check(cudaGetLastError(), fn);
}

int query_readout(const void* lam, const float* log_dt, const float* D, const void* commit_h,
                  const float* commit_t, const float* commit_u, const void* commit_B,
                  const void* commit_C, const float* t_query, const int* idx, float* y, int64_t B,
                  int64_t L, int64_t Q, int64_t H, int64_t N, float dt_min, float dt_max,
                  cudaStream_t stream) {
    const char* fn = "eacs_query_readout";
    if (B < 0 || L < 0 || Q < 0 || H < 0 || N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)N);
    if (B > 65535 || Q > (1LL << 30) || L > (1LL << 30) || H > (1LL << 24))
        return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    if (B == 0 || Q == 0 || H == 0) return EACS_OK;
    if (L == 0 || N == 0) return fail(EACS_ERR_INVALID, "%s: no frames or no state", fn);
    if (!lam || !log_dt || !D || !commit_h || !commit_t || !commit_u || !commit_B || !commit_C ||
        !t_query || !idx || !y)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    QArgs a{};
    a.lam = static_cast<const float2*>(lam);
    a.log_dt = log_dt;
    a.D = D;
    a.ch = static_cast<const float2*>(commit_h);
    a.ct = commit_t;
    a.cu = commit_u;
    a.cB = static_cast<const float2*>(commit_B);
    a.cC = static_cast<const float2*>(commit_C);
    a.tq = t_query;
    a.idx = idx;
    a.y = y;
    a.dt_min = dt_min;
    a.dt_max = dt_max;
    a.B = static_cast<int>(B);
    a.L = static_cast<int>(L);
    a.Q = static_cast<int>(Q);
    a.H = static_cast<int>(H);
    a.N = static_cast<int>(N);
    const int lanes = N <= 8 ? 4 : N <= 16 ? 8 : N <= 32 ? 16 : 32;
    const int HT = kQT / lanes;
    const int qb = static_cast<int>((Q + kQB - 1) / kQB);
    if (qb > 65535) return fail(EACS_ERR_UNSUPPORTED, "%s: Q=%lld too large", fn, (long long)Q);
    const dim3 grid(static_cast<unsigned>((H + HT - 1) / HT), static_cast<unsigned>(B), qb);
    if (lanes == 4) query_readout_k<4, 2><<<grid, kQT, 0, stream>>>(a);
    else if (lanes == 8) query_readout_k<8, 2><<<grid, kQT, 0, stream>>>(a);
    else if (lanes == 16) query_readout_k<16, 2><<<grid, kQT, 0, stream>>>(a);
    else query_readout_k<32, 2><<<grid, kQT, 0, stream>>>(a);
    note_launch();
    return cuda_check(cudaGetLastError(), fn);
}

}  // namespace eacs

namespace eacs {

size_t query_readout_bwd_workspace_size(int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N) {
    if (B <= 0 || L <= 0 || Q < 0 || H <= 0 || N <= 0 || N > 64) return 0;
    const int64_t HT = kQBT / qb_lanes(N);
    const int ntile = static_cast<int>((H + HT - 1) / HT);
    const int nSB = static_cast<int>((L + kSB - 1) / kSB);
    return qbws(B, L, Q, H, N, ntile, nSB).total;
}

int query_readout_bwd(const QueryBwdCall& c, cudaStream_t stream) {
    const char* fn = "eacs_query_readout_bwd";
    const int64_t B = c.B, L = c.L, Q = c.Q, H = c.H, N = c.N;
    if (B < 0 || L < 0 || Q < 0 || H < 0 || N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld > 64 is not supported", fn, (long long)N);
    if (B > 65535 || Q > (1LL << 30) || L > (1LL << 30) || H > (1LL << 24))
        return fail(EACS_ERR_UNSUPPORTED, "%s: too large", fn);
    if (B == 0 || L == 0 || H == 0) return EACS_OK;
    if (N == 0) return fail(EACS_ERR_INVALID, "%s: no state", fn);
    if (!c.lam || !c.log_dt || !c.D || !c.commit_h || !c.commit_t || !c.commit_u || !c.commit_B ||
        !c.commit_C || (Q > 0 && (!c.t_query || !c.idx || !c.gy)) || !c.g_commit_h || !c.g_commit_t ||
        !c.g_commit_u || !c.g_commit_B || !c.g_commit_C || !c.dlam || !c.dlog || !c.dD)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    const int lanes = qb_lanes(N);
    const int64_t HT = kQBT / lanes;
    const int ntile = static_cast<int>((H + HT - 1) / HT);
    const int nSB = static_cast<int>((L + kSB - 1) / kSB);
    if (nSB > 65535) return fail(EACS_ERR_UNSUPPORTED, "%s: L=%lld too large", fn, (long long)L);
    const QBWs w = qbws(B, L, Q, H, N, ntile, nSB);
    if (!c.workspace || c.workspace_bytes < w.total)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, w.total,
                    c.workspace_bytes);
    char* ws = static_cast<char*>(c.workspace);
    QBArgs a{};
    a.lam = static_cast<const float2*>(c.lam);
    a.log_dt = c.log_dt;
    a.D = c.D;
    a.ch = static_cast<const float2*>(c.commit_h);
    a.ct = c.commit_t;
    a.cu = c.commit_u;
    a.cB = static_cast<const float2*>(c.commit_B);
    a.cC = static_cast<const float2*>(c.commit_C);
    a.tq = c.t_query;
    a.gy = c.gy;
    a.gch = static_cast<float2*>(c.g_commit_h);
    a.gct = c.g_commit_t;
    a.gcu = c.g_commit_u;
    a.gcB = static_cast<float2*>(c.g_commit_B);
    a.gcC = static_cast<float2*>(c.g_commit_C);
    a.gtq = c.g_t_query;
    a.dlam = static_cast<float2*>(c.dlam);
    a.dlog = c.dlog;
    a.dD = c.dD;
    a.seg = reinterpret_cast<int*>(ws + w.seg);
    a.pB = reinterpret_cast<float2*>(ws + w.pB);
    a.pC = reinterpret_cast<float2*>(ws + w.pC);
    a.pQ = reinterpret_cast<float*>(ws + w.pQ);
    a.plam = reinterpret_cast<float2*>(ws + w.plam);
    a.plog = reinterpret_cast<float*>(ws + w.plog);
    a.pD = reinterpret_cast<float*>(ws + w.pD);
    a.dt_min = c.dt_min;
    a.dt_max = c.dt_max;
    a.B = static_cast<int>(B);
    a.L = static_cast<int>(L);
    a.Q = static_cast<int>(Q);
    a.H = static_cast<int>(H);
    a.N = static_cast<int>(N);
    a.ntile = ntile;
    a.nSB = nSB;
    int* seg = const_cast<int*>(a.seg);
    const int64_t n0 = std::max<int64_t>(B * (L + 1), B * Q);
    if (Q > 0) {
        query_seg_k<<<static_cast<unsigned>((n0 + 255) / 256), 256, 0, stream>>>(c.idx, seg, a.B, a.L, a.Q);
    } else {
        cudaError_t e = cudaMemsetAsync(seg, 0, sizeof(int) * B * (L + 1), stream);
        if (e != cudaSuccess) return cuda_check(e, fn);
    }
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_check(e, fn);
    const dim3 grid(static_cast<unsigned>(ntile), static_cast<unsigned>(B), static_cast<unsigned>(nSB));
    if (lanes == 4) query_bwd_k<4, 2><<<grid, kQBT, 0, stream>>>(a);
    else if (lanes == 8) query_bwd_k<8, 2><<<grid, kQBT, 0, stream>>>(a);
    else if (lanes == 16) query_bwd_k<16, 2><<<grid, kQBT, 0, stream>>>(a);
    else query_bwd_k<32, 2><<<grid, kQBT, 0, stream>>>(a);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_check(e, fn);
    const int64_t n1 = std::max({B * L * N, B * Q, H * N, H, static_cast<int64_t>(1)});
    query_bwd_post_k<<<static_cast<unsigned>((n1 + 255) / 256), 256, 0, stream>>>(a, ntile * (kQBT / 32));
    note_launch();
    return cuda_check(cudaGetLastError(), fn);
}

cudaError_t query_read_status(int* out, cudaStream_t stream) { return read_clear_status(out, stream); }

}  // namespace eacs
