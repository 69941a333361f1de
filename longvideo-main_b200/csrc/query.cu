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
