/*
 * eacs_oracle.c -- CPU restatement of CST-SSM's EACS temporal hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * longvideo-main_b200/csrc: it is loaded by tests/, by __graft_entry__.smoke()
 * and by bench.py's CPU-baseline / reference arm, never by the product path.
 *
 * Parity pin: every entry point below is checked against golden vectors made
 * by running the reference's own PyTorch code (tests/golden/make_golden.py).
 *
 * Layouts (all row-major, complex = interleaved float pairs, i.e. complex64):
 *   lam (H,N) complex, log_dt/D/mean/var (H), u (B,L,H), Bc/Cc (B,L,N) complex,
 *   t (B,L), y (B,L,H), gate/resid (B,L), scan tensors (B,L,H,N) complex.
 *
 * Forward math is done in float with the reference's operation order (so the
 * oracle reproduces the reference to a few ulp); the hand-derived backward of
 * the gated cell is done in double.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct { float re, im; } cf;
typedef struct { double re, im; } cd;

static inline cf cf_mul(cf a, cf b) {
    cf r = {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re};
    return r;
}
static inline cf cf_add(cf a, cf b) { cf r = {a.re + b.re, a.im + b.im}; return r; }
static inline cf cf_scale(cf a, float s) { cf r = {a.re * s, a.im * s}; return r; }

/* 1/lam = conj(lam)/|lam|^2 (torch.reciprocal on complex64). */
static inline cf cf_recip(cf z) {
    float d = z.re * z.re + z.im * z.im;
    cf r = {z.re / d, -z.im / d};
    return r;
}

static inline cd cd_mul(cd a, cd b) {
    cd r = {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re};
    return r;
}
static inline cd cd_conj(cd a) { cd r = {a.re, -a.im}; return r; }
static inline cd cd_add(cd a, cd b) { cd r = {a.re + b.re, a.im + b.im}; return r; }
static inline cd cd_sub(cd a, cd b) { cd r = {a.re - b.re, a.im - b.im}; return r; }
static inline cd cd_scale(cd a, double s) { cd r = {a.re * s, a.im * s}; return r; }
static inline cd cd_of(const float* p) { cd r = {p[0], p[1]}; return r; }
static inline double cd_redot(cd a, cd b) { return a.re * b.re + a.im * b.im; } /* Re(conj(a) b) */

static int g_threads = 0;
void eacs_oracle_set_threads(int n) { g_threads = n; }
static int nthreads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ZOH kernels, discretization.py:20-36 (zoh_kernels): z = lam*dt,
 * dA = (expm1(a)+1)(cos b, sin b), E = complex_expm1(z), dB_bar = E * inv_lam. */
static inline void zoh_f(cf lam, cf ilam, float dte, cf* dA, cf* dBbar) {
    float a = lam.re * dte, b = lam.im * dte;
    float em1 = expm1f(a);
    float ea = em1 + 1.0f;
    float sb = sinf(b), cb = cosf(b);
    float im = ea * sb;
    dA->re = ea * cb;
    dA->im = im;
    float sh = sinf(0.5f * b);
    cf E = {em1 * cb - 2.0f * (sh * sh), im};
    *dBbar = cf_mul(E, ilam);
}

/* effective_dt, discretization.py:63-82: clamp(dt*exp(log_dt), dt_min, dt_max). */
static inline float eff_dt(float delta, float scale, float dt_min, float dt_max) {
    float v = delta * scale;
    if (v < dt_min) v = dt_min;
    if (v > dt_max) v = dt_max;
    return v;
}

/* ---------------------------------------------------------------------------
 * scan_fwd: h_l = a_l * h_{l-1} + b_l (scan.py:36-44 sequential_scan_diag;
 * eacs_scan_cuda.cu:23-38).  a, b, h: (B,L,H,N) complex.
 * ------------------------------------------------------------------------- */
int eacs_oracle_scan_fwd(const float* a, const float* b, float* h,
                         int64_t B, int64_t L, int64_t H, int64_t N) {
    int64_t C = H * N;
#pragma omp parallel for num_threads(nthreads()) collapse(2)
    for (int64_t bi = 0; bi < B; ++bi)
        for (int64_t c = 0; c < C; ++c) {
            cf s = {0.f, 0.f};
            for (int64_t l = 0; l < L; ++l) {
                int64_t o = ((bi * L + l) * C + c) * 2;
                cf av = {a[o], a[o + 1]}, bv = {b[o], b[o + 1]};
                s = cf_add(cf_mul(av, s), bv);
                h[o] = s.re;
                h[o + 1] = s.im;
            }
        }
    return 0;
}

/* scan_bwd: reverse adjoint of the scan (eacs_scan_cuda.cu:40-60):
 * s_l = g_l + conj(a_{l+1}) s_{l+1}; grad_b_l = s_l; grad_a_l = s_l conj(h_{l-1}). */
int eacs_oracle_scan_bwd(const float* a, const float* h, const float* gh,
                         float* ga, float* gb,
                         int64_t B, int64_t L, int64_t H, int64_t N) {
    int64_t C = H * N;
#pragma omp parallel for num_threads(nthreads()) collapse(2)
    for (int64_t bi = 0; bi < B; ++bi)
        for (int64_t c = 0; c < C; ++c) {
            cf s = {0.f, 0.f};
            for (int64_t l = L - 1; l >= 0; --l) {
                int64_t o = ((bi * L + l) * C + c) * 2;
                s.re += gh[o];
                s.im += gh[o + 1];
                gb[o] = s.re;
                gb[o + 1] = s.im;
                cf hp = {0.f, 0.f};
                if (l > 0) { hp.re = h[o - 2 * C]; hp.im = -h[o - 2 * C + 1]; }
                cf g = cf_mul(s, hp);
                ga[o] = g.re;
                ga[o + 1] = g.im;
                cf ac = {a[o], -a[o + 1]};
                s = cf_mul(ac, s);
            }
        }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Ungated continuous SSM core, continuous_ssm.py:44-55:
 *   dt_l = max(t_l - t_{l-1}, 0) (dt_0 = dt_1), dt_eff = clamp(dt e^{log_dt}),
 *   h_l = dA h_{l-1} + (dB_bar B_l) u_l,  y = Re sum_n C_l h_l + D u.
 * ------------------------------------------------------------------------- */
int eacs_oracle_ssm_fwd(const float* lam, const float* log_dt, const float* t,
                        const float* Bc, const float* Cc, const float* u,
                        const float* D, float* y,
                        int64_t B, int64_t L, int64_t H, int64_t N,
                        float dt_min, float dt_max) {
#pragma omp parallel for num_threads(nthreads()) collapse(2)
    for (int64_t bi = 0; bi < B; ++bi)
        for (int64_t hh = 0; hh < H; ++hh) {
            float scale = expf(log_dt[hh]);
            cf* st = (cf*)calloc((size_t)N, sizeof(cf));
            for (int64_t l = 0; l < L; ++l) {
                float dt;
                if (L == 1) dt = 0.f;
                else {
                    int64_t l1 = l == 0 ? 1 : l;
                    dt = t[bi * L + l1] - t[bi * L + l1 - 1];
                    if (dt < 0.f) dt = 0.f;
                }
                float dte = eff_dt(dt, scale, dt_min, dt_max);
                float ul = u[(bi * L + l) * H + hh];
                float acc = 0.f;
                for (int64_t n = 0; n < N; ++n) {
                    cf lm = {lam[(hh * N + n) * 2], lam[(hh * N + n) * 2 + 1]};
                    cf dA, dBb;
                    zoh_f(lm, cf_recip(lm), dte, &dA, &dBb);
                    const float* bp = Bc + ((bi * L + l) * N + n) * 2;
                    cf dB = cf_mul(dBb, (cf){bp[0], bp[1]});
                    cf dBu = cf_scale(dB, ul);
                    st[n] = cf_add(cf_mul(dA, st[n]), dBu);
                    const float* cp = Cc + ((bi * L + l) * N + n) * 2;
                    acc += cp[0] * st[n].re - cp[1] * st[n].im;
                }
                y[(bi * L + l) * H + hh] = acc + D[hh] * ul;
            }
            free(st);
        }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Backward of the ungated core (autograd of continuous_ssm.py:44-55 through
 * effective_dt, zoh_discretize, the scan and the readout), in double.
 * Upstream gy (B,L,H).  Outputs (float, overwritten): du (B,L,H), dBc, dCc
 * (B,L,N) complex, dt (B,L), dlam (H,N) complex, dlog (H), dD (H).
 * ------------------------------------------------------------------------- */
int eacs_oracle_ssm_bwd(const float* lam, const float* log_dt, const float* t,
                        const float* Bc, const float* Cc, const float* u,
                        const float* D, const float* gy, float* du, float* dBc,
                        float* dCc, float* dtg, float* dlam, float* dlog, float* dD,
                        int64_t B, int64_t L, int64_t H, int64_t N,
                        float dt_min, float dt_max) {
    double* alam = (double*)calloc((size_t)(B * H * N * 2), sizeof(double));
    double* alog = (double*)calloc((size_t)(B * H), sizeof(double));
    double* aD = (double*)calloc((size_t)(B * H), sizeof(double));
#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        const float* tb = t + bi * L;
        double* dtraw = (double*)malloc(sizeof(double) * (size_t)L);   /* dt before the clamp */
        double* mdt = (double*)malloc(sizeof(double) * (size_t)L);     /* clamp_min(0) mask of t-diff */
        for (int64_t l = 0; l < L; ++l) {
            if (L == 1) { dtraw[l] = 0; mdt[l] = 0; continue; }
            int64_t l1 = l == 0 ? 1 : l;
            double d = (double)tb[l1] - (double)tb[l1 - 1];
            mdt[l] = d >= 0 ? 1.0 : 0.0;
            dtraw[l] = d > 0 ? d : 0;
        }
        double* dtbar = (double*)calloc((size_t)L, sizeof(double));
        cd* gBr = (cd*)calloc((size_t)(L * N), sizeof(cd));
        cd* gCr = (cd*)calloc((size_t)(L * N), sizeof(cd));
        cd* hs = (cd*)malloc(sizeof(cd) * (size_t)((L + 1) * N));
        for (int64_t hh = 0; hh < H; ++hh) {
            double sc = exp((double)log_dt[hh]);
            /* forward states (double) */
            for (int64_t n = 0; n < N; ++n) hs[n] = (cd){0, 0};
            for (int64_t l = 0; l < L; ++l) {
                double v = dtraw[l] * sc, dte = v < dt_min ? dt_min : (v > dt_max ? dt_max : v);
                double ul = u[(bi * L + l) * H + hh];
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    double a = lam[2 * i] * dte, b = lam[2 * i + 1] * dte, e = exp(a);
                    cd dA = {e * cos(b), e * sin(b)};
                    cd E = {expm1(a) * cos(b) - 2 * sin(0.5 * b) * sin(0.5 * b), e * sin(b)};
                    double lr = lam[2 * i], li = lam[2 * i + 1], dd = lr * lr + li * li;
                    cd il = {lr / dd, -li / dd};
                    cd dB = cd_mul(E, il);
                    cd q = cd_mul(dB, cd_of(Bc + ((bi * L + l) * N + n) * 2));
                    hs[(l + 1) * N + n] = cd_add(cd_mul(dA, hs[l * N + n]), cd_scale(q, ul));
                }
            }
            /* reverse */
            cd* s = (cd*)calloc((size_t)N, sizeof(cd));
            for (int64_t l = L - 1; l >= 0; --l) {
                double v = dtraw[l] * sc, dte = v < dt_min ? dt_min : (v > dt_max ? dt_max : v);
                double m = (v >= dt_min && v <= dt_max) ? 1.0 : 0.0;
                double ul = u[(bi * L + l) * H + hh];
                double yb = gy[(bi * L + l) * H + hh];
                double dub = yb * D[hh];
                aD[bi * H + hh] += yb * ul;
                double dtebar = 0;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    double lr = lam[2 * i], li = lam[2 * i + 1], dd = lr * lr + li * li;
                    double a = lr * dte, b = li * dte, e = exp(a);
                    cd dA = {e * cos(b), e * sin(b)};
                    cd E = {expm1(a) * cos(b) - 2 * sin(0.5 * b) * sin(0.5 * b), e * sin(b)};
                    cd il = {lr / dd, -li / dd};
                    cd dB = cd_mul(E, il);
                    cd Bl = cd_of(Bc + ((bi * L + l) * N + n) * 2);
                    cd Cl = cd_of(Cc + ((bi * L + l) * N + n) * 2);
                    /* adjoint of h_l: readout + carried */
                    s[n] = cd_add(s[n], cd_scale(cd_conj(Cl), yb));
                    cd hl = hs[(l + 1) * N + n], hp = hs[l * N + n];
                    /* dC_l += yb conj(h_l) */
                    gCr[l * N + n] = cd_add(gCr[l * N + n], cd_scale(cd_conj(hl), yb));
                    cd q = cd_mul(dB, Bl);
                    dub += cd_redot(s[n], q);
                    cd aq = cd_scale(s[n], ul);
                    gBr[l * N + n] = cd_add(gBr[l * N + n], cd_mul(cd_conj(dB), aq));
                    cd adB = cd_mul(aq, cd_conj(Bl));
                    cd adA = cd_mul(cd_conj(hp), s[n]);
                    cd aE = cd_mul(adB, cd_conj(il));
                    cd ail = cd_mul(adB, cd_conj(E));
                    cd il2 = cd_mul(il, il);
                    cd alm = cd_scale(cd_mul(cd_conj(il2), ail), -1.0);
                    cd az = cd_mul(cd_conj(dA), cd_add(adA, aE));
                    alm = cd_add(alm, cd_scale(az, dte));
                    dtebar += cd_redot(az, (cd){lr, li});
                    alam[(bi * H * N + i) * 2] += alm.re;
                    alam[(bi * H * N + i) * 2 + 1] += alm.im;
                    s[n] = cd_mul(cd_conj(dA), s[n]);
                }
                du[(bi * L + l) * H + hh] = (float)dub;
                double drb = m * dtebar;
                alog[bi * H + hh] += drb * dtraw[l] * sc;
                dtbar[l] += drb * sc;
            }
            free(s);
        }
        /* dt_l = max(t_l - t_{l-1}, 0), dt_0 = dt_1 */
        for (int64_t l = 0; l < L; ++l) dtg[bi * L + l] = 0;
        if (L > 1) {
            for (int64_t l = 0; l < L; ++l) {
                int64_t l1 = l == 0 ? 1 : l;
                double g = dtbar[l] * mdt[l];
                dtg[bi * L + l1] += (float)g;
                dtg[bi * L + l1 - 1] -= (float)g;
            }
        }
        for (int64_t l = 0; l < L; ++l)
            for (int64_t n = 0; n < N; ++n) {
                int64_t o = ((bi * L + l) * N + n) * 2;
                dBc[o] = (float)gBr[l * N + n].re;
                dBc[o + 1] = (float)gBr[l * N + n].im;
                dCc[o] = (float)gCr[l * N + n].re;
                dCc[o + 1] = (float)gCr[l * N + n].im;
            }
        free(dtraw); free(mdt); free(dtbar); free(hs); free(gBr); free(gCr);
    }
    for (int64_t i = 0; i < H * N * 2; ++i) {
        double s2 = 0;
        for (int64_t bi = 0; bi < B; ++bi) s2 += alam[bi * H * N * 2 + i];
        dlam[i] = (float)s2;
    }
    for (int64_t hh = 0; hh < H; ++hh) {
        double s1 = 0, s2 = 0;
        for (int64_t bi = 0; bi < B; ++bi) { s1 += alog[bi * H + hh]; s2 += aD[bi * H + hh]; }
        dlog[hh] = (float)s1;
        dD[hh] = (float)s2;
    }
    free(alam); free(alog); free(aD);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Gated EACS cell, inference (eacs.py:78-142 eacs_step with skip_compute and
 * eacs.py:145-173 scan_range, including robust_guard).  Per batch row:
 *   state (h_pi, t_pi, u_pi, B_pi, C_pi) initialised to (0, t_0-dt_init, u_0, B_0, C_0)
 *   x_hat = dA h_pi + (dB_bar B_pi) u_pi,  y_hat = Re sum_n C_pi x_hat
 *   r = ||(u-mu)/s - (y_hat-mu)/s|| / (||(u-mu)/s|| + eta),  gate = r > eps_l
 *   commit: h_pi = dA h_pi + (dB_bar B_l) u_l, t/u/B/C_pi = current inputs
 *   y = Re sum_n C_l h_cur + D u_l  (h_cur = committed update or x_hat)
 * robust: eps_l = spike >= k ? eps*eps_factor : eps; spike counts consecutive
 *   steps with r_l > r_{l-1}*spike_ratio.
 * gate_mode: 0 = hard gate (inference / STE forward values), 1 = soft gate
 *   sigmoid((r-eps)/max(T,1e-4)) blended into the state (eacs_cell_train.py:47-63).
 * Outputs y (B,L,H), gate, resid (B,L).
 * ------------------------------------------------------------------------- */
static void cell_row(const float* lam, const float* log_dt, const float* u,
                     const float* Bc, const float* Cc, const float* t,
                     const float* D, const float* mean, const float* var,
                     float eps, float eta, float var_eps, float dt_init,
                     float dt_min, float dt_max, int robust, int robust_k,
                     float spike_ratio, float eps_factor, int gate_mode, float T,
                     int train_exp, float* y, float* gate, float* resid,
                     float* ch, float* ct, float* cu, float* cB, float* cC,
                     int64_t L, int64_t H, int64_t N, int nthr) {
    cf* hpi = (cf*)calloc((size_t)(H * N), sizeof(cf));
    cf* dA = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
    cf* dBb = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
    cf* xh = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
    cf* ilam = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
    float* upi = (float*)malloc(sizeof(float) * (size_t)H);
    float* scale = (float*)malloc(sizeof(float) * (size_t)H);
    float* sd = (float*)malloc(sizeof(float) * (size_t)H);
    float* dsq = (float*)malloc(sizeof(float) * (size_t)H);
    float* osq = (float*)malloc(sizeof(float) * (size_t)H);
    cf* Bpi = (cf*)malloc(sizeof(cf) * (size_t)N);
    cf* Cpi = (cf*)malloc(sizeof(cf) * (size_t)N);
    for (int64_t i = 0; i < H * N; ++i) {
        cf lm = {lam[2 * i], lam[2 * i + 1]};
        ilam[i] = cf_recip(lm);
    }
    for (int64_t hh = 0; hh < H; ++hh) {
        scale[hh] = expf(log_dt[hh]);
        sd[hh] = sqrtf(var[hh] + var_eps);
        upi[hh] = u[hh];
    }
    for (int64_t n = 0; n < N; ++n) {
        Bpi[n] = (cf){Bc[2 * n], Bc[2 * n + 1]};
        Cpi[n] = (cf){Cc[2 * n], Cc[2 * n + 1]};
    }
    float tpi = t[0] - dt_init;
    float spike = 0.f, prev_r = 0.f;
    float eps_lo = eps * eps_factor;
    float Tp = T > 1e-4f ? T : 1e-4f;
    float delta = 0.f, g = 0.f;
    /* With nthr > 1 one row's channels are split over threads inside every
     * step (long rows of few videos); the residual's sums are still taken
     * over h in order, in double, so the result does not depend on nthr. */
#pragma omp parallel num_threads(nthr) if (nthr > 1)
    for (int64_t l = 0; l < L; ++l) {
        const float* Bl = Bc + l * N * 2;
        const float* Cl = Cc + l * N * 2;
#pragma omp single
        {
            delta = t[l] - tpi;
            if (delta < 0.f) delta = 0.f;
        }
#pragma omp for schedule(static)
        for (int64_t hh = 0; hh < H; ++hh) {
            float dte = eff_dt(delta, scale[hh], dt_min, dt_max);
            float yhat = 0.f;
            for (int64_t n = 0; n < N; ++n) {
                int64_t i = hh * N + n;
                cf lm = {lam[2 * i], lam[2 * i + 1]};
                if (train_exp) {
                    /* eacs_cell_train.py:32-36: dA = exp(z), dB_bar = complex_expm1(z)/lam */
                    float a = lm.re * dte, b = lm.im * dte;
                    float e = expf(a);
                    dA[i] = (cf){e * cosf(b), e * sinf(b)};
                    float em1 = expm1f(a);
                    float sb = sinf(b), cb = cosf(b);
                    float sh = sinf(0.5f * b);
                    cf E = {em1 * cb - 2.0f * (sh * sh), (em1 + 1.0f) * sb};
                    dBb[i] = cf_mul(E, ilam[i]);
                } else {
                    zoh_f(lm, ilam[i], dte, &dA[i], &dBb[i]);
                }
                cf hf = cf_mul(dA[i], hpi[i]);
                cf q = cf_mul(dBb[i], Bpi[n]);
                xh[i] = cf_add(hf, cf_scale(q, upi[hh]));
                yhat += Cpi[n].re * xh[i].re - Cpi[n].im * xh[i].im;
            }
            float ul = u[l * H + hh];
            float obs = (ul - mean[hh]) / sd[hh];
            float pred = (yhat - mean[hh]) / sd[hh];
            float d = obs - pred;
            dsq[hh] = d;
            osq[hh] = obs;
        }
#pragma omp single
        {
            double sdiff = 0.0, sobs = 0.0;
            for (int64_t hh = 0; hh < H; ++hh) {
                sdiff += (double)dsq[hh] * dsq[hh];
                sobs += (double)osq[hh] * osq[hh];
            }
            float r = sqrtf((float)sdiff) / (sqrtf((float)sobs) + eta);
            float eps_l = eps;
            if (robust) eps_l = (spike >= (float)robust_k) ? eps_lo : eps;
            if (gate_mode == 1) g = 1.0f / (1.0f + expf(-((r - eps_l) / Tp)));
            else g = (r > eps_l) ? 1.0f : 0.0f;
            gate[l] = g;
            resid[l] = r;
            if (robust) {
                if (l > 0) spike = (r > prev_r * spike_ratio) ? spike + 1.0f : 0.0f;
                prev_r = r;
            }
        }
#pragma omp for schedule(static)
        for (int64_t hh = 0; hh < H; ++hh) {
            float ul = u[l * H + hh];
            float acc = 0.f;
            for (int64_t n = 0; n < N; ++n) {
                int64_t i = hh * N + n;
                cf hcur;
                if (gate_mode == 1 || g > 0.5f) {
                    cf hf = cf_mul(dA[i], hpi[i]);
                    cf q = cf_mul(dBb[i], (cf){Bl[2 * n], Bl[2 * n + 1]});
                    cf hu = cf_add(hf, cf_scale(q, ul));
                    if (gate_mode == 1) {
                        cf a1 = cf_scale(hu, g);
                        hcur = cf_add(a1, cf_scale(xh[i], 1.0f - g));
                        hpi[i] = cf_add(a1, cf_scale(hpi[i], 1.0f - g));
                    } else {
                        hcur = hu;
                        hpi[i] = hu;
                    }
                } else {
                    hcur = xh[i];
                }
                acc += Cl[2 * n] * hcur.re - Cl[2 * n + 1] * hcur.im;
            }
            y[l * H + hh] = acc + D[hh] * ul;
            if (gate_mode == 1) upi[hh] = g * ul + (1.0f - g) * upi[hh];
            else if (g > 0.5f) upi[hh] = ul;
            if (ch) {
                /* commits after step l (eacs.py:386-402): the committed state */
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    ch[(l * H * N + i) * 2] = hpi[i].re;
                    ch[(l * H * N + i) * 2 + 1] = hpi[i].im;
                }
                cu[l * H + hh] = upi[hh];
            }
        }
#pragma omp single
        {
            if (gate_mode == 1) {
                for (int64_t n = 0; n < N; ++n) {
                    Bpi[n].re = g * Bl[2 * n] + (1.0f - g) * Bpi[n].re;
                    Bpi[n].im = g * Bl[2 * n + 1] + (1.0f - g) * Bpi[n].im;
                    Cpi[n].re = g * Cl[2 * n] + (1.0f - g) * Cpi[n].re;
                    Cpi[n].im = g * Cl[2 * n + 1] + (1.0f - g) * Cpi[n].im;
                }
                tpi = g * t[l] + (1.0f - g) * tpi;
            } else if (g > 0.5f) {
                for (int64_t n = 0; n < N; ++n) {
                    Bpi[n] = (cf){Bl[2 * n], Bl[2 * n + 1]};
                    Cpi[n] = (cf){Cl[2 * n], Cl[2 * n + 1]};
                }
                tpi = t[l];
            }
            if (ch) {
                ct[l] = tpi;
                for (int64_t n = 0; n < N; ++n) {
                    cB[(l * N + n) * 2] = Bpi[n].re;
                    cB[(l * N + n) * 2 + 1] = Bpi[n].im;
                    cC[(l * N + n) * 2] = Cpi[n].re;
                    cC[(l * N + n) * 2 + 1] = Cpi[n].im;
                }
            }
        }
    }
    free(hpi); free(dA); free(dBb); free(xh); free(ilam); free(upi);
    free(scale); free(sd); free(dsq); free(osq); free(Bpi); free(Cpi);
}

/* Rows in parallel; when there are fewer rows than threads, each row is split
 * over the threads left over (nested parallel regions: nt / B threads per row). */
#define CELL_ROWS(CALL)                                                            \
    do {                                                                           \
        int nt_ = nthreads();                                                      \
        int outer_ = (int)(B < nt_ ? B : nt_);                                     \
        int rt_ = B < nt_ ? nt_ / (int)(B > 0 ? B : 1) : 1;                        \
        if (rt_ > 1) omp_set_max_active_levels(2);                                 \
        _Pragma("omp parallel for num_threads(outer_) schedule(dynamic, 1)")       \
        for (int64_t bi = 0; bi < B; ++bi) { CALL; }                               \
    } while (0)

int eacs_oracle_cell_fwd(const float* lam, const float* log_dt, const float* u,
                         const float* Bc, const float* Cc, const float* t,
                         const float* D, const float* mean, const float* var,
                         float eps, float eta, float var_eps, float dt_init,
                         float dt_min, float dt_max, int robust, int robust_k,
                         float spike_ratio, float eps_factor, int gate_mode, float T,
                         int train_exp, float* y, float* gate, float* resid,
                         int64_t B, int64_t L, int64_t H, int64_t N) {
    CELL_ROWS(cell_row(lam, log_dt, u + bi * L * H, Bc + bi * L * N * 2, Cc + bi * L * N * 2,
                       t + bi * L, D, mean, var, eps, eta, var_eps, dt_init, dt_min, dt_max,
                       robust, robust_k, spike_ratio, eps_factor, gate_mode, T, train_exp,
                       y + bi * L * H, gate + bi * L, resid + bi * L, NULL, NULL, NULL, NULL,
                       NULL, L, H, N, rt_));
    return 0;
}

/* ---------------------------------------------------------------------------
 * Gated cell with per-frame commits (EACSLayer.run_with_commits /
 * _commit_range, eacs.py:386-439): eacs_oracle_cell_fwd plus, after every
 * step, the committed state h_pi (B,L,H,N) complex, t_pi (B,L), u_pi (B,L,H),
 * B_pi, C_pi (B,L,N) complex.
 * ------------------------------------------------------------------------- */
int eacs_oracle_cell_commits(const float* lam, const float* log_dt, const float* u,
                             const float* Bc, const float* Cc, const float* t,
                             const float* D, const float* mean, const float* var,
                             float eps, float eta, float var_eps, float dt_init,
                             float dt_min, float dt_max, int robust, int robust_k,
                             float spike_ratio, float eps_factor,
                             float* y, float* gate, float* resid,
                             float* ch, float* ct, float* cu, float* cB, float* cC,
                             int64_t B, int64_t L, int64_t H, int64_t N) {
    CELL_ROWS(cell_row(lam, log_dt, u + bi * L * H, Bc + bi * L * N * 2, Cc + bi * L * N * 2,
                       t + bi * L, D, mean, var, eps, eta, var_eps, dt_init, dt_min, dt_max,
                       robust, robust_k, spike_ratio, eps_factor, 0, 0.1f, 0,
                       y + bi * L * H, gate + bi * L, resid + bi * L,
                       ch + bi * L * H * N * 2, ct + bi * L, cu + bi * L * H,
                       cB + bi * L * N * 2, cC + bi * L * N * 2, L, H, N, rt_));
    return 0;
}

/* ---------------------------------------------------------------------------
 * Continuous-time query readout (continuous_query.py:12-61).  Per query
 * (b, q): k = last frame with frame_t <= t_query (searchsorted right, minus 1,
 * clamped to [0, L-1]) unless idx is given; then from the commits at k:
 *   delta = max(t_q - t_pi, 0), dte = clamp(delta e^log_dt, dt_min, dt_max)
 *   x* = dA h_pi + dB_bar B_pi u_pi,  y = Re sum_n C_pi x* + D u_pi
 * Output y (B,Q,H) (before the layer's proj_out).
 * ------------------------------------------------------------------------- */
static int64_t segment_index(const float* ft, int64_t L, float tq) {
    int64_t lo = 0, hi = L;  /* first index with ft > tq */
    while (lo < hi) {
        int64_t mid = (lo + hi) / 2;
        if (ft[mid] <= tq) lo = mid + 1; else hi = mid;
    }
    int64_t k = lo - 1;
    return k < 0 ? 0 : (k > L - 1 ? L - 1 : k);
}

int eacs_oracle_query_readout(const float* lam, const float* log_dt, const float* D,
                              const float* ch, const float* ct, const float* cu,
                              const float* cB, const float* cC, const float* frame_t,
                              const float* t_query, const int32_t* idx, float* y,
                              int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N,
                              float dt_min, float dt_max) {
#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        for (int64_t q = 0; q < Q; ++q) {
            float tq = t_query[bi * Q + q];
            int64_t k = idx ? idx[bi * Q + q] : segment_index(frame_t + bi * L, L, tq);
            int64_t row = bi * L + k;
            float delta = tq - ct[row];
            if (delta < 0.f) delta = 0.f;
            for (int64_t hh = 0; hh < H; ++hh) {
                float dte = eff_dt(delta, expf(log_dt[hh]), dt_min, dt_max);
                float upi = cu[row * H + hh];
                float acc = 0.f;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    cf lm = {lam[2 * i], lam[2 * i + 1]};
                    cf dA, dBb;
                    zoh_f(lm, cf_recip(lm), dte, &dA, &dBb);
                    int64_t o = (row * H + hh) * N + n;
                    cf hp = {ch[2 * o], ch[2 * o + 1]};
                    cf Bp = {cB[(row * N + n) * 2], cB[(row * N + n) * 2 + 1]};
                    cf Cp = {cC[(row * N + n) * 2], cC[(row * N + n) * 2 + 1]};
                    cf xs = cf_add(cf_mul(dA, hp), cf_scale(cf_mul(dBb, Bp), upi));
                    acc += Cp.re * xs.re - Cp.im * xs.im;
                }
                y[(bi * Q + q) * H + hh] = acc + D[hh] * upi;
            }
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Adjoint of readout_from_commits (continuous_query.py:20-54) before the
 * layer's proj_out: given gy (B,Q,H) = dLoss/dy, accumulate (in double, rows
 * in order, queries in order) the adjoints of the commits the queries read,
 *   x* = dA h_pi + dB_bar B_pi u_pi,  y = Re sum_n C_pi x* + D u_pi,
 *   dA = e^z, dB_bar = expm1(z)/lam, z = lam dte,
 *   dte = clamp(max(t_q - t_pi, 0) e^log_dt, dt_min, dt_max),
 * into gcH (B,L,H,N) complex, gcT (B,L), gcU (B,L,H), gcB, gcC (B,L,N) complex
 * (overwritten: zero where no query reads a frame), the query times' gtq
 * (B,Q) (may be NULL) and the parameters' dlam (H,N) complex, dlog (H), dD (H).
 * idx as for eacs_oracle_query_readout (NULL = segment_index of t_query).
 * ------------------------------------------------------------------------- */
int eacs_oracle_query_readout_bwd(const float* lam, const float* log_dt, const float* D,
                                  const float* ch, const float* ct, const float* cu,
                                  const float* cB, const float* cC, const float* frame_t,
                                  const float* t_query, const int32_t* idx, const float* gy,
                                  float* gcH, float* gcT, float* gcU, float* gcB, float* gcC,
                                  float* gtq, float* dlam, float* dlog, float* dD,
                                  int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N,
                                  float dt_min, float dt_max) {
    const int64_t HN = H * N;
    double* acc_lam = (double*)calloc((size_t)(B * HN * 2), sizeof(double));
    double* acc_log = (double*)calloc((size_t)(B * H), sizeof(double));
    double* acc_D = (double*)calloc((size_t)(B * H), sizeof(double));
#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        cd* aH = (cd*)calloc((size_t)(L * HN), sizeof(cd));
        cd* aB = (cd*)calloc((size_t)(L * N), sizeof(cd));
        cd* aC = (cd*)calloc((size_t)(L * N), sizeof(cd));
        double* aU = (double*)calloc((size_t)(L * H), sizeof(double));
        double* aT = (double*)calloc((size_t)L, sizeof(double));
        double* alam = acc_lam + bi * HN * 2;
        double* alog = acc_log + bi * H;
        double* aD = acc_D + bi * H;
        for (int64_t q = 0; q < Q; ++q) {
            const float tq = t_query[bi * Q + q];
            const int64_t k = idx ? idx[bi * Q + q] : segment_index(frame_t + bi * L, L, tq);
            const int64_t row = bi * L + k;
            const double draw = (double)tq - (double)ct[row];
            const double delta = draw > 0 ? draw : 0;
            double deltabar = 0;
            for (int64_t hh = 0; hh < H; ++hh) {
                const double sc = exp((double)log_dt[hh]);
                const double dte_raw = delta * sc;
                double dte = dte_raw < dt_min ? dt_min : dte_raw;
                if (dte > dt_max) dte = dt_max;
                const double upi = cu[row * H + hh];
                const double gyv = gy[(bi * Q + q) * H + hh];
                aD[hh] += gyv * upi;
                aU[k * H + hh] += gyv * D[hh];
                double dtebar = 0;
                for (int64_t n = 0; n < N; ++n) {
                    const int64_t i = hh * N + n;
                    const cd lm = {lam[2 * i], lam[2 * i + 1]};
                    const double d2 = lm.re * lm.re + lm.im * lm.im;
                    const cd il = {lm.re / d2, -lm.im / d2};
                    const double a = lm.re * dte, b = lm.im * dte, e = exp(a);
                    const cd dA = {e * cos(b), e * sin(b)};
                    const cd E = {expm1(a) * cos(b) - 2 * sin(0.5 * b) * sin(0.5 * b), e * sin(b)};
                    const cd dB = cd_mul(E, il);
                    const cd hp = cd_of(ch + ((row * H + hh) * N + n) * 2);
                    const cd Bp = cd_of(cB + (row * N + n) * 2);
                    const cd Cp = cd_of(cC + (row * N + n) * 2);
                    const cd qv = cd_mul(dB, Bp);
                    const cd xs = cd_add(cd_mul(dA, hp), cd_scale(qv, upi));
                    const cd ax = cd_scale(cd_conj(Cp), gyv);
                    aC[k * N + n] = cd_add(aC[k * N + n], cd_scale(cd_conj(xs), gyv));
                    aH[k * HN + i] = cd_add(aH[k * HN + i], cd_mul(cd_conj(dA), ax));
                    aU[k * H + hh] += cd_redot(ax, qv);
                    const cd aq = cd_scale(ax, upi);
                    aB[k * N + n] = cd_add(aB[k * N + n], cd_mul(cd_conj(dB), aq));
                    const cd adB = cd_mul(aq, cd_conj(Bp));
                    const cd adA = cd_mul(cd_conj(hp), ax);
                    const cd aE = cd_mul(adB, cd_conj(il));
                    const cd ail = cd_mul(adB, cd_conj(E));
                    cd alm = cd_scale(cd_mul(cd_conj(cd_mul(il, il)), ail), -1.0);
                    const cd az = cd_mul(cd_conj(dA), cd_add(adA, aE));
                    alm = cd_add(alm, cd_scale(az, dte));
                    dtebar += cd_redot(az, lm);
                    alam[2 * i] += alm.re;
                    alam[2 * i + 1] += alm.im;
                }
                const double m = (dte_raw >= dt_min && dte_raw <= (double)dt_max) ? 1.0 : 0.0;
                const double drb = m * dtebar;
                deltabar += drb * sc;
                alog[hh] += drb * delta * sc;
            }
            const double mdel = draw >= 0 ? 1.0 : 0.0;
            if (gtq) gtq[bi * Q + q] = (float)(mdel * deltabar);
            aT[k] -= mdel * deltabar;
        }
        for (int64_t l = 0; l < L; ++l) {
            const int64_t rl = bi * L + l;
            gcT[rl] = (float)aT[l];
            for (int64_t hh = 0; hh < H; ++hh) gcU[rl * H + hh] = (float)aU[l * H + hh];
            for (int64_t i = 0; i < HN; ++i) {
                gcH[(rl * HN + i) * 2] = (float)aH[l * HN + i].re;
                gcH[(rl * HN + i) * 2 + 1] = (float)aH[l * HN + i].im;
            }
            for (int64_t n = 0; n < N; ++n) {
                gcB[(rl * N + n) * 2] = (float)aB[l * N + n].re;
                gcB[(rl * N + n) * 2 + 1] = (float)aB[l * N + n].im;
                gcC[(rl * N + n) * 2] = (float)aC[l * N + n].re;
                gcC[(rl * N + n) * 2 + 1] = (float)aC[l * N + n].im;
            }
        }
        free(aH); free(aB); free(aC); free(aU); free(aT);
    }
    for (int64_t i = 0; i < HN * 2; ++i) {
        double s = 0;
        for (int64_t bi = 0; bi < B; ++bi) s += acc_lam[bi * HN * 2 + i];
        dlam[i] = (float)s;
    }
    for (int64_t hh = 0; hh < H; ++hh) {
        double s = 0, s2 = 0;
        for (int64_t bi = 0; bi < B; ++bi) { s += acc_log[bi * H + hh]; s2 += acc_D[bi * H + hh]; }
        dlog[hh] = (float)s;
        dD[hh] = (float)s2;
    }
    free(acc_lam); free(acc_log); free(acc_D);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Streaming steps with explicit branch state (streaming.py:45-85 per branch,
 * over eacs_step eacs.py:78-142 and EventGate.forward event_gate.py:86-105).
 * Per row and step k (valid masks, first observation of a row commits with
 * itself as predecessor, CPI-modulated threshold, hard or soft gate):
 *   state in (h, t, u, B, C, init) -> state out; outputs y (before proj_out),
 *   gate (1 on the first step), resid, innov (resid once initialised).
 * ------------------------------------------------------------------------- */
int eacs_oracle_stream_chunk(const float* lam, const float* log_dt, const float* D,
                             const float* mean, const float* var, const float* u,
                             const float* Bc, const float* Cc, const float* t,
                             const uint8_t* valid, const float* cpi,
                             const float* h_in, const float* t_in, const float* u_in,
                             const float* B_in, const float* C_in, const uint8_t* init_in,
                             float* h_out, float* t_out, float* u_out, float* B_out,
                             float* C_out, uint8_t* init_out, float* y, float* gate,
                             float* resid, float* innov, float eps, float eta, float var_eps,
                             float dt_init, float dt_min, float dt_max, float cpi_mod,
                             int gate_mode, float T, int64_t B, int64_t K, int64_t H,
                             int64_t N) {
    float Tp = T > 1e-4f ? T : 1e-4f;
#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        cf* h = (cf*)(h_out + bi * H * N * 2);
        float* up = u_out + bi * H;
        cf* Bp = (cf*)(B_out + bi * N * 2);
        cf* Cp = (cf*)(C_out + bi * N * 2);
        memcpy(h, h_in + bi * H * N * 2, sizeof(float) * (size_t)(H * N * 2));
        memcpy(up, u_in + bi * H, sizeof(float) * (size_t)H);
        memcpy(Bp, B_in + bi * N * 2, sizeof(float) * (size_t)(N * 2));
        memcpy(Cp, C_in + bi * N * 2, sizeof(float) * (size_t)(N * 2));
        float tp = t_in[bi];
        int init = init_in[bi] != 0;
        cf* dA = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
        cf* dBb = (cf*)malloc(sizeof(cf) * (size_t)(H * N));
        for (int64_t k = 0; k < K; ++k) {
            int64_t rk = bi * K + k;
            if (valid && !valid[rk]) {
                for (int64_t hh = 0; hh < H; ++hh) y[rk * H + hh] = 0.f;
                gate[rk] = resid[rk] = innov[rk] = 0.f;
                continue;
            }
            const float* ul = u + rk * H;
            const float* Bl = Bc + rk * N * 2;
            const float* Cl = Cc + rk * N * 2;
            float tl = t[rk];
            int first = !init;
            if (first) {
                for (int64_t hh = 0; hh < H; ++hh) up[hh] = ul[hh];
                for (int64_t n = 0; n < N; ++n) {
                    Bp[n] = (cf){Bl[2 * n], Bl[2 * n + 1]};
                    Cp[n] = (cf){Cl[2 * n], Cl[2 * n + 1]};
                }
                tp = tl - dt_init;
            }
            float delta = tl - tp;
            if (delta < 0.f) delta = 0.f;
            double sdiff = 0.0, sobs = 0.0;
            for (int64_t hh = 0; hh < H; ++hh) {
                float dte = eff_dt(delta, expf(log_dt[hh]), dt_min, dt_max);
                float yhat = 0.f;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    cf lm = {lam[2 * i], lam[2 * i + 1]};
                    zoh_f(lm, cf_recip(lm), dte, &dA[i], &dBb[i]);
                    cf xh = cf_add(cf_mul(dA[i], h[i]), cf_scale(cf_mul(dBb[i], Bp[n]), up[hh]));
                    yhat += Cp[n].re * xh.re - Cp[n].im * xh.im;
                }
                float sd = sqrtf(var[hh] + var_eps);
                float obs = (ul[hh] - mean[hh]) / sd;
                float pred = (yhat - mean[hh]) / sd;
                float d = obs - pred;
                sdiff += (double)d * d;
                sobs += (double)obs * obs;
            }
            float r = sqrtf((float)sdiff) / (sqrtf((float)sobs) + eta);
            float eps_l = first ? -1.f : eps;
            if (cpi && cpi_mod > 0.f) {
                float c = cpi[rk] < 0.f ? 0.f : (cpi[rk] > 1.f ? 1.f : cpi[rk]);
                eps_l = eps_l * (1.f - cpi_mod * c);
                if (eps_l < 1e-3f) eps_l = 1e-3f;
            }
            float g = gate_mode == 1 ? 1.0f / (1.0f + expf(-((r - eps_l) / Tp)))
                                     : (r > eps_l ? 1.f : 0.f);
            gate[rk] = first ? 1.f : g;
            resid[rk] = r;
            innov[rk] = init ? r : 0.f;
            for (int64_t hh = 0; hh < H; ++hh) {
                float acc = 0.f;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    cf P = cf_mul(dA[i], h[i]);
                    cf xh = cf_add(P, cf_scale(cf_mul(dBb[i], Bp[n]), up[hh]));
                    cf hu = cf_add(P, cf_scale(cf_mul(dBb[i], (cf){Bl[2 * n], Bl[2 * n + 1]}), ul[hh]));
                    cf hc = cf_add(cf_scale(hu, g), cf_scale(xh, 1.f - g));
                    h[i] = first ? hc : cf_add(cf_scale(hu, g), cf_scale(h[i], 1.f - g));
                    acc += Cl[2 * n] * hc.re - Cl[2 * n + 1] * hc.im;
                }
                y[rk * H + hh] = acc + D[hh] * ul[hh];
                up[hh] = first ? ul[hh] : g * ul[hh] + (1.f - g) * up[hh];
            }
            for (int64_t n = 0; n < N; ++n) {
                cf b = {Bl[2 * n], Bl[2 * n + 1]}, c = {Cl[2 * n], Cl[2 * n + 1]};
                Bp[n] = first ? b : cf_add(cf_scale(b, g), cf_scale(Bp[n], 1.f - g));
                Cp[n] = first ? c : cf_add(cf_scale(c, g), cf_scale(Cp[n], 1.f - g));
            }
            tp = first ? tl : g * tl + (1.f - g) * tp;
            init = 1;
        }
        t_out[bi] = tp;
        init_out[bi] = (uint8_t)init;
        free(dA); free(dBb);
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Backward of GatedEACSCellFunction (eacs_cell_train.py:117-175): the VJP of
 * _step_functional (eacs_cell_train.py:15-66) chained in reverse over L,
 * derived by hand and evaluated in double.  Hard gates are pinned to the
 * forward's gates for gate_mode 0 (STE); gate_mode 1 is the soft gate.
 * Inputs: forward inputs, forward gates gs (B,L), upstream gy (B,L,H),
 *   ggs, grs, gns (B,L) (any may be NULL = zero).
 * Outputs (float, overwritten): du (B,L,H), dBc, dCc (B,L,N) complex, dt (B,L),
 *   dlam (H,N) complex, dlog (H), dD (H), deps (1).
 * ------------------------------------------------------------------------- */
typedef struct {
    double tpi, *upi;
    cd *hpi, *Bpi, *Cpi;
} dstate;

static int cell_bwd_impl(const float* lam, const float* log_dt, const float* u,
                         const float* Bc, const float* Cc, const float* t,
                         const float* D, const float* mean, const float* var,
                         float eps, float eta, float var_eps, float dt_init,
                         float dt_max, float T, int gate_mode, const float* gs,
                         const float* gy, const float* ggs, const float* grs,
                         const float* gns, const float* gcH, const float* gcT,
                         const float* gcU, const float* gcB, const float* gcC,
                         float* du, float* dBc, float* dCc,
                         float* dt, float* dlam, float* dlog, float* dD, float* deps,
                         float* y_out, float* g_out, float* r_out, float* ch_out,
                         float* ct_out, float* cu_out, float* cB_out, float* cC_out,
                         int64_t B, int64_t L, int64_t H, int64_t N) {
    const double dt_min = 1e-3;
    const double Tp = T > 1e-4f ? (double)T : 1e-4;
    int64_t HN = H * N;
    double* acc_lam = (double*)calloc((size_t)(B * HN * 2), sizeof(double));
    double* acc_log = (double*)calloc((size_t)(B * H), sizeof(double));
    double* acc_D = (double*)calloc((size_t)(B * H), sizeof(double));
    double* acc_eps = (double*)calloc((size_t)B, sizeof(double));

#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        const float* ub = u + bi * L * H;
        const float* Bb = Bc + bi * L * N * 2;
        const float* Cb = Cc + bi * L * N * 2;
        const float* tb = t + bi * L;
        /* Forward recompute of all states (double). */
        dstate* st = (dstate*)malloc(sizeof(dstate) * (size_t)(L + 1));
        for (int64_t l = 0; l <= L; ++l) {
            st[l].upi = (double*)malloc(sizeof(double) * (size_t)H);
            st[l].hpi = (cd*)malloc(sizeof(cd) * (size_t)HN);
            st[l].Bpi = (cd*)malloc(sizeof(cd) * (size_t)N);
            st[l].Cpi = (cd*)malloc(sizeof(cd) * (size_t)N);
        }
        st[0].tpi = (double)(tb[0] - dt_init);
        for (int64_t hh = 0; hh < H; ++hh) st[0].upi[hh] = ub[hh];
        for (int64_t i = 0; i < HN; ++i) st[0].hpi[i] = (cd){0, 0};
        for (int64_t n = 0; n < N; ++n) {
            st[0].Bpi[n] = cd_of(Bb + 2 * n);
            st[0].Cpi[n] = cd_of(Cb + 2 * n);
        }
        cd* ilam = (cd*)malloc(sizeof(cd) * (size_t)HN);
        for (int64_t i = 0; i < HN; ++i) {
            double a = lam[2 * i], b = lam[2 * i + 1], d = a * a + b * b;
            ilam[i] = (cd){a / d, -b / d};
        }
        double* sdv = (double*)malloc(sizeof(double) * (size_t)H);
        double* sc = (double*)malloc(sizeof(double) * (size_t)H);
        for (int64_t hh = 0; hh < H; ++hh) {
            sdv[hh] = sqrt((double)var[hh] + (double)var_eps);
            sc[hh] = exp((double)log_dt[hh]);
        }
        /* per-step scratch */
        cd* dA = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* E = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* dB = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* hf = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* xh = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* hu = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd* hcur = (cd*)malloc(sizeof(cd) * (size_t)HN);
        double* dte = (double*)malloc(sizeof(double) * (size_t)H);
        double* dte_raw = (double*)malloc(sizeof(double) * (size_t)H);
        double* obs = (double*)malloc(sizeof(double) * (size_t)H);
        double* dv = (double*)malloc(sizeof(double) * (size_t)H);

        /* step function: fills per-step arrays for step l from state st[l]; returns
         * r pieces through pointers; if adv, writes st[l+1]. */
#define STEP_FWD(l, adv)                                                              \
        do {                                                                          \
            dstate* S = &st[l];                                                       \
            double tl = tb[l];                                                        \
            draw = tl - S->tpi;                                                       \
            delta = draw > 0 ? draw : 0;                                              \
            for (int64_t hh = 0; hh < H; ++hh) {                                      \
                dte_raw[hh] = delta * sc[hh];                                         \
                double v = dte_raw[hh];                                               \
                if (v < dt_min) v = dt_min;                                           \
                if (v > dt_max) v = dt_max;                                           \
                dte[hh] = v;                                                          \
            }                                                                         \
            sdiff = 0; sobs = 0;                                                      \
            for (int64_t hh = 0; hh < H; ++hh) {                                      \
                double yh = 0;                                                        \
                for (int64_t n = 0; n < N; ++n) {                                     \
                    int64_t i = hh * N + n;                                           \
                    double a = lam[2 * i] * dte[hh], b = lam[2 * i + 1] * dte[hh];    \
                    double e = exp(a);                                                \
                    dA[i] = (cd){e * cos(b), e * sin(b)};                             \
                    E[i] = (cd){expm1(a) * cos(b) - 2 * sin(0.5 * b) * sin(0.5 * b),  \
                                e * sin(b)};                                          \
                    dB[i] = cd_mul(E[i], ilam[i]);                                    \
                    hf[i] = cd_mul(dA[i], S->hpi[i]);                                 \
                    xh[i] = cd_add(hf[i], cd_scale(cd_mul(dB[i], S->Bpi[n]), S->upi[hh])); \
                    yh += S->Cpi[n].re * xh[i].re - S->Cpi[n].im * xh[i].im;          \
                }                                                                     \
                double ul = ub[l * H + hh];                                           \
                obs[hh] = (ul - mean[hh]) / sdv[hh];                                  \
                double pred = (yh - mean[hh]) / sdv[hh];                              \
                dv[hh] = obs[hh] - pred;                                              \
                sdiff += dv[hh] * dv[hh];                                             \
                sobs += obs[hh] * obs[hh];                                            \
            }                                                                         \
            num = sqrt(sdiff); nobs = sqrt(sobs); den = nobs + eta;                   \
            r = num / den;                                                            \
            soft = 1.0 / (1.0 + exp(-((r - (double)eps) / Tp)));                      \
            g = gate_mode == 1 ? soft : gs ? (double)gs[bi * L + l] : (r > (double)eps ? 1.0 : 0.0); \
            for (int64_t hh = 0; hh < H; ++hh) {                                      \
                double ul = ub[l * H + hh];                                           \
                for (int64_t n = 0; n < N; ++n) {                                     \
                    int64_t i = hh * N + n;                                           \
                    hu[i] = cd_add(hf[i], cd_scale(cd_mul(dB[i], cd_of(Bb + 2 * (l * N + n))), ul)); \
                    hcur[i] = cd_add(cd_scale(hu[i], g), cd_scale(xh[i], 1 - g));    \
                }                                                                     \
            }                                                                         \
            if (adv) {                                                                \
                dstate* S2 = &st[l + 1];                                              \
                S2->tpi = g * tl + (1 - g) * S->tpi;                                  \
                for (int64_t hh = 0; hh < H; ++hh)                                    \
                    S2->upi[hh] = g * ub[l * H + hh] + (1 - g) * S->upi[hh];          \
                for (int64_t i = 0; i < HN; ++i)                                      \
                    S2->hpi[i] = cd_add(cd_scale(hu[i], g), cd_scale(S->hpi[i], 1 - g)); \
                for (int64_t n = 0; n < N; ++n) {                                     \
                    S2->Bpi[n] = cd_add(cd_scale(cd_of(Bb + 2 * (l * N + n)), g), cd_scale(S->Bpi[n], 1 - g)); \
                    S2->Cpi[n] = cd_add(cd_scale(cd_of(Cb + 2 * (l * N + n)), g), cd_scale(S->Cpi[n], 1 - g)); \
                }                                                                     \
            }                                                                         \
        } while (0)

        double draw, delta, sdiff, sobs, num, nobs, den, r, soft, g;
        for (int64_t l = 0; l < L; ++l) {
            STEP_FWD(l, 1);
            /* optional forward outputs: y, gate, residual and the commits
             * (the state after the step) */
            const int64_t rl = bi * L + l;
            if (y_out) {
                for (int64_t hh = 0; hh < H; ++hh) {
                    double acc = 0;
                    for (int64_t n = 0; n < N; ++n) {
                        cd c = cd_of(Cb + 2 * (l * N + n));
                        acc += c.re * hcur[hh * N + n].re - c.im * hcur[hh * N + n].im;
                    }
                    y_out[rl * H + hh] = (float)(acc + (double)D[hh] * ub[l * H + hh]);
                }
            }
            if (g_out) g_out[rl] = (float)g;
            if (r_out) r_out[rl] = (float)r;
            const dstate* S2 = &st[l + 1];
            if (ch_out)
                for (int64_t i = 0; i < HN; ++i) {
                    ch_out[(rl * HN + i) * 2] = (float)S2->hpi[i].re;
                    ch_out[(rl * HN + i) * 2 + 1] = (float)S2->hpi[i].im;
                }
            if (ct_out) ct_out[rl] = (float)S2->tpi;
            if (cu_out)
                for (int64_t hh = 0; hh < H; ++hh) cu_out[rl * H + hh] = (float)S2->upi[hh];
            if (cB_out && cC_out)
                for (int64_t n = 0; n < N; ++n) {
                    cB_out[(rl * N + n) * 2] = (float)S2->Bpi[n].re;
                    cB_out[(rl * N + n) * 2 + 1] = (float)S2->Bpi[n].im;
                    cC_out[(rl * N + n) * 2] = (float)S2->Cpi[n].re;
                    cC_out[(rl * N + n) * 2 + 1] = (float)S2->Cpi[n].im;
                }
        }

        /* Adjoints of the carried state (state after step l). */
        cd* ah = (cd*)calloc((size_t)HN, sizeof(cd));
        double at = 0;
        double* au = (double*)calloc((size_t)H, sizeof(double));
        cd* aB = (cd*)calloc((size_t)N, sizeof(cd));
        cd* aC = (cd*)calloc((size_t)N, sizeof(cd));
        cd* ahn = (cd*)malloc(sizeof(cd) * (size_t)HN);
        double* aun = (double*)malloc(sizeof(double) * (size_t)H);
        cd* aBn = (cd*)malloc(sizeof(cd) * (size_t)N);
        cd* aCn = (cd*)malloc(sizeof(cd) * (size_t)N);
        double* dul = (double*)malloc(sizeof(double) * (size_t)H);
        cd* dBl = (cd*)malloc(sizeof(cd) * (size_t)N);
        cd* dCl = (cd*)malloc(sizeof(cd) * (size_t)N);
        double* dtl = (double*)calloc((size_t)L, sizeof(double));
        double* dub = (double*)calloc((size_t)(L * H), sizeof(double));
        cd* dBb = (cd*)calloc((size_t)(L * N), sizeof(cd));
        cd* dCb = (cd*)calloc((size_t)(L * N), sizeof(cd));
        double* alam = acc_lam + bi * HN * 2;
        double* alog = acc_log + bi * H;
        double* aD = acc_D + bi * H;

        for (int64_t l = L - 1; l >= 0; --l) {
            STEP_FWD(l, 0);
            dstate* S = &st[l];
            double tl = tb[l];
            /* upstream adjoints of the commits of step l (the state after it,
             * eacs.py:386-401 returns it per frame) join the carried ones */
            {
                const int64_t rl = bi * L + l;
                if (gcH)
                    for (int64_t i = 0; i < HN; ++i) {
                        ah[i].re += gcH[(rl * HN + i) * 2];
                        ah[i].im += gcH[(rl * HN + i) * 2 + 1];
                    }
                if (gcT) at += gcT[rl];
                if (gcU)
                    for (int64_t hh = 0; hh < H; ++hh) au[hh] += gcU[rl * H + hh];
                for (int64_t n = 0; n < N; ++n) {
                    if (gcB) { aB[n].re += gcB[(rl * N + n) * 2]; aB[n].im += gcB[(rl * N + n) * 2 + 1]; }
                    if (gcC) { aC[n].re += gcC[(rl * N + n) * 2]; aC[n].im += gcC[(rl * N + n) * 2 + 1]; }
                }
            }
            double gyl_any = gy != NULL;
            double gbar = ggs ? ggs[bi * L + l] : 0.0;
            double rbar = grs ? grs[bi * L + l] : 0.0;
            double nbar = gns ? gns[bi * L + l] : 0.0;
            for (int64_t hh = 0; hh < H; ++hh) dul[hh] = 0;
            for (int64_t n = 0; n < N; ++n) { dBl[n] = (cd){0, 0}; dCl[n] = (cd){0, 0}; }
            /* y = Re sum C_l hcur + D u_l */
            for (int64_t hh = 0; hh < H; ++hh) {
                double yb = gyl_any ? gy[(bi * L + l) * H + hh] : 0.0;
                double ul = ub[l * H + hh];
                aD[hh] += yb * ul;
                dul[hh] += yb * D[hh];
            }
            /* blends and the gate adjoint */
            for (int64_t hh = 0; hh < H; ++hh) {
                double yb = gyl_any ? gy[(bi * L + l) * H + hh] : 0.0;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    cd Cl = cd_of(Cb + 2 * (l * N + n));
                    cd ahc = cd_scale(cd_conj(Cl), yb);
                    /* dC_l += yb * conj(hcur) */
                    dCl[n] = cd_add(dCl[n], cd_scale(cd_conj(hcur[i]), yb));
                    gbar += cd_redot(ahc, cd_sub(hu[i], xh[i]));
                    gbar += cd_redot(ah[i], cd_sub(hu[i], S->hpi[i]));
                    /* store ahcur in hcur slot for later use */
                    hcur[i] = ahc;
                }
            }
            gbar += at * (tl - S->tpi);
            for (int64_t hh = 0; hh < H; ++hh) gbar += au[hh] * (ub[l * H + hh] - S->upi[hh]);
            for (int64_t n = 0; n < N; ++n) {
                gbar += cd_redot(aB[n], cd_sub(cd_of(Bb + 2 * (l * N + n)), S->Bpi[n]));
                gbar += cd_redot(aC[n], cd_sub(cd_of(Cb + 2 * (l * N + n)), S->Cpi[n]));
            }
            double dtl_l = g * at;
            double atn = (1 - g) * at;
            for (int64_t hh = 0; hh < H; ++hh) { dul[hh] += g * au[hh]; aun[hh] = (1 - g) * au[hh]; }
            for (int64_t n = 0; n < N; ++n) {
                dBl[n] = cd_add(dBl[n], cd_scale(aB[n], g));
                aBn[n] = cd_scale(aB[n], 1 - g);
                dCl[n] = cd_add(dCl[n], cd_scale(aC[n], g));
                aCn[n] = cd_scale(aC[n], 1 - g);
            }
            /* gate -> soft -> r, eps */
            /* gate_mode 2: the eval-mode gate r > eps, a constant */
            double xbar = gate_mode == 2 ? 0.0 : gbar * soft * (1 - soft);
            rbar += xbar / Tp;
            acc_eps[bi] += -xbar / Tp;
            double numbar = rbar / den;
            double denbar = -rbar * num / (den * den);
            double numtbar = nbar / den;
            for (int64_t hh = 0; hh < H; ++hh) {
                double dbar = num > 0 ? numbar * dv[hh] / num : 0.0;
                double obar = dbar + (nobs > 0 ? denbar * obs[hh] / nobs : 0.0);
                double pbar = -dbar - (num > 0 ? numtbar * dv[hh] / num : 0.0);
                dul[hh] += obar / sdv[hh];
                obs[hh] = pbar / sdv[hh]; /* reuse as yhat_bar */
            }
            double deltabar = 0;
            for (int64_t hh = 0; hh < H; ++hh) {
                double ul = ub[l * H + hh];
                double yhb = obs[hh];
                double dtebar = 0;
                for (int64_t n = 0; n < N; ++n) {
                    int64_t i = hh * N + n;
                    cd ahc = hcur[i];
                    cd ahu = cd_add(cd_scale(ahc, g), cd_scale(ah[i], g));
                    cd axh = cd_scale(ahc, 1 - g);
                    cd ahp = cd_scale(ah[i], 1 - g);
                    /* yhat = Re sum C_pi xhat */
                    axh = cd_add(axh, cd_scale(cd_conj(S->Cpi[n]), yhb));
                    aCn[n] = cd_add(aCn[n], cd_scale(cd_conj(xh[i]), yhb));
                    /* xhat = hf + (dB B_pi) u_pi ; hupd = hf + (dB B_l) u_l */
                    cd ahf = cd_add(axh, ahu);
                    cd Bl = cd_of(Bb + 2 * (l * N + n));
                    cd qpi = cd_mul(dB[i], S->Bpi[n]);
                    cd ql = cd_mul(dB[i], Bl);
                    cd aqpi = cd_scale(axh, S->upi[hh]);
                    cd aql = cd_scale(ahu, ul);
                    aun[hh] += cd_redot(axh, qpi);
                    dul[hh] += cd_redot(ahu, ql);
                    cd adB = cd_add(cd_mul(aqpi, cd_conj(S->Bpi[n])), cd_mul(aql, cd_conj(Bl)));
                    aBn[n] = cd_add(aBn[n], cd_mul(cd_conj(dB[i]), aqpi));
                    dBl[n] = cd_add(dBl[n], cd_mul(cd_conj(dB[i]), aql));
                    /* hf = dA h_pi */
                    ahp = cd_add(ahp, cd_mul(cd_conj(dA[i]), ahf));
                    cd adA = cd_mul(cd_conj(S->hpi[i]), ahf);
                    /* dB = E * ilam */
                    cd aE = cd_mul(adB, cd_conj(ilam[i]));
                    cd ail = cd_mul(adB, cd_conj(E[i]));
                    cd il2 = cd_mul(ilam[i], ilam[i]);
                    cd alm = cd_scale(cd_mul(cd_conj(il2), ail), -1.0);
                    /* dA = exp(z), E = expm1(z): dz = conj(exp z)(adA + aE) */
                    cd az = cd_mul(cd_conj(dA[i]), cd_add(adA, aE));
                    alm = cd_add(alm, cd_scale(az, dte[hh]));
                    cd lm = {lam[2 * i], lam[2 * i + 1]};
                    dtebar += cd_redot(az, lm);
                    alam[2 * i] += alm.re;
                    alam[2 * i + 1] += alm.im;
                    ahn[i] = ahp;
                }
                double m = (dte_raw[hh] >= dt_min && dte_raw[hh] <= (double)dt_max) ? 1.0 : 0.0;
                double drb = m * dtebar;
                deltabar += drb * sc[hh];
                alog[hh] += drb * delta * sc[hh];
            }
            double mdel = draw >= 0 ? 1.0 : 0.0;
            dtl_l += mdel * deltabar;
            atn += -mdel * deltabar;
            dtl[l] += dtl_l;
            for (int64_t hh = 0; hh < H; ++hh) dub[l * H + hh] += dul[hh];
            for (int64_t n = 0; n < N; ++n) {
                dBb[l * N + n] = cd_add(dBb[l * N + n], dBl[n]);
                dCb[l * N + n] = cd_add(dCb[l * N + n], dCl[n]);
            }
            /* roll adjoints */
            cd* tmp = ah; ah = ahn; ahn = tmp;
            at = atn;
            double* tu = au; au = aun; aun = tu;
            cd* tB = aB; aB = aBn; aBn = tB;
            cd* tC = aC; aC = aCn; aCn = tC;
        }
        /* initial state: t_pi = t_0 - dt_init, u_pi = u_0, B_pi = B_0, C_pi = C_0 */
        dtl[0] += at;
        for (int64_t hh = 0; hh < H; ++hh) dub[hh] += au[hh];
        for (int64_t n = 0; n < N; ++n) {
            dBb[n] = cd_add(dBb[n], aB[n]);
            dCb[n] = cd_add(dCb[n], aC[n]);
        }
        for (int64_t l = 0; l < L; ++l) {
            dt[bi * L + l] = (float)dtl[l];
            for (int64_t hh = 0; hh < H; ++hh) du[(bi * L + l) * H + hh] = (float)dub[l * H + hh];
            for (int64_t n = 0; n < N; ++n) {
                int64_t o = ((bi * L + l) * N + n) * 2;
                dBc[o] = (float)dBb[l * N + n].re;
                dBc[o + 1] = (float)dBb[l * N + n].im;
                dCc[o] = (float)dCb[l * N + n].re;
                dCc[o + 1] = (float)dCb[l * N + n].im;
            }
        }
#undef STEP_FWD
        for (int64_t l = 0; l <= L; ++l) {
            free(st[l].upi); free(st[l].hpi); free(st[l].Bpi); free(st[l].Cpi);
        }
        free(st); free(ilam); free(sdv); free(sc); free(dA); free(E); free(dB); free(hf);
        free(xh); free(hu); free(hcur); free(dte); free(dte_raw); free(obs); free(dv);
        free(ah); free(au); free(aB); free(aC); free(ahn); free(aun);
        free(aBn); free(aCn); free(dul); free(dBl); free(dCl); free(dtl); free(dub);
        free(dBb); free(dCb);
    }
    /* deterministic cross-row reduction of the parameter gradients */
    for (int64_t i = 0; i < HN * 2; ++i) {
        double s = 0;
        for (int64_t bi = 0; bi < B; ++bi) s += acc_lam[bi * HN * 2 + i];
        dlam[i] = (float)s;
    }
    for (int64_t hh = 0; hh < H; ++hh) {
        double s = 0, s2 = 0;
        for (int64_t bi = 0; bi < B; ++bi) { s += acc_log[bi * H + hh]; s2 += acc_D[bi * H + hh]; }
        dlog[hh] = (float)s;
        dD[hh] = (float)s2;
    }
    double se = 0;
    for (int64_t bi = 0; bi < B; ++bi) se += acc_eps[bi];
    deps[0] = (float)se;
    free(acc_lam); free(acc_log); free(acc_D); free(acc_eps);
    return 0;
}

int eacs_oracle_cell_bwd(const float* lam, const float* log_dt, const float* u,
                         const float* Bc, const float* Cc, const float* t,
                         const float* D, const float* mean, const float* var,
                         float eps, float eta, float var_eps, float dt_init,
                         float dt_max, float T, int gate_mode, const float* gs,
                         const float* gy, const float* ggs, const float* grs,
                         const float* gns, float* du, float* dBc, float* dCc,
                         float* dt, float* dlam, float* dlog, float* dD, float* deps,
                         int64_t B, int64_t L, int64_t H, int64_t N) {
    return cell_bwd_impl(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps, dt_init,
                         dt_max, T, gate_mode, gs, gy, ggs, grs, gns, NULL, NULL, NULL, NULL,
                         NULL, du, dBc, dCc, dt, dlam, dlog, dD, deps, NULL, NULL, NULL, NULL,
                         NULL, NULL, NULL, NULL, B, L, H, N);
}

/* ---------------------------------------------------------------------------
 * Training through per-frame commits: EACSLayer._commit_range (eacs.py:386-401)
 * under autograd, i.e. the gated cell of eacs_step (eacs.py:78-142) with the
 * training gate (STE hard forward for gate_mode 0, soft for 1; 2 is the
 * eval-mode gate r > eps, which passes no gradient; event_gate.py:84-105),
 * which also returns the state after every step.
 * Forward outputs (any may be NULL): y (B,L,H), gate, resid (B,L) and the
 * commits h (B,L,H,N) complex, t (B,L), u (B,L,H), B, C (B,L,N) complex.
 * Backward: the cell backward above with the upstream adjoints of the commits
 * gcH, gcT, gcU, gcB, gcC (same shapes; any may be NULL = zero) added to the
 * carried state adjoints at their step.  gy may be NULL.
 * ------------------------------------------------------------------------- */
int eacs_oracle_cell_bwd_commits(const float* lam, const float* log_dt, const float* u,
                                 const float* Bc, const float* Cc, const float* t,
                                 const float* D, const float* mean, const float* var,
                                 float eps, float eta, float var_eps, float dt_init,
                                 float dt_max, float T, int gate_mode, const float* gs,
                                 const float* gy, const float* ggs, const float* grs,
                                 const float* gcH, const float* gcT, const float* gcU,
                                 const float* gcB, const float* gcC, float* du, float* dBc,
                                 float* dCc, float* dt, float* dlam, float* dlog, float* dD,
                                 float* deps, float* y_out, float* g_out, float* r_out,
                                 float* ch_out, float* ct_out, float* cu_out, float* cB_out,
                                 float* cC_out, int64_t B, int64_t L, int64_t H, int64_t N) {
    return cell_bwd_impl(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps, dt_init,
                         dt_max, T, gate_mode, gs, gy, ggs, grs, NULL, gcH, gcT, gcU, gcB, gcC,
                         du, dBc, dCc, dt, dlam, dlog, dD, deps, y_out, g_out, r_out, ch_out,
                         ct_out, cu_out, cB_out, cC_out, B, L, H, N);
}

/* ---------------------------------------------------------------------------
 * Backward of one streaming step of one branch (the per-branch body of
 * temporal_step, streaming.py:55-80, over eacs_step, eacs.py:78-142, and
 * EventGate.forward, event_gate.py:84-105), under autograd: the
 * vector-Jacobian product with respect to the frame's u (B,H), Bc, Cc (B,N)
 * complex, t (B), cpi (B), the state in h (B,H,N) complex, t, u, B, C, and
 * lam (H,N) complex, log_dt (H), D (H), eps (1).  Upstream: gy (B,H) of y
 * (before proj_out), gg, gr, gn (B) of the gate (1 on the first step), resid
 * and innov outputs, and gh, gt, gu, gB, gC of the state out (any may be
 * NULL = 0).  gate_mode 0: STE (hard forward, soft backward); 1: soft; 2:
 * hard with no gradient through the gate (eval).  gs (B) or NULL: the
 * forward's gate output to pin for rows past their first observation (hard
 * modes).  Rows with valid = 0 pass the state's adjoints through.  Outputs
 * overwritten; dcpi may be NULL.  Double precision throughout.
 * ------------------------------------------------------------------------- */
int eacs_oracle_stream_step_bwd(const float* lam, const float* log_dt, const float* D,
                                const float* mean, const float* var, const float* u,
                                const float* Bc, const float* Cc, const float* t,
                                const uint8_t* valid, const float* cpi, const float* h_in,
                                const float* t_in, const float* u_in, const float* B_in,
                                const float* C_in, const uint8_t* init_in, const float* gs,
                                const float* gy, const float* gg, const float* gr,
                                const float* gn, const float* gh, const float* gt,
                                const float* gu, const float* gB, const float* gC, float* du,
                                float* dBc, float* dCc, float* dt, float* dcpi, float* dh_in,
                                float* dt_in, float* du_in, float* dB_in, float* dC_in,
                                float* dlam, float* dlog, float* dD, float* deps, float eps,
                                float eta, float var_eps, float dt_init, float dt_min,
                                float dt_max, float cpi_mod, int gate_mode, float T, int64_t B,
                                int64_t H, int64_t N) {
    const double Tp = T > 1e-4f ? (double)T : 1e-4;
    const int64_t HN = H * N;
    double* acc_lam = (double*)calloc((size_t)(B * HN * 2), sizeof(double));
    double* acc_log = (double*)calloc((size_t)(B * H), sizeof(double));
    double* acc_D = (double*)calloc((size_t)(B * H), sizeof(double));
    double* acc_eps = (double*)calloc((size_t)B, sizeof(double));
#pragma omp parallel for num_threads(nthreads()) schedule(dynamic, 1)
    for (int64_t bi = 0; bi < B; ++bi) {
        const int v = valid ? valid[bi] != 0 : 1;
        const float* hs = h_in + bi * HN * 2;
        float* dhs = dh_in + bi * HN * 2;
        if (!v) {  /* masked: the state passes through */
            for (int64_t i = 0; i < HN * 2; ++i) dhs[i] = gh ? gh[bi * HN * 2 + i] : 0.f;
            dt_in[bi] = gt ? gt[bi] : 0.f;
            for (int64_t hh = 0; hh < H; ++hh) {
                du_in[bi * H + hh] = gu ? gu[bi * H + hh] : 0.f;
                du[bi * H + hh] = 0.f;
            }
            for (int64_t q = 0; q < 2 * N; ++q) {
                dB_in[bi * 2 * N + q] = gB ? gB[bi * 2 * N + q] : 0.f;
                dC_in[bi * 2 * N + q] = gC ? gC[bi * 2 * N + q] : 0.f;
                dBc[bi * 2 * N + q] = 0.f;
                dCc[bi * 2 * N + q] = 0.f;
            }
            dt[bi] = 0.f;
            if (dcpi) dcpi[bi] = 0.f;
            continue;
        }
        const int first = !init_in[bi];
        const double tl = t[bi];
        const double t0 = first ? tl - (double)dt_init : (double)t_in[bi];
        double* u0 = (double*)malloc(sizeof(double) * (size_t)H);
        cd* B0 = (cd*)malloc(sizeof(cd) * (size_t)N);
        cd* C0 = (cd*)malloc(sizeof(cd) * (size_t)N);
        cd* Bf = (cd*)malloc(sizeof(cd) * (size_t)N);
        cd* Cf = (cd*)malloc(sizeof(cd) * (size_t)N);
        for (int64_t hh = 0; hh < H; ++hh) u0[hh] = first ? u[bi * H + hh] : u_in[bi * H + hh];
        for (int64_t n = 0; n < N; ++n) {
            Bf[n] = cd_of(Bc + (bi * N + n) * 2);
            Cf[n] = cd_of(Cc + (bi * N + n) * 2);
            B0[n] = first ? Bf[n] : cd_of(B_in + (bi * N + n) * 2);
            C0[n] = first ? Cf[n] : cd_of(C_in + (bi * N + n) * 2);
        }
        const double draw = tl - t0, delta = draw > 0 ? draw : 0;
        cd *dA = (cd*)malloc(sizeof(cd) * (size_t)HN), *E = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd *dB = (cd*)malloc(sizeof(cd) * (size_t)HN), *xh = (cd*)malloc(sizeof(cd) * (size_t)HN);
        cd *hu = (cd*)malloc(sizeof(cd) * (size_t)HN), *il = (cd*)malloc(sizeof(cd) * (size_t)HN);
        double *dte = (double*)malloc(sizeof(double) * (size_t)H), *sc = (double*)malloc(sizeof(double) * (size_t)H);
        double *obs = (double*)malloc(sizeof(double) * (size_t)H), *dv = (double*)malloc(sizeof(double) * (size_t)H);
        double *sd = (double*)malloc(sizeof(double) * (size_t)H), *mdt = (double*)malloc(sizeof(double) * (size_t)H);
        double sdiff = 0, sobs = 0;
        for (int64_t hh = 0; hh < H; ++hh) {
            sc[hh] = exp((double)log_dt[hh]);
            const double raw = delta * sc[hh];
            double v2 = raw < dt_min ? dt_min : raw;
            if (v2 > dt_max) v2 = dt_max;
            dte[hh] = v2;
            mdt[hh] = (raw >= dt_min && raw <= (double)dt_max) ? 1.0 : 0.0;
            double yh = 0;
            for (int64_t n = 0; n < N; ++n) {
                const int64_t i = hh * N + n;
                const cd lm = {lam[2 * i], lam[2 * i + 1]};
                const double d2 = lm.re * lm.re + lm.im * lm.im;
                il[i] = (cd){lm.re / d2, -lm.im / d2};
                const double a = lm.re * dte[hh], b = lm.im * dte[hh], e = exp(a);
                dA[i] = (cd){e * cos(b), e * sin(b)};
                E[i] = (cd){expm1(a) * cos(b) - 2 * sin(0.5 * b) * sin(0.5 * b), e * sin(b)};
                dB[i] = cd_mul(E[i], il[i]);
                const cd P = cd_mul(dA[i], cd_of(hs + 2 * i));
                xh[i] = cd_add(P, cd_scale(cd_mul(dB[i], B0[n]), u0[hh]));
                hu[i] = cd_add(P, cd_scale(cd_mul(dB[i], Bf[n]), u[bi * H + hh]));
                yh += C0[n].re * xh[i].re - C0[n].im * xh[i].im;
            }
            sd[hh] = sqrt((double)var[hh] + (double)var_eps);
            obs[hh] = (u[bi * H + hh] - mean[hh]) / sd[hh];
            dv[hh] = obs[hh] - (yh - mean[hh]) / sd[hh];
            sdiff += dv[hh] * dv[hh];
            sobs += obs[hh] * obs[hh];
        }
        const double num = sqrt(sdiff), nobs = sqrt(sobs), den = nobs + eta, r = num / den;
        double epsl = first ? -1.0 : (double)eps, e1 = epsl, cc = 0;
        const int mod = cpi != NULL && cpi_mod > 0.f;
        if (mod) {
            cc = cpi[bi] < 0 ? 0 : (cpi[bi] > 1 ? 1 : cpi[bi]);
            e1 = epsl * (1.0 - cpi_mod * cc);
            epsl = e1 > 1e-3 ? e1 : 1e-3;
        }
        const double soft = 1.0 / (1.0 + exp(-((r - epsl) / Tp)));
        double g = gate_mode == 1 ? soft : (r > epsl ? 1.0 : 0.0);
        if (gate_mode != 1 && gs && !first) g = gs[bi];
        /* ---- adjoints ---- */
        double gbar = 0, dtl = 0, dt0 = 0;
        double *dul = (double*)calloc((size_t)H, sizeof(double)), *du0 = (double*)calloc((size_t)H, sizeof(double));
        cd *dBl = (cd*)calloc((size_t)N, sizeof(cd)), *dCl = (cd*)calloc((size_t)N, sizeof(cd));
        cd *aB0 = (cd*)calloc((size_t)N, sizeof(cd)), *aC0 = (cd*)calloc((size_t)N, sizeof(cd));
        cd *ahu = (cd*)calloc((size_t)HN, sizeof(cd)), *axh = (cd*)calloc((size_t)HN, sizeof(cd));
        cd *ah0 = (cd*)calloc((size_t)HN, sizeof(cd));
        double* alam = acc_lam + bi * HN * 2;
        double* alog = acc_log + bi * H;
        double* aD = acc_D + bi * H;
        for (int64_t hh = 0; hh < H; ++hh) {
            const double yb = gy ? gy[bi * H + hh] : 0.0, ul = u[bi * H + hh];
            dul[hh] += yb * D[hh];
            aD[hh] += yb * ul;
            for (int64_t n = 0; n < N; ++n) {
                const int64_t i = hh * N + n;
                const cd hc = cd_add(cd_scale(hu[i], g), cd_scale(xh[i], 1 - g));
                cd ahc = cd_scale(cd_conj(Cf[n]), yb);
                dCl[n] = cd_add(dCl[n], cd_scale(cd_conj(hc), yb));
                const cd Ah = gh ? cd_of(gh + (bi * HN + i) * 2) : (cd){0, 0};
                if (first) {
                    ahc = cd_add(ahc, Ah);
                } else {
                    ahu[i] = cd_add(ahu[i], cd_scale(Ah, g));
                    ah0[i] = cd_add(ah0[i], cd_scale(Ah, 1 - g));
                    gbar += cd_redot(Ah, cd_sub(hu[i], cd_of(hs + 2 * i)));
                }
                ahu[i] = cd_add(ahu[i], cd_scale(ahc, g));
                axh[i] = cd_add(axh[i], cd_scale(ahc, 1 - g));
                gbar += cd_redot(ahc, cd_sub(hu[i], xh[i]));
            }
        }
        const double At = gt ? gt[bi] : 0.0;
        if (first) {
            dtl += At;
            for (int64_t hh = 0; hh < H; ++hh) dul[hh] += gu ? gu[bi * H + hh] : 0.0;
            for (int64_t n = 0; n < N; ++n) {
                if (gB) dBl[n] = cd_add(dBl[n], cd_of(gB + (bi * N + n) * 2));
                if (gC) dCl[n] = cd_add(dCl[n], cd_of(gC + (bi * N + n) * 2));
            }
        } else {
            dtl += g * At;
            dt0 += (1 - g) * At;
            gbar += At * (tl - t0);
            for (int64_t hh = 0; hh < H; ++hh) {
                const double Au = gu ? gu[bi * H + hh] : 0.0;
                dul[hh] += g * Au;
                du0[hh] += (1 - g) * Au;
                gbar += Au * (u[bi * H + hh] - u0[hh]);
            }
            for (int64_t n = 0; n < N; ++n) {
                const cd AB = gB ? cd_of(gB + (bi * N + n) * 2) : (cd){0, 0};
                const cd AC = gC ? cd_of(gC + (bi * N + n) * 2) : (cd){0, 0};
                dBl[n] = cd_add(dBl[n], cd_scale(AB, g));
                aB0[n] = cd_add(aB0[n], cd_scale(AB, 1 - g));
                dCl[n] = cd_add(dCl[n], cd_scale(AC, g));
                aC0[n] = cd_add(aC0[n], cd_scale(AC, 1 - g));
                gbar += cd_redot(AB, cd_sub(Bf[n], B0[n])) + cd_redot(AC, cd_sub(Cf[n], C0[n]));
            }
            if (gg) gbar += gg[bi];
        }
        const double xbar = gate_mode == 2 ? 0.0 : gbar * soft * (1 - soft) / Tp;
        const double rbar = (gr ? gr[bi] : 0.0) + xbar;
        double dcp = 0;
        if (!first) {
            const double ebar = -xbar;
            if (mod) {
                if (e1 >= 1e-3) {
                    acc_eps[bi] += ebar * (1.0 - cpi_mod * cc);
                    if (cpi[bi] >= 0 && cpi[bi] <= 1) dcp = -ebar * (double)eps * cpi_mod;
                }
            } else {
                acc_eps[bi] += ebar;
            }
        }
        if (dcpi) dcpi[bi] = (float)dcp;
        const double nbar = (!first && gn) ? gn[bi] : 0.0;
        const double numbar = rbar / den, denbar = -rbar * num / (den * den), numnbar = nbar / den;
        double deltabar = 0;
        for (int64_t hh = 0; hh < H; ++hh) {
            const double dbar = num > 0 ? numbar * dv[hh] / num : 0.0;
            const double obar = dbar + (nobs > 0 ? denbar * obs[hh] / nobs : 0.0);
            const double pbar = -dbar - (num > 0 ? numnbar * dv[hh] / num : 0.0);
            dul[hh] += obar / sd[hh];
            const double yhb = pbar / sd[hh];
            const double ul = u[bi * H + hh];
            double dtebar = 0;
            for (int64_t n = 0; n < N; ++n) {
                const int64_t i = hh * N + n;
                axh[i] = cd_add(axh[i], cd_scale(cd_conj(C0[n]), yhb));
                aC0[n] = cd_add(aC0[n], cd_scale(cd_conj(xh[i]), yhb));
                const cd aP = cd_add(axh[i], ahu[i]);
                const cd qp = cd_mul(dB[i], B0[n]), qc = cd_mul(dB[i], Bf[n]);
                const cd aqp = cd_scale(axh[i], u0[hh]), aqc = cd_scale(ahu[i], ul);
                du0[hh] += cd_redot(axh[i], qp);
                dul[hh] += cd_redot(ahu[i], qc);
                const cd adB = cd_add(cd_mul(aqp, cd_conj(B0[n])), cd_mul(aqc, cd_conj(Bf[n])));
                aB0[n] = cd_add(aB0[n], cd_mul(cd_conj(dB[i]), aqp));
                dBl[n] = cd_add(dBl[n], cd_mul(cd_conj(dB[i]), aqc));
                const cd h0 = cd_of(hs + 2 * i);
                const cd adA = cd_mul(aP, cd_conj(h0));
                ah0[i] = cd_add(ah0[i], cd_mul(cd_conj(dA[i]), aP));
                const cd aE = cd_mul(adB, cd_conj(il[i]));
                const cd ail = cd_mul(adB, cd_conj(E[i]));
                cd alm = cd_scale(cd_mul(cd_conj(cd_mul(il[i], il[i])), ail), -1.0);
                const cd az = cd_mul(cd_conj(dA[i]), cd_add(adA, aE));
                alm = cd_add(alm, cd_scale(az, dte[hh]));
                const cd lm = {lam[2 * i], lam[2 * i + 1]};
                dtebar += cd_redot(az, lm);
                alam[2 * i] += alm.re;
                alam[2 * i + 1] += alm.im;
            }
            const double drb = mdt[hh] * dtebar;
            alog[hh] += drb * delta * sc[hh];
            deltabar += drb * sc[hh];
        }
        const double mdel = draw >= 0 ? 1.0 : 0.0;
        dtl += mdel * deltabar;
        dt0 -= mdel * deltabar;
        if (first) {
            dtl += dt0;
            for (int64_t hh = 0; hh < H; ++hh) dul[hh] += du0[hh];
            for (int64_t n = 0; n < N; ++n) {
                dBl[n] = cd_add(dBl[n], aB0[n]);
                dCl[n] = cd_add(dCl[n], aC0[n]);
            }
            dt_in[bi] = 0.f;
            for (int64_t hh = 0; hh < H; ++hh) du_in[bi * H + hh] = 0.f;
            for (int64_t q = 0; q < 2 * N; ++q) { dB_in[bi * 2 * N + q] = 0.f; dC_in[bi * 2 * N + q] = 0.f; }
        } else {
            dt_in[bi] = (float)dt0;
            for (int64_t hh = 0; hh < H; ++hh) du_in[bi * H + hh] = (float)du0[hh];
            for (int64_t n = 0; n < N; ++n) {
                dB_in[(bi * N + n) * 2] = (float)aB0[n].re;
                dB_in[(bi * N + n) * 2 + 1] = (float)aB0[n].im;
                dC_in[(bi * N + n) * 2] = (float)aC0[n].re;
                dC_in[(bi * N + n) * 2 + 1] = (float)aC0[n].im;
            }
        }
        dt[bi] = (float)dtl;
        for (int64_t hh = 0; hh < H; ++hh) du[bi * H + hh] = (float)dul[hh];
        for (int64_t n = 0; n < N; ++n) {
            dBc[(bi * N + n) * 2] = (float)dBl[n].re;
            dBc[(bi * N + n) * 2 + 1] = (float)dBl[n].im;
            dCc[(bi * N + n) * 2] = (float)dCl[n].re;
            dCc[(bi * N + n) * 2 + 1] = (float)dCl[n].im;
        }
        for (int64_t i = 0; i < HN; ++i) {
            dhs[2 * i] = (float)ah0[i].re;
            dhs[2 * i + 1] = (float)ah0[i].im;
        }
        free(u0); free(B0); free(C0); free(Bf); free(Cf); free(dA); free(E); free(dB); free(xh);
        free(hu); free(il); free(dte); free(sc); free(obs); free(dv); free(sd); free(mdt);
        free(dul); free(du0); free(dBl); free(dCl); free(aB0); free(aC0); free(ahu); free(axh); free(ah0);
    }
    for (int64_t i = 0; i < HN * 2; ++i) {
        double s = 0;
        for (int64_t bi = 0; bi < B; ++bi) s += acc_lam[bi * HN * 2 + i];
        dlam[i] = (float)s;
    }
    for (int64_t hh = 0; hh < H; ++hh) {
        double s = 0, s2 = 0;
        for (int64_t bi = 0; bi < B; ++bi) { s += acc_log[bi * H + hh]; s2 += acc_D[bi * H + hh]; }
        dlog[hh] = (float)s;
        dD[hh] = (float)s2;
    }
    double se = 0;
    for (int64_t bi = 0; bi < B; ++bi) se += acc_eps[bi];
    deps[0] = (float)se;
    free(acc_lam); free(acc_log); free(acc_D); free(acc_eps);
    return 0;
}

const char* eacs_oracle_version(void) { return "eacs-oracle 2"; }
