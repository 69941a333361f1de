// capi.cu -- the extern "C" entry points of libeacs_b200.so (include/eacs_b200.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/eacs_b200.h"
#include "eacs_host.h"

namespace eacs {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};
static thread_local cudaEvent_t g_ev_start = nullptr;
static thread_local cudaEvent_t g_ev_stop = nullptr;

void note_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }
void mark_start(cudaStream_t s) {
    if (g_ev_start && g_ev_stop) cudaEventRecord(g_ev_start, s);
}
void mark_stop(cudaStream_t s) {
    if (g_ev_start && g_ev_stop) cudaEventRecord(g_ev_stop, s);
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return EACS_OK;
    return fail(EACS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

}  // namespace eacs

extern "C" {

const char* eacs_version(void) { return "eacs_b200 0.1.0 (sm_100a)"; }

const char* eacs_last_error(void) { return eacs::g_last_error.c_str(); }

uint64_t eacs_kernel_launches(void) { return eacs::g_launches.load(std::memory_order_relaxed); }

int eacs_set_kernel_events(void* start, void* stop) {
    eacs::g_ev_start = static_cast<cudaEvent_t>(start);
    eacs::g_ev_stop = static_cast<cudaEvent_t>(stop);
    return EACS_OK;
}

int eacs_device_status(int* status, void* stream) {
    if (!status) return eacs::fail(EACS_ERR_INVALID, "eacs_device_status: null status pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int a = 0, b = 0;
    int rc = eacs::cuda_check(eacs::scan_read_status(&a, s), "eacs_device_status");
    if (rc) return rc;
    rc = eacs::cuda_check(eacs::cell_read_status(&b, s), "eacs_device_status");
    if (rc) return rc;
    int c = 0, d = 0;
    rc = eacs::cuda_check(eacs::train_read_status(&c, s), "eacs_device_status");
    if (rc) return rc;
    rc = eacs::cuda_check(eacs::query_read_status(&d, s), "eacs_device_status");
    if (rc) return rc;
    *status = a ? a : (b ? b : (c ? c : d));
    return EACS_OK;
}

size_t eacs_project_workspace_size(int64_t M) { return eacs::project_workspace_size(M); }

int eacs_project(const void* x, int x_dtype, const float* gamma, const float* beta, float ln_eps,
                 const void* weight, int w_dtype, int64_t w_rows, const float* bias, void* u, int u_dtype,
                 void* Bc, void* Cc, void* workspace, size_t workspace_bytes, int64_t M, int64_t d, int64_t H,
                 int64_t N, void* stream) {
    eacs::ProjectCall c{x, x_dtype, gamma, beta, ln_eps, weight, w_dtype, w_rows, bias, u, u_dtype, Bc, Cc,
                        M, d, H, N, workspace, workspace_bytes};
    return eacs::project_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_wait_selftest(int polls, void* stream) {
    return eacs::wait_selftest(polls, static_cast<cudaStream_t>(stream));
}

int eacs_scan_fwd(const void* a, const void* b, void* h, int64_t B, int64_t L, int64_t H, int64_t N,
                  void* stream) {
    if (B < 0 || L < 0 || H < 0 || N < 0) return eacs::fail(EACS_ERR_INVALID, "eacs_scan_fwd: negative size");
    return eacs::scan_fwd(a, b, h, B, L, H * N, static_cast<cudaStream_t>(stream));
}

int eacs_scan_bwd(const void* a, const void* h, const void* grad_h, void* grad_a, void* grad_b,
                  int64_t B, int64_t L, int64_t H, int64_t N, void* stream) {
    if (B < 0 || L < 0 || H < 0 || N < 0) return eacs::fail(EACS_ERR_INVALID, "eacs_scan_bwd: negative size");
    return eacs::scan_bwd(a, h, grad_h, grad_a, grad_b, B, L, H * N, static_cast<cudaStream_t>(stream));
}

int eacs_ssm_fwd(const void* lam, const float* log_dt, const float* t, const void* Bc, const void* Cc,
                 const void* u, int u_dtype, const float* D, float* y, int64_t B, int64_t L, int64_t H,
                 int64_t N, float dt_min, float dt_max, void* stream) {
    return eacs::ssm_fwd(lam, log_dt, t, Bc, Cc, u, u_dtype, D, y, B, L, H, N, dt_min, dt_max,
                         nullptr, 0, static_cast<cudaStream_t>(stream));
}

size_t eacs_ssm_ckpt_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::ssm_ckpt_size(B, L, H, N);
}

int eacs_ssm_train_fwd(const void* lam, const float* log_dt, const float* t, const void* Bc,
                       const void* Cc, const void* u, int u_dtype, const float* D, float* y,
                       void* ckpt, size_t ckpt_bytes, int64_t B, int64_t L, int64_t H, int64_t N,
                       float dt_min, float dt_max, void* stream) {
    if (!ckpt) return eacs::fail(EACS_ERR_INVALID, "eacs_ssm_train_fwd: null checkpoint buffer");
    return eacs::ssm_fwd(lam, log_dt, t, Bc, Cc, u, u_dtype, D, y, B, L, H, N, dt_min, dt_max,
                         ckpt, ckpt_bytes, static_cast<cudaStream_t>(stream));
}

size_t eacs_ssm_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::ssm_bwd_workspace_size(B, L, H, N);
}

int eacs_ssm_bwd(const void* lam, const float* log_dt, const float* t, const void* Bc, const void* Cc,
                 const void* u, int u_dtype, const float* D, const float* gy, const void* ckpt,
                 size_t ckpt_bytes, float* du, void* dBc, void* dCc, float* dt, void* dlam,
                 float* dlog_dt, float* dD, void* workspace, size_t workspace_bytes, int64_t B,
                 int64_t L, int64_t H, int64_t N, float dt_min, float dt_max, void* stream) {
    eacs::SsmBwdCall c{lam, log_dt, t,  Bc,   Cc,      u,  u_dtype, D,         gy,
                       ckpt, ckpt_bytes, du, dBc, dCc, dt, dlam, dlog_dt, dD, workspace,
                       workspace_bytes, B, L, H, N, dt_min, dt_max};
    return eacs::ssm_bwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_zoh_kernels(const void* lam, const float* dt, void* dA, void* dB_bar, int64_t M, int64_t H,
                     int64_t N, void* stream) {
    return eacs::zoh_kernels(lam, dt, dA, dB_bar, M, H, N, static_cast<cudaStream_t>(stream));
}

size_t eacs_cell_fwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::cell_workspace_size(B, L, H, N);
}

int eacs_cell_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                  const void* Cc, const float* t, const float* D, const float* mean, const float* var,
                  float eps, float eta, float var_eps, float dt_init, float dt_min, float dt_max,
                  int robust, int robust_k, float spike_ratio, float eps_factor, int gate_mode,
                  float temperature, float* y, float* gate, float* resid, void* workspace,
                  size_t workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t N, void* stream) {
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,          t,           D,
                     mean, var,    eps,     eta,     var_eps, dt_init,    dt_min,      dt_max,
                     robust, robust_k, spike_ratio, eps_factor, gate_mode, temperature, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    return eacs::cell_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_cell_fwd_side_by_side(const void* lam, const float* log_dt, const void* u, int u_dtype,
                               const void* Bc, const void* Cc, const float* t, const float* D,
                               const float* mean, const float* var, float eps, float eta,
                               float var_eps, float dt_init, float dt_min, float dt_max, int robust,
                               int robust_k, float spike_ratio, float eps_factor, int gate_mode,
                               float temperature, float* y, float* gate, float* resid,
                               void* workspace, size_t workspace_bytes, int64_t B, int64_t L,
                               int64_t H, int64_t N, int cells_side_by_side, void* stream) {
    if (cells_side_by_side < 1)
        return eacs::fail(EACS_ERR_INVALID, "eacs_cell_fwd_side_by_side: cells_side_by_side must be >= 1");
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,          t,           D,
                     mean, var,    eps,     eta,     var_eps, dt_init,    dt_min,      dt_max,
                     robust, robust_k, spike_ratio, eps_factor, gate_mode, temperature, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    c.side_by_side = cells_side_by_side;
    return eacs::cell_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_cell_train_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                        const void* Cc, const float* t, const float* D, const float* mean,
                        const float* var, float eps, float eta, float var_eps, float dt_init,
                        float dt_min, float dt_max, int gate_mode, float temperature, float* y,
                        float* gate, float* resid, float* stats, void* workspace,
                        size_t workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t N,
                        void* stream) {
    if (!stats) return eacs::fail(EACS_ERR_INVALID, "eacs_cell_train_fwd: null stats");
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,      t,      D,
                     mean, var,    eps,     eta,     var_eps, dt_init, dt_min, dt_max,
                     0,    3,      2.0f,    0.3f,    gate_mode, temperature, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    c.stats = stats;
    return eacs::cell_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_cell_train_fwd_ckpt(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                             const void* Cc, const float* t, const float* D, const float* mean,
                             const float* var, float eps, float eta, float var_eps, float dt_init,
                             float dt_min, float dt_max, int gate_mode, float temperature, float* y,
                             float* gate, float* resid, float* stats, void* workspace,
                             size_t workspace_bytes, void* bwd_workspace, size_t bwd_workspace_bytes,
                             int64_t B, int64_t L, int64_t H, int64_t N, void* stream) {
    if (!stats) return eacs::fail(EACS_ERR_INVALID, "eacs_cell_train_fwd_ckpt: null stats");
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,      t,      D,
                     mean, var,    eps,     eta,     var_eps, dt_init, dt_min, dt_max,
                     0,    3,      2.0f,    0.3f,    gate_mode, temperature, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    c.stats = stats;
    if (B == 0 || L == 0 || H == 0) return EACS_OK;
    const int rc = eacs::train_ckpt_layout(B, L, H, N, bwd_workspace, bwd_workspace_bytes, &c);
    if (rc) return rc;
    return eacs::cell_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_cell_train_bwd_ckpt(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                             const void* Cc, const float* t, const float* D, const float* mean,
                             const float* var, float eps, float eta, float var_eps, float dt_init,
                             float dt_min, float dt_max, float temperature, const float* gate,
                             const float* resid, const float* stats, const float* gy, const float* ggs,
                             const float* grs, const float* gns, float* du, void* dBc, void* dCc,
                             float* dt, void* dlam, float* dlog_dt, float* dD, float* deps,
                             void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                             int64_t N, void* stream) {
    eacs::TrainBwdCall c{lam,   log_dt, u,     u_dtype, Bc,      Cc,     t,      D,       mean,
                         var,   eps,    eta,   var_eps, dt_init, dt_min, dt_max, temperature,
                         gate,  resid,  stats, gy,      ggs,     grs,    gns,    du,      dBc,
                         dCc,   dt,     dlam,  dlog_dt, dD,      deps,   workspace, workspace_bytes,
                         B,     L,      H,     N};
    c.have_ckpt = true;
    return eacs::train_bwd(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_cell_train_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::train_workspace_size(B, L, H, N);
}

int eacs_cell_train_bwd(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                        const void* Cc, const float* t, const float* D, const float* mean,
                        const float* var, float eps, float eta, float var_eps, float dt_init,
                        float dt_min, float dt_max, float temperature, const float* gate,
                        const float* resid, const float* stats, const float* gy, const float* ggs,
                        const float* grs, const float* gns, float* du, void* dBc, void* dCc,
                        float* dt, void* dlam, float* dlog_dt, float* dD, float* deps,
                        void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                        int64_t N, void* stream) {
    eacs::TrainBwdCall c{lam,   log_dt, u,     u_dtype, Bc,      Cc,     t,      D,       mean,
                         var,   eps,    eta,   var_eps, dt_init, dt_min, dt_max, temperature,
                         gate,  resid,  stats, gy,      ggs,     grs,    gns,    du,      dBc,
                         dCc,   dt,     dlam,  dlog_dt, dD,      deps,   workspace, workspace_bytes,
                         B,     L,      H,     N};
    return eacs::train_bwd(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_cell_train_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::train_commits_workspace_size(B, L, H, N);
}

int eacs_cell_train_commits_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                const void* Bc, const void* Cc, const float* t, const float* D,
                                const float* mean, const float* var, float eps, float eta, float var_eps,
                                float dt_init, float dt_min, float dt_max, int gate_mode, float temperature,
                                float* y, float* gate, float* resid, float* stats, void* commit_h,
                                float* commit_t, float* commit_u, void* commit_B, void* commit_C,
                                void* workspace, size_t workspace_bytes, void* bwd_workspace,
                                size_t bwd_workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t N,
                                void* stream) {
    const char* fn = "eacs_cell_train_commits_fwd";
    if (!stats) return eacs::fail(EACS_ERR_INVALID, "%s: null stats", fn);
    if (gate_mode < 0 || gate_mode > 2) return eacs::fail(EACS_ERR_INVALID, "%s: gate_mode %d not in 0..2", fn, gate_mode);
    if (gate_mode == 2) gate_mode = 0;  // the hard gate's forward is the STE forward
    if (B < 0 || L < 0 || H < 0 || N < 0) return eacs::fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (B == 0 || L == 0 || H == 0) return EACS_OK;
    const size_t need = eacs::train_commits_workspace_size(B, L, H, N);
    if (need == 0)
        return eacs::fail(EACS_ERR_UNSUPPORTED, "%s: no training backward for B=%lld L=%lld H=%lld N=%lld", fn,
                          (long long)B, (long long)L, (long long)H, (long long)N);
    if (!bwd_workspace || bwd_workspace_bytes < need)
        return eacs::fail(EACS_ERR_WORKSPACE, "%s: backward workspace of %zu bytes needed, %zu given", fn, need,
                          bwd_workspace_bytes);
    if (!commit_h || !commit_t || !commit_u || !commit_B || !commit_C)
        return eacs::fail(EACS_ERR_INVALID, "%s: null commit buffer", fn);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,      t,      D,
                     mean, var,    eps,     eta,     var_eps, dt_init, dt_min, dt_max,
                     0,    3,      2.0f,    0.3f,    gate_mode, temperature, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    c.stats = stats;
    int rc = eacs::cell_fwd(c, s);
    if (rc) return rc;
    eacs::TrainBwdCall r{};
    r.lam = lam;
    r.log_dt = log_dt;
    r.u = u;
    r.u_dtype = u_dtype;
    r.Bc = Bc;
    r.Cc = Cc;
    r.t = t;
    r.D = D;
    r.mean = mean;
    r.var = var;
    r.eps = eps;
    r.eta = eta;
    r.var_eps = var_eps;
    r.dt_init = dt_init;
    r.dt_min = dt_min;
    r.dt_max = dt_max;
    r.temperature = temperature;
    r.gates = gate;
    r.workspace = bwd_workspace;
    r.workspace_bytes = bwd_workspace_bytes;
    r.B = B;
    r.L = L;
    r.H = H;
    r.N = N;
    eacs::CommitOut out{commit_h, commit_t, commit_u, commit_B, commit_C};
    return eacs::train_commits_replay(r, out, s);
}

int eacs_cell_train_commits_bwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                const void* Bc, const void* Cc, const float* t, const float* D,
                                const float* mean, const float* var, float eps, float eta, float var_eps,
                                float dt_init, float dt_min, float dt_max, int gate_mode, float temperature,
                                const float* gate, const float* resid, const float* stats, const float* gy,
                                const float* ggs, const float* grs, const void* g_commit_h,
                                const float* g_commit_t, const float* g_commit_u, const void* g_commit_B,
                                const void* g_commit_C, float* du, void* dBc, void* dCc, float* dt,
                                void* dlam, float* dlog_dt, float* dD, float* deps, void* workspace,
                                size_t workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t N,
                                void* stream) {
    eacs::TrainBwdCall c{lam,   log_dt, u,     u_dtype, Bc,      Cc,     t,       D,       mean,
                         var,   eps,    eta,   var_eps, dt_init, dt_min, dt_max,  temperature,
                         gate,  resid,  stats, gy,      ggs,     grs,    nullptr, du,      dBc,
                         dCc,   dt,     dlam,  dlog_dt, dD,      deps,   workspace, workspace_bytes,
                         B,     L,      H,     N};
    if (gate_mode < 0 || gate_mode > 2)
        return eacs::fail(EACS_ERR_INVALID, "eacs_cell_train_commits_bwd: gate_mode %d not in 0..2", gate_mode);
    c.commits = true;
    c.gate_const = gate_mode == 2;
    c.gc_h = g_commit_h;
    c.gc_t = g_commit_t;
    c.gc_u = g_commit_u;
    c.gc_B = g_commit_B;
    c.gc_C = g_commit_C;
    return eacs::train_bwd(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_query_readout_bwd_workspace_size(int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N) {
    return eacs::query_readout_bwd_workspace_size(B, L, Q, H, N);
}

int eacs_query_readout_bwd(const void* lam, const float* log_dt, const float* D, const void* commit_h,
                           const float* commit_t, const float* commit_u, const void* commit_B,
                           const void* commit_C, const float* t_query, const int32_t* idx, const float* gy,
                           void* g_commit_h, float* g_commit_t, float* g_commit_u, void* g_commit_B,
                           void* g_commit_C, float* g_t_query, void* dlam, float* dlog_dt, float* dD,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t Q,
                           int64_t H, int64_t N, float dt_min, float dt_max, void* stream) {
    eacs::QueryBwdCall c{lam,        log_dt,     D,          commit_h,   commit_t,   commit_u,
                         commit_B,   commit_C,   t_query,    idx,        gy,         g_commit_h,
                         g_commit_t, g_commit_u, g_commit_B, g_commit_C, g_t_query,  dlam,
                         dlog_dt,    dD,         workspace,  workspace_bytes, B,     L,
                         Q,          H,          N,          dt_min,     dt_max};
    return eacs::query_readout_bwd(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_cell_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N) {
    return eacs::cell_commits_workspace_size(B, L, H, N);
}

int eacs_cell_commits(const void* lam, const float* log_dt, const void* u, int u_dtype, const void* Bc,
                      const void* Cc, const float* t, const float* D, const float* mean,
                      const float* var, float eps, float eta, float var_eps, float dt_init,
                      float dt_min, float dt_max, int robust, int robust_k, float spike_ratio,
                      float eps_factor, float* y, float* gate, float* resid, void* commit_h,
                      float* commit_t, float* commit_u, void* commit_B, void* commit_C,
                      void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                      int64_t N, void* stream) {
    if (!commit_h) return eacs::fail(EACS_ERR_INVALID, "eacs_cell_commits: null commit_h");
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,          t,           D,
                     mean, var,    eps,     eta,     var_eps, dt_init,    dt_min,      dt_max,
                     robust, robust_k, spike_ratio, eps_factor, 0, 0.1f, y, gate,
                     resid, workspace, workspace_bytes, B, L, H, N};
    c.commit_h = commit_h;
    c.commit_t = commit_t;
    c.commit_u = commit_u;
    c.commit_B = commit_B;
    c.commit_C = commit_C;
    return eacs::cell_fwd(c, static_cast<cudaStream_t>(stream));
}

int eacs_query_index(const float* frame_t, const float* t_query, int32_t* idx, int64_t B, int64_t L,
                     int64_t Q, void* stream) {
    return eacs::query_index(frame_t, t_query, idx, B, L, Q, static_cast<cudaStream_t>(stream));
}

int eacs_query_readout(const void* lam, const float* log_dt, const float* D, const void* commit_h,
                       const float* commit_t, const float* commit_u, const void* commit_B,
                       const void* commit_C, const float* t_query, const int32_t* idx, float* y,
                       int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N, float dt_min,
                       float dt_max, void* stream) {
    return eacs::query_readout(lam, log_dt, D, commit_h, commit_t, commit_u, commit_B, commit_C,
                               t_query, idx, y, B, L, Q, H, N, dt_min, dt_max,
                               static_cast<cudaStream_t>(stream));
}

int eacs_stream_chunk(const void* lam, const float* log_dt, const float* D, const float* mean,
                      const float* var, const void* u, int u_dtype, const void* Bc, const void* Cc,
                      const float* t, const uint8_t* valid, const float* cpi, const void* h_in,
                      const float* t_in, const float* u_in, const void* B_in, const void* C_in,
                      const uint8_t* init_in, void* h_out, float* t_out, float* u_out, void* B_out,
                      void* C_out, uint8_t* init_out, float* y, float* gate, float* resid,
                      float* innov, float eps, float eta, float var_eps, float dt_init, float dt_min,
                      float dt_max, float cpi_modulation, int gate_mode, float temperature,
                      int64_t B, int64_t K, int64_t H, int64_t N, void* stream) {
    eacs::StreamCall c{lam,   log_dt, D,       mean,    var,      u,      u_dtype, Bc,    Cc,
                       t,     valid,  cpi,     h_in,    t_in,     u_in,   B_in,    C_in,  init_in,
                       h_out, t_out,  u_out,   B_out,   C_out,    init_out, y,     gate,  resid,
                       innov, eps,    eta,     var_eps, dt_init,  dt_min, dt_max,  cpi_modulation,
                       temperature, gate_mode, B, K, H, N};
    return eacs::stream_chunk(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_stream_step_bwd_workspace_size(int64_t B, int64_t H, int64_t N) {
    return eacs::stream_step_bwd_workspace_size(B, H, N);
}

int eacs_stream_step_bwd(const void* lam, const float* log_dt, const float* D, const float* mean,
                         const float* var, const float* u, const void* Bc, const void* Cc, const float* t,
                         const uint8_t* valid, const float* cpi, const void* h_in, const float* t_in,
                         const float* u_in, const void* B_in, const void* C_in, const uint8_t* init_in,
                         const float* gate, const float* gy, const float* gg, const float* gr,
                         const float* gn, const void* gh, const float* gt, const float* gu, const void* gB,
                         const void* gC, float* du, void* dBc, void* dCc, float* dt, float* dcpi,
                         void* dh_in, float* dt_in, float* du_in, void* dB_in, void* dC_in, void* dlam,
                         float* dlog_dt, float* dD, float* deps, void* workspace, size_t workspace_bytes,
                         float eps, float eta, float var_eps, float dt_init, float dt_min, float dt_max,
                         float cpi_modulation, int gate_mode, float temperature, int64_t B, int64_t H,
                         int64_t N, void* stream) {
    eacs::StreamBwdCall c{lam,   log_dt, D,      mean,    var,    u,     Bc,      Cc,      t,
                          valid, cpi,    h_in,   t_in,    u_in,   B_in,  C_in,    init_in, gate,
                          gy,    gg,     gr,     gn,      gh,     gt,    gu,      gB,      gC,
                          du,    dBc,    dCc,    dt,      dcpi,   dh_in, dt_in,   du_in,   dB_in,
                          dC_in, dlam,   dlog_dt, dD,     deps,   workspace, workspace_bytes,
                          eps,   eta,    var_eps, dt_init, dt_min, dt_max, cpi_modulation, temperature,
                          gate_mode, B,  H,      N};
    return eacs::stream_step_bwd(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_stream_frame_workspace_size(const EacsFrameBranch* branches, int S, int64_t B, int64_t d) {
    return eacs::stream_frame_workspace_size(branches, S, B, d);
}

int eacs_stream_frame(const float* x, const float* t, const uint8_t* valid, const float* cpi,
                      const EacsFrameBranch* branches, int S, const float* fusion_w, const float* fusion_b,
                      const float* out_norm_w, const float* out_norm_b, float out_norm_eps, float* y,
                      float* weights, float* gate, float* resid, float* innov, void* workspace,
                      size_t workspace_bytes, int64_t B, int64_t d, void* stream) {
    eacs::FrameCall c{x,        t,          valid,      cpi,   branches, S,      fusion_w, fusion_b,
                      out_norm_w, out_norm_b, out_norm_eps, y,   weights,  gate,   resid,    innov,
                      workspace, workspace_bytes, B,    d};
    return eacs::stream_frame(c, static_cast<cudaStream_t>(stream));
}

size_t eacs_cell_fwd_host_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N, int64_t chunk) {
    return eacs::cell_host_workspace_size(B, L, H, N, chunk);
}

int eacs_cell_fwd_host(const void* lam, const float* log_dt, const float* D, const float* mean,
                       const float* var, const void* u, int u_dtype, const void* Bc, const void* Cc,
                       const float* t, float eps, float eta, float var_eps, float dt_init,
                       float dt_min, float dt_max, int robust, int robust_k, float spike_ratio,
                       float eps_factor, float* y, float* gate, float* resid, void* workspace,
                       size_t workspace_bytes, int64_t B, int64_t L, int64_t H, int64_t N,
                       int64_t chunk, void* stream) {
    eacs::CellHostCall c{lam,   log_dt, D,       mean,    var,    u,           u_dtype,
                         Bc,    Cc,     t,       eps,     eta,    var_eps,     dt_init,
                         dt_min, dt_max, robust, robust_k, spike_ratio, eps_factor, y,
                         gate,  resid,  workspace, workspace_bytes, B, L, H, N, chunk};
    return eacs::cell_fwd_host(c, static_cast<cudaStream_t>(stream));
}

int eacs_branch_fuse(const void* x, const void* const* deltas, int S, int dtype,
                     const float* fusion_weight, const float* fusion_bias, const float* ln_weight,
                     const float* ln_bias, float ln_eps, void* y, float* weights, int64_t rows,
                     int64_t d, void* stream) {
    if (S <= 0 || S > 8 || !deltas)
        return eacs::fail(EACS_ERR_INVALID, "eacs_branch_fuse: S=%d outside 1..8 or no branch outputs", S);
    if (d <= 0 || d > (1 << 20)) return eacs::fail(EACS_ERR_INVALID, "eacs_branch_fuse: d=%lld", (long long)d);
    eacs::FuseCall c{};
    c.x = x;
    for (int s = 0; s < S; ++s) c.delta[s] = deltas[s];
    c.S = S;
    c.dtype = dtype;
    c.wf = fusion_weight;
    c.bf = fusion_bias;
    c.gamma = ln_weight;
    c.beta = ln_bias;
    c.ln_eps = ln_eps;
    c.y = y;
    c.w = weights;
    c.rows = rows;
    c.d = static_cast<int>(d);
    return eacs::branch_fuse(c, static_cast<cudaStream_t>(stream));
}

int eacs_cell_fwd_noalloc(const void* lam, const float* log_dt, const void* u, int u_dtype,
                          const void* Bc, const void* Cc, const float* t, const float* D,
                          const float* mean, const float* var, float eps, float eta, float var_eps,
                          float dt_init, float dt_min, float dt_max, int robust, int robust_k,
                          float spike_ratio, float eps_factor, int gate_mode, float temperature,
                          float* y, float* gate, float* resid, int64_t B, int64_t L, int64_t H,
                          int64_t N, void* stream) {
    eacs::CellCall c{lam,  log_dt, u,       u_dtype, Bc,     Cc,          t,           D,
                     mean, var,    eps,     eta,     var_eps, dt_init,    dt_min,      dt_max,
                     robust, robust_k, spike_ratio, eps_factor, gate_mode, temperature, y, gate,
                     resid, nullptr, 0, B, L, H, N};
    return eacs::cell_fwd_noalloc(c, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
