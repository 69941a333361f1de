/*
 * eacs_b200.h -- C ABI of the B200 (sm_100a) EACS temporal hot path.
 *
 * Plain pointers and sizes only.  Every pointer is a device pointer on the
 * current CUDA device unless noted; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  Complex tensors are complex64 (interleaved float pairs).
 * Shapes: lam (H,N), log_dt/D/mean/var (H), u (B,L,H), Bc/Cc (B,L,N),
 * t (B,L), y (B,L,H), gate/resid (B,L), scan tensors (B,L,H,N).  All tensors
 * are dense row-major (C-contiguous).
 *
 * Every entry point returns EACS_OK or an error code; a message for the last
 * failure on the calling thread is available from eacs_last_error().  Nothing
 * here allocates device memory unless stated: outputs and workspaces are the
 * caller's.  Calls are asynchronous on `stream`.
 *
 * Reference interface each entry replaces (paths inside the CST-SSM project,
 * BitGao-ai/LongVideo-main) is cited on the declaration.
 */
#ifndef EACS_B200_H
#define EACS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EACS_API __attribute__((visibility("default")))
#else
#define EACS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define EACS_OK 0
#define EACS_ERR_INVALID 1     /* bad shape, pointer, alignment or argument */
#define EACS_ERR_CUDA 2        /* a CUDA runtime call or kernel launch failed */
#define EACS_ERR_WORKSPACE 3   /* workspace missing or too small */
#define EACS_ERR_TIMEOUT 4     /* a bounded device-side wait expired */
#define EACS_ERR_UNSUPPORTED 5 /* shape outside what the kernels handle (e.g. N > 64) */

/* element types of the `u` input */
#define EACS_DTYPE_F32 0
#define EACS_DTYPE_F16 1
#define EACS_DTYPE_BF16 2

/* Library version string. */
EACS_API const char* eacs_version(void);

/* Message describing the last failing call on this host thread ("" if none). */
EACS_API const char* eacs_last_error(void);

/* Synchronises `stream`, then reads and clears the device status word that
 * kernels set instead of trapping (EACS_ERR_TIMEOUT for an expired bounded
 * wait).  *status receives EACS_OK when nothing was recorded. */
EACS_API int eacs_device_status(int* status, void* stream);

/* LayerNorm and the three input projections of an EACS layer in one kernel
 * on the tensor cores (tcgen05.mma, weights staged by TMA).  Replaces, for a
 * float16 / bfloat16 autocast region, x = self.norm(x) then _project(x)
 * (cst_ssm/modules/eacs.py:334 / :376 and :261-267): u = proj_u(x),
 * Bc = complex(b[..., :N], b[..., N:]) with b = proj_B(x), Cc likewise.
 * x (M, d) in x_dtype; gamma, beta (d) float32 (LayerNorm affine, eps ln_eps);
 * weight (w_rows, d) in w_dtype (float16 or bfloat16: the GEMM type T) holds
 * proj_u.weight (H rows), proj_B.weight (2N), proj_C.weight (2N), then zero
 * rows up to w_rows, a multiple of 256; bias (H + 4N) float32 likewise.
 * LayerNorm runs in float32 and is rounded to T; products accumulate in
 * float32, the bias (rounded to T) is added and the sum rounded to T, as an
 * autocast Linear does.  u (M, H) is written in u_dtype, Bc and Cc (M, N) as
 * complex64 of the T-rounded values.  d must be a multiple of 8; x, weight,
 * gamma and beta 16-byte aligned; workspace (8-byte aligned) of
 * eacs_project_workspace_size(M) bytes, the caller's. */
EACS_API int eacs_project(const void* x, int x_dtype, const float* gamma, const float* beta, float ln_eps,
                          const void* weight, int w_dtype, int64_t w_rows, const float* bias, void* u,
                          int u_dtype, void* Bc, void* Cc, void* workspace, size_t workspace_bytes,
                          int64_t M, int64_t d, int64_t H, int64_t N, void* stream);
/* Bytes of eacs_project's workspace for M rows (its LayerNorm statistics). */
EACS_API size_t eacs_project_workspace_size(int64_t M);

/* Failure-path check (no counterpart in the reference): one CTA waits, with
 * the library's bounded waits (CTA scope and cluster scope) limited to
 * `polls` polls (1..65536), on an mbarrier phase that nothing completes.
 * Both waits expire, record EACS_ERR_TIMEOUT in the device status word and
 * return, so the kernel ends and the context stays usable; a following
 * eacs_device_status() reports EACS_ERR_TIMEOUT once. */
EACS_API int eacs_wait_selftest(int polls, void* stream);

/* Number of kernel launches this library has issued in this process (all
 * devices).  Lets a caller prove the native path ran. */
EACS_API uint64_t eacs_kernel_launches(void);

/* Per host thread: when both events are non-NULL (cudaEvent_t), every later
 * call records `start` just before and `stop` just after its dominant kernel
 * (the chain kernel of eacs_cell_fwd / eacs_ssm_fwd, the scan kernel of
 * eacs_scan_fwd / eacs_scan_bwd) on the call's stream.  NULL, NULL turns it
 * off.  Used to time that kernel alone inside a larger call. */
EACS_API int eacs_set_kernel_events(void* start, void* stop);

/* Variable-step diagonal complex scan forward, h_l = a_l * h_{l-1} + b_l.
 * Replaces scan_fwd(a, b) -> [h] (cst_ssm/ops/csrc/eacs_scan_cuda.cu:62-77,
 * bound at eacs_scan_cuda.cu:98-101 and called from ops/scan_cuda.py:38-42).
 * a, b, h: (B,L,H,N) complex64. */
EACS_API int eacs_scan_fwd(const void* a, const void* b, void* h,
                  int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Reverse adjoint of the scan: s_l = g_l + conj(a_{l+1}) s_{l+1},
 * grad_b = s, grad_a = s * conj(h_{l-1}).
 * Replaces scan_bwd(a, h, grad_h) -> [grad_a, grad_b]
 * (cst_ssm/ops/csrc/eacs_scan_cuda.cu:79-96, called from ops/scan_cuda.py:44-49). */
EACS_API int eacs_scan_bwd(const void* a, const void* h, const void* grad_h,
                  void* grad_a, void* grad_b,
                  int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Zero-order-hold discretisation kernels: for lam (H,N) complex64 and
 * dt (M,H) float32, dA = exp(lam dt) and dB_bar = expm1(lam dt) / lam, each
 * (M,H,N) complex64, with expm1 in the branch-free form of
 * cst_ssm/ops/discretization.py:10-17.
 * Replaces zoh_kernels(lam, dt) -> (dA, dB_bar) (ops/discretization.py:20-36)
 * for callers that want the discretisation materialised; the fused kernels
 * below compute the same values in registers. */
EACS_API int eacs_zoh_kernels(const void* lam, const float* dt, void* dA, void* dB_bar,
                              int64_t M, int64_t H, int64_t N, void* stream);

/* Fused ungated continuous SSM core (ContinuousSSMLayer.forward,
 * cst_ssm/modules/continuous_ssm.py:44-55 with ops/discretization.py:20-82):
 * dt from timestamp differences (dt_0 = dt_1), ZOH discretisation, scan and
 * readout y = Re sum_n C h + D u, with no (B,L,H,N) tensor in memory.
 * lam (H,N) complex64, log_dt (H), t (B,L), Bc/Cc (B,L,N) complex64,
 * u (B,L,H) of u_dtype, D (H); y (B,L,H) float32. */
EACS_API int eacs_ssm_fwd(const void* lam, const float* log_dt, const float* t,
                 const void* Bc, const void* Cc, const void* u, int u_dtype,
                 const float* D, float* y,
                 int64_t B, int64_t L, int64_t H, int64_t N,
                 float dt_min, float dt_max, void* stream);

/* Bytes of the state checkpoints eacs_ssm_train_fwd writes for these sizes:
 * one (B,H,N) complex64 state every 8 steps, B*ceil(L/8)*H*N*8 bytes
 * (0 if the sizes are unsupported). */
EACS_API size_t eacs_ssm_ckpt_size(int64_t B, int64_t L, int64_t H, int64_t N);

/* Training forward of the fused ungated core: eacs_ssm_fwd, and also the
 * state before every 8th step into `ckpt` (ckpt_bytes >= eacs_ssm_ckpt_size)
 * for eacs_ssm_bwd.  Replaces the forward of ContinuousSSMLayer's core under
 * autograd (cst_ssm/modules/continuous_ssm.py:44-55), which keeps dA, dB*u
 * and h, three (B,L,H,N) complex64 tensors, for its backward
 * (ops/scan_cuda.py:36-49 saves a and h). */
EACS_API int eacs_ssm_train_fwd(const void* lam, const float* log_dt, const float* t,
                                const void* Bc, const void* Cc, const void* u, int u_dtype,
                                const float* D, float* y, void* ckpt, size_t ckpt_bytes,
                                int64_t B, int64_t L, int64_t H, int64_t N,
                                float dt_min, float dt_max, void* stream);

/* Workspace bytes eacs_ssm_bwd needs for these sizes (0 if unsupported). */
EACS_API size_t eacs_ssm_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);

/* Backward of the fused ungated core: given the forward's inputs, its
 * checkpoints and gy = dLoss/dy (B,L,H) float32, writes du (B,L,H) float32,
 * dBc, dCc (B,L,N) complex64, dt (B,L) float32 (the gradient of the
 * timestamps t), dlam (H,N) complex64, dlog_dt (H) and dD (H) float32, all
 * overwritten.  Replaces what autograd runs for continuous_ssm.py:44-55:
 * the readout's backward, scan_bwd (ops/csrc/eacs_scan_cuda.cu:79-96 via
 * ops/scan_cuda.py:44-49) and the backward of zoh_discretize /
 * effective_dt / the timestamp differences (ops/discretization.py:20-82).
 * Deterministic: partial sums are added in a fixed order. */
EACS_API int eacs_ssm_bwd(const void* lam, const float* log_dt, const float* t,
                          const void* Bc, const void* Cc, const void* u, int u_dtype,
                          const float* D, const float* gy, const void* ckpt, size_t ckpt_bytes,
                          float* du, void* dBc, void* dCc, float* dt, void* dlam,
                          float* dlog_dt, float* dD, void* workspace, size_t workspace_bytes,
                          int64_t B, int64_t L, int64_t H, int64_t N,
                          float dt_min, float dt_max, void* stream);

/* Workspace bytes eacs_cell_fwd needs for these sizes. */
EACS_API size_t eacs_cell_fwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);

/* Gated EACS cell forward over all L (event gate, ZOH predict/update,
 * commit, optional robust_guard).
 * Replaces eacs_cell_fwd(lam, log_dt, u, Bc, Cc, t, Dp, mean, var, eps, eta,
 * var_eps, dt_init, dt_min, dt_max) -> [y, gate, resid]
 * (cst_ssm/ops/csrc/eacs_cell_cuda.cu:170-223, called from
 * ops/eacs_gated_scan.py:35-49), and extends it with the semantics of
 * modules/eacs.py:145-173 (scan_range): robust != 0 enables robust_guard
 * (eps_l = eps*eps_factor after robust_k consecutive steps with
 * r_l > r_{l-1}*spike_ratio, eacs.py:155-170); gate_mode 1 selects the soft
 * gate sigmoid((r-eps)/max(T,1e-4)) blended into the state
 * (ops/eacs_cell_train.py:47-63).  gate_mode 0 is the hard gate r > eps_l.
 * Outputs y (B,L,H) float32, gate and resid (B,L) float32. */
EACS_API int eacs_cell_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                  const void* Bc, const void* Cc, const float* t, const float* D,
                  const float* mean, const float* var,
                  float eps, float eta, float var_eps, float dt_init,
                  float dt_min, float dt_max,
                  int robust, int robust_k, float spike_ratio, float eps_factor,
                  int gate_mode, float temperature,
                  float* y, float* gate, float* resid,
                  void* workspace, size_t workspace_bytes,
                  int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* eacs_cell_fwd for a caller that runs cells_side_by_side cells of this
 * shape at the same time on separate streams, this one included (the
 * branches of MultiScaleEACS, modules/multiscale.py:162-179, which the
 * reference runs one after another).  Same arguments, workspace and
 * results as eacs_cell_fwd (outputs equal to its tolerance: the layout
 * changes the order of the residual and readout sums); the count only picks
 * the layout of the speculative pass, so that the cells' CTAs together fit
 * the GPU in one wave.  cells_side_by_side < 1 is EACS_ERR_INVALID; 1 is
 * eacs_cell_fwd. */
EACS_API int eacs_cell_fwd_side_by_side(const void* lam, const float* log_dt, const void* u,
                  int u_dtype, const void* Bc, const void* Cc, const float* t, const float* D,
                  const float* mean, const float* var,
                  float eps, float eta, float var_eps, float dt_init,
                  float dt_min, float dt_max,
                  int robust, int robust_k, float spike_ratio, float eps_factor,
                  int gate_mode, float temperature,
                  float* y, float* gate, float* resid,
                  void* workspace, size_t workspace_bytes,
                  int64_t B, int64_t L, int64_t H, int64_t N, int cells_side_by_side,
                  void* stream);

/* Training forward of the gated cell: eacs_cell_fwd plus, in `stats`
 * (B,L,2) float32, the two norms of each step's residual
 * (||obs - pred||, ||obs||) that the backward needs.  gate_mode 0 gives the
 * straight-through forward (hard gate values), 1 the soft gate.
 * Replaces the forward of GatedEACSCellFunction
 * (cst_ssm/ops/eacs_cell_train.py:81-115: ys, gs, rs; its fourth output, the
 * stop-target innovation, has the values of rs). */
EACS_API int eacs_cell_train_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                 const void* Bc, const void* Cc, const float* t, const float* D,
                                 const float* mean, const float* var,
                                 float eps, float eta, float var_eps, float dt_init,
                                 float dt_min, float dt_max, int gate_mode, float temperature,
                                 float* y, float* gate, float* resid, float* stats,
                                 void* workspace, size_t workspace_bytes,
                                 int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Workspace bytes eacs_cell_train_bwd needs for these sizes (0 if the sizes
 * are unsupported). */
EACS_API size_t eacs_cell_train_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);

/* Backward of the gated cell: the vector-Jacobian product of the whole L-step
 * scan with the forward's gate values pinned (STE) or soft.
 * Replaces GatedEACSCellFunction.backward (cst_ssm/ops/eacs_cell_train.py:
 * 117-175).  Inputs are the forward's inputs and its gate, resid and stats
 * outputs, and the upstream gradients gy (B,L,H) and ggs, grs, gns (B,L) of
 * ys, gs, rs and the innovation (each of the last three may be NULL = 0).
 * Outputs (overwritten, float32 / complex64): du (B,L,H), dBc, dCc (B,L,N),
 * dt (B,L), dlam (H,N), dlog_dt (H), dD (H), deps (1).  temperature is T of
 * sigmoid((r - eps)/max(T, 1e-4)).  Rows are handled by one thread-block
 * cluster of up to 16 CTAs of at most 512 threads (H*lanes <= 8192): four
 * chains a thread for N > 8 (lanes = 4 for N <= 16, 8 for N <= 32, 16 for
 * N <= 64), two for N <= 8 (lanes = 4). */
EACS_API int eacs_cell_train_bwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                 const void* Bc, const void* Cc, const float* t, const float* D,
                                 const float* mean, const float* var,
                                 float eps, float eta, float var_eps, float dt_init,
                                 float dt_min, float dt_max, float temperature,
                                 const float* gate, const float* resid, const float* stats,
                                 const float* gy, const float* ggs, const float* grs,
                                 const float* gns,
                                 float* du, void* dBc, void* dCc, float* dt, void* dlam,
                                 float* dlog_dt, float* dD, float* deps,
                                 void* workspace, size_t workspace_bytes,
                                 int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* The training forward (eacs_cell_train_fwd's arguments and outputs) that
 * also writes the checkpoints the training backward recomputes from -- the
 * committed state before every K-th step, K chosen by the backward -- into
 * `bwd_workspace` (eacs_cell_train_bwd_workspace_size bytes, kept unchanged
 * until the matching eacs_cell_train_bwd_ckpt call).  The forward computes
 * those states anyway, so the backward's own checkpoint pass (a second
 * forward) is skipped.  Same reference function as eacs_cell_train_fwd
 * (GatedEACSCellFunction.forward, cst_ssm/ops/eacs_cell_train.py:81-116);
 * needs rows that one thread-block cluster holds (as the repair pass does)
 * and returns EACS_ERR_UNSUPPORTED otherwise. */
EACS_API int eacs_cell_train_fwd_ckpt(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                      const void* Bc, const void* Cc, const float* t, const float* D,
                                      const float* mean, const float* var,
                                      float eps, float eta, float var_eps, float dt_init,
                                      float dt_min, float dt_max, int gate_mode, float temperature,
                                      float* y, float* gate, float* resid, float* stats,
                                      void* workspace, size_t workspace_bytes,
                                      void* bwd_workspace, size_t bwd_workspace_bytes,
                                      int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* eacs_cell_train_bwd reading the checkpoints that eacs_cell_train_fwd_ckpt
 * wrote into `workspace` for the same inputs and sizes (the backward of
 * GatedEACSCellFunction, cst_ssm/ops/eacs_cell_train.py:117-175). */
EACS_API int eacs_cell_train_bwd_ckpt(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                      const void* Bc, const void* Cc, const float* t, const float* D,
                                      const float* mean, const float* var,
                                      float eps, float eta, float var_eps, float dt_init,
                                      float dt_min, float dt_max, float temperature,
                                      const float* gate, const float* resid, const float* stats,
                                      const float* gy, const float* ggs, const float* grs,
                                      const float* gns,
                                      float* du, void* dBc, void* dCc, float* dt, void* dlam,
                                      float* dlog_dt, float* dD, float* deps,
                                      void* workspace, size_t workspace_bytes,
                                      int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Workspace bytes eacs_cell_commits needs (eacs_cell_fwd's plus one int per
 * (b, l)); 0 if the sizes are unsupported. */
EACS_API size_t eacs_cell_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);

/* Gated cell (hard gate, optional robust_guard) that also records the
 * committed state after every step, for continuous-time queries.
 * Replaces EACSLayer.run_with_commits / _commit_range
 * (cst_ssm/modules/eacs.py:386-439) after the projections: outputs y, gate,
 * resid as eacs_cell_fwd, and commit_h (B,L,H,N) complex64 = h_pi after step
 * l, commit_t (B,L) = t_pi, commit_u (B,L,H) float32 = u_pi, commit_B,
 * commit_C (B,L,N) complex64 = B_pi, C_pi. */
EACS_API int eacs_cell_commits(const void* lam, const float* log_dt, const void* u, int u_dtype,
                               const void* Bc, const void* Cc, const float* t, const float* D,
                               const float* mean, const float* var,
                               float eps, float eta, float var_eps, float dt_init,
                               float dt_min, float dt_max,
                               int robust, int robust_k, float spike_ratio, float eps_factor,
                               float* y, float* gate, float* resid,
                               void* commit_h, float* commit_t, float* commit_u,
                               void* commit_B, void* commit_C,
                               void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Segment index of each query time: the last frame k with frame_t[b,k] <= t*
 * (binary search, clamped to [0, L-1]); frame_t (B,L) ascending, t_query
 * (B,Q), idx (B,Q) int32.  Replaces segment_index
 * (cst_ssm/modules/continuous_query.py:12-17). */
EACS_API int eacs_query_index(const float* frame_t, const float* t_query, int32_t* idx,
                              int64_t B, int64_t L, int64_t Q, void* stream);

/* Readout at query times from recorded commits: per (b, q) the commits of
 * frame idx[b,q] (clamped to [0, L-1]) evolved by delta = max(t* - t_pi, 0):
 * y (B,Q,H) float32 = Re sum_n C_pi (dA h_pi + dB_bar B_pi u_pi) + D u_pi.
 * Replaces readout_from_commits before its proj_out
 * (cst_ssm/modules/continuous_query.py:20-61). */
EACS_API int eacs_query_readout(const void* lam, const float* log_dt, const float* D,
                                const void* commit_h, const float* commit_t,
                                const float* commit_u, const void* commit_B,
                                const void* commit_C, const float* t_query,
                                const int32_t* idx, float* y,
                                int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N,
                                float dt_min, float dt_max, void* stream);

/* Training through per-frame commits.  Replaces EACSLayer._commit_range
 * (cst_ssm/modules/eacs.py:386-401) run under autograd by run_with_commits
 * (:404-439), after the projections: the training forward
 * (eacs_cell_train_fwd's arguments and outputs: STE gate for gate_mode 0,
 * soft gate for 1; 2 is the eval-mode hard gate r > eps, whose forward is
 * the STE forward and whose backward passes no gradient through the gate,
 * event_gate.py:99-100), then a replay with the decided gates that records the
 * commits after every step -- commit_h (B,L,H,N) complex64 = h_pi, commit_t
 * (B,L) = t_pi, commit_u (B,L,H) float32 = u_pi, commit_B, commit_C (B,L,N)
 * complex64 = B_pi, C_pi (blends of the previous and the new values under a
 * soft gate) -- and writes the backward's checkpoints into bwd_workspace
 * (eacs_cell_train_commits_workspace_size bytes, kept until the matching
 * eacs_cell_train_commits_bwd call).  workspace: eacs_cell_workspace_size. */
EACS_API size_t eacs_cell_train_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
EACS_API int eacs_cell_train_commits_fwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                         const void* Bc, const void* Cc, const float* t, const float* D,
                                         const float* mean, const float* var,
                                         float eps, float eta, float var_eps, float dt_init,
                                         float dt_min, float dt_max, int gate_mode, float temperature,
                                         float* y, float* gate, float* resid, float* stats,
                                         void* commit_h, float* commit_t, float* commit_u,
                                         void* commit_B, void* commit_C,
                                         void* workspace, size_t workspace_bytes,
                                         void* bwd_workspace, size_t bwd_workspace_bytes,
                                         int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Backward of eacs_cell_train_commits_fwd: eacs_cell_train_bwd_ckpt's
 * arguments with the forward's gate_mode (no innovation term: _commit_range
 * does not return one) plus the
 * upstream adjoints of the commits, g_commit_h (B,L,H,N) complex64,
 * g_commit_t (B,L), g_commit_u (B,L,H), g_commit_B, g_commit_C (B,L,N)
 * complex64 (any may be NULL = 0), which join the scan's adjoint at their
 * step.  workspace: the bwd_workspace eacs_cell_train_commits_fwd filled. */
EACS_API int eacs_cell_train_commits_bwd(const void* lam, const float* log_dt, const void* u, int u_dtype,
                                         const void* Bc, const void* Cc, const float* t, const float* D,
                                         const float* mean, const float* var,
                                         float eps, float eta, float var_eps, float dt_init,
                                         float dt_min, float dt_max, int gate_mode, float temperature,
                                         const float* gate, const float* resid, const float* stats,
                                         const float* gy, const float* ggs, const float* grs,
                                         const void* g_commit_h, const float* g_commit_t,
                                         const float* g_commit_u, const void* g_commit_B,
                                         const void* g_commit_C,
                                         float* du, void* dBc, void* dCc, float* dt, void* dlam,
                                         float* dlog_dt, float* dD, float* deps,
                                         void* workspace, size_t workspace_bytes,
                                         int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* Adjoint of eacs_query_readout (the backward of readout_from_commits before
 * proj_out, cst_ssm/modules/continuous_query.py:20-54 under autograd).
 * gy (B,Q,H) = dLoss/dy; idx (B,Q) int32 must be nondecreasing per row (a
 * frame's queries contiguous: sort the queries, or pass 0..L-1 for the frame
 * times); out-of-order indices record EACS_ERR_INVALID in the device status
 * word.  Outputs, overwritten: the commits' adjoints g_commit_h (B,L,H,N)
 * complex64, g_commit_t (B,L), g_commit_u (B,L,H), g_commit_B, g_commit_C
 * (B,L,N) complex64 (zero for frames no query reads), the query times'
 * g_t_query (B,Q) (may be NULL), dlam (H,N) complex64, dlog_dt (H), dD (H).
 * Sums run in a fixed order (no atomics).  workspace:
 * eacs_query_readout_bwd_workspace_size bytes. */
EACS_API size_t eacs_query_readout_bwd_workspace_size(int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N);
EACS_API int eacs_query_readout_bwd(const void* lam, const float* log_dt, const float* D,
                                    const void* commit_h, const float* commit_t,
                                    const float* commit_u, const void* commit_B,
                                    const void* commit_C, const float* t_query,
                                    const int32_t* idx, const float* gy,
                                    void* g_commit_h, float* g_commit_t, float* g_commit_u,
                                    void* g_commit_B, void* g_commit_C, float* g_t_query,
                                    void* dlam, float* dlog_dt, float* dD,
                                    void* workspace, size_t workspace_bytes,
                                    int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N,
                                    float dt_min, float dt_max, void* stream);

/* K steps of one EACS branch with explicit state, per row (streaming).
 * Replaces the per-branch body of temporal_step (cst_ssm/modules/streaming.py:
 * 45-85: first-observation commit, valid masks, CPI-modulated threshold) over
 * eacs_step (modules/eacs.py:78-142), after the projections.
 * Inputs u (B,K,H) of u_dtype, Bc/Cc (B,K,N) complex64, t (B,K), valid (B,K)
 * uint8 or NULL (all valid), cpi (B,K) or NULL.  State in: h (B,H,N)
 * complex64, t (B), u (B,H), B/C (B,N) complex64, initialized (B) uint8;
 * state out: the same shapes in separate buffers (the input state is not
 * modified).  Outputs y (B,K,H) = Re sum_n C h_cur + D u (zeros where not
 * valid), gate (1 on a row's first valid step), resid, innov (resid where the
 * row was already initialised, else 0), all (B,K) float32.  gate_mode 0 hard
 * (r > eps_l), 1 soft sigmoid((r - eps_l)/max(T, 1e-4)); cpi_modulation m > 0
 * with cpi: eps_l = max(eps (1 - m clamp(cpi, 0, 1)), 1e-3).  No workspace. */
EACS_API int eacs_stream_chunk(const void* lam, const float* log_dt, const float* D,
                               const float* mean, const float* var,
                               const void* u, int u_dtype, const void* Bc, const void* Cc,
                               const float* t, const uint8_t* valid, const float* cpi,
                               const void* h_in, const float* t_in, const float* u_in,
                               const void* B_in, const void* C_in, const uint8_t* init_in,
                               void* h_out, float* t_out, float* u_out, void* B_out,
                               void* C_out, uint8_t* init_out,
                               float* y, float* gate, float* resid, float* innov,
                               float eps, float eta, float var_eps, float dt_init,
                               float dt_min, float dt_max, float cpi_modulation,
                               int gate_mode, float temperature,
                               int64_t B, int64_t K, int64_t H, int64_t N, void* stream);

/* Backward of one streaming step (eacs_stream_chunk with K = 1, float32 u):
 * the per-branch body of temporal_step (cst_ssm/modules/streaming.py:55-80,
 * eacs_step eacs.py:78-142, EventGate.forward event_gate.py:84-105) under
 * autograd.  Inputs: the step's inputs and state in as eacs_stream_chunk
 * (u (B,H), Bc/Cc (B,N), t (B), valid/cpi (B) or NULL, h_in (B,H,N), t_in,
 * u_in, B_in, C_in, init_in), its gate output (B) or NULL (pins the hard
 * decision), and the upstream gradients of y (B,H) (before proj_out), of the
 * gate output, resid and innov (B), and of the state out gh (B,H,N), gt,
 * gu, gB, gC -- any of them NULL = 0.  Outputs (overwritten): du (B,H), dBc,
 * dCc (B,N), dt (B), dcpi (B) (may be NULL), the state in's dh_in, dt_in,
 * du_in, dB_in, dC_in, and dlam (H,N), dlog_dt (H), dD (H), deps (1).
 * gate_mode 0: STE (hard forward, sigmoid slope backward), 1: soft, 2: hard
 * with no gradient through the gate (eval mode).  One CTA per row; the
 * parameter sums run in row order (workspace:
 * eacs_stream_step_bwd_workspace_size bytes). */
EACS_API size_t eacs_stream_step_bwd_workspace_size(int64_t B, int64_t H, int64_t N);
EACS_API int eacs_stream_step_bwd(const void* lam, const float* log_dt, const float* D,
                                  const float* mean, const float* var, const float* u,
                                  const void* Bc, const void* Cc, const float* t,
                                  const uint8_t* valid, const float* cpi,
                                  const void* h_in, const float* t_in, const float* u_in,
                                  const void* B_in, const void* C_in, const uint8_t* init_in,
                                  const float* gate, const float* gy, const float* gg,
                                  const float* gr, const float* gn, const void* gh,
                                  const float* gt, const float* gu, const void* gB, const void* gC,
                                  float* du, void* dBc, void* dCc, float* dt, float* dcpi,
                                  void* dh_in, float* dt_in, float* du_in, void* dB_in, void* dC_in,
                                  void* dlam, float* dlog_dt, float* dD, float* deps,
                                  void* workspace, size_t workspace_bytes,
                                  float eps, float eta, float var_eps, float dt_init, float dt_min,
                                  float dt_max, float cpi_modulation, int gate_mode, float temperature,
                                  int64_t B, int64_t H, int64_t N, void* stream);

/* Device workspace bytes eacs_cell_fwd_host needs (0 if unsupported). */
EACS_API size_t eacs_cell_fwd_host_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N,
                                                  int64_t chunk);

/* eacs_cell_fwd (hard gate) with the sequences and outputs in HOST memory:
 * u (B,L,H) of u_dtype, Bc/Cc (B,L,N) complex64, t (B,L) float32 in, y
 * (B,L,H), gate, resid (B,L) float32 out -- pinned (cudaHostAlloc /
 * cudaHostRegister) for the copies to overlap; pageable memory works but
 * copies synchronously.  Parameters (lam, log_dt, D, mean, var) and the
 * workspace are device pointers.  The frames are processed in chunks of
 * `chunk` frames (rounded up to a multiple of 32; <= 0 picks 512): the
 * copy-in of one chunk and the copy-out of another overlap the cell of a
 * third, each row resuming from the state the previous chunk left, on two
 * copy streams the library owns for the device and on `stream`, which
 * completes when the outputs are in host memory.  Results equal one
 * eacs_cell_fwd over the whole sequence.  Same semantics and gate options as
 * eacs_cell_fwd; shapes whose repair pass cannot resume rows (more than 16
 * CTAs of 512 threads per row) return EACS_ERR_UNSUPPORTED.  Calls on one
 * device are enqueued one at a time.  No reference counterpart: it is the
 * host-buffer form of eacs_cell_fwd for callers whose features are in host
 * memory (long videos streamed from a feature cache). */
EACS_API int eacs_cell_fwd_host(const void* lam, const float* log_dt, const float* D,
                                const float* mean, const float* var,
                                const void* u, int u_dtype, const void* Bc, const void* Cc,
                                const float* t, float eps, float eta, float var_eps,
                                float dt_init, float dt_min, float dt_max,
                                int robust, int robust_k, float spike_ratio, float eps_factor,
                                float* y, float* gate, float* resid,
                                void* workspace, size_t workspace_bytes,
                                int64_t B, int64_t L, int64_t H, int64_t N, int64_t chunk,
                                void* stream);

/* MultiScaleEACS branch epilogue in one pass (cst_ssm/modules/multiscale.py:
 * 176-179): per row, w = softmax(x W^T + b) over the S branches, then
 * y = LayerNorm(x + sum_s w_s delta_s) * ln_weight + ln_bias.
 * x, y and the S branch outputs delta[s] (proj_out outputs): (rows, d) of
 * `dtype` (float32, float16 or bfloat16), 16-byte aligned, d a multiple of 8
 * (4 for float32) and at most 2048 (1024 for float32); `deltas` is a HOST
 * array of S device pointers, S <= 8.  fusion_weight (S, d) and
 * fusion_bias (S) float32 (bias may be NULL); ln_weight / ln_bias (d)
 * float32 or NULL (1 / 0); weights (rows, S) float32 output or NULL.
 * Computes in float32 with one rounding to `dtype` at the end. */
EACS_API int eacs_branch_fuse(const void* x, const void* const* deltas, int S, int dtype,
                              const float* fusion_weight, const float* fusion_bias,
                              const float* ln_weight, const float* ln_bias, float ln_eps,
                              void* y, float* weights, int64_t rows, int64_t d, void* stream);

/* ---- feature cache (host side; no device memory is touched except by
 * eacs_fc_upload's copy) ----
 * One video's features <vid>.npy (C-order little-endian float16 or float32,
 * shape (L, P, d) or (L, d)) and timestamps <vid>.ts.npy (L float32 or
 * float64), the layout the reference writes (data_pipeline/src/npz_to_npy.py)
 * and memory-maps (cst_ssm/data/dataset.py:58-67, numpy.load mmap_mode="r").
 * The feature file is mapped read-only; frames are copied out of the mapping
 * with several threads.  Functions return EACS_OK or an error code with the
 * message in eacs_last_error(). */
typedef struct eacs_fc eacs_fc;

/* Open `npy_path` and its "<stem>.ts.npy"; *out receives the handle. */
EACS_API int eacs_fc_open(const char* npy_path, eacs_fc** out);
/* Frames L, patches P (1 for (L, d) files), width d, EACS_DTYPE_F16/F32. */
EACS_API int eacs_fc_info(const eacs_fc* fc, int64_t* L, int64_t* P, int64_t* d, int* dtype);
/* The L timestamps as float32 into host memory `out`. */
EACS_API int eacs_fc_timestamps(const eacs_fc* fc, float* out);
/* Frames [l0, l0+n) (n*P*d elements of the file's dtype) into host `dst`. */
EACS_API int eacs_fc_read(const eacs_fc* fc, int64_t l0, int64_t n, void* dst);
/* eacs_fc_read into host `staging` (pinned, staging_bytes >= n*P*d*size),
 * then an asynchronous copy to device `dst_device` on `stream`; `staging`
 * must stay untouched until that copy has completed. */
EACS_API int eacs_fc_upload(const eacs_fc* fc, int64_t l0, int64_t n, void* staging,
                            size_t staging_bytes, void* dst_device, void* stream);
/* Unmap and free the handle (NULL is a no-op). */
EACS_API void eacs_fc_close(eacs_fc* fc);

/* Bytes of the library-owned scratch array behind eacs_cell_fwd_noalloc. */
#define EACS_NOALLOC_SCRATCH_BYTES (32u << 20)

/* eacs_cell_fwd without a workspace argument: the gated cell's scratch
 * (residual partials, row state, committed state) lives in a file-scope
 * __device__ array of EACS_NOALLOC_SCRATCH_BYTES (32 MiB) inside the library,
 * for callers that cannot allocate device memory -- a host that binds only
 * this C ABI with no device allocator of its own, or a process whose device
 * memory belongs to another allocator and must not see a cudaMalloc (which
 * also synchronises the device).  No counterpart in the reference.
 * Nothing is allocated by this call; the array is created when the library's
 * device code is loaded and every GPU that loads it keeps it until exit.
 * The first call on each device looks up the array's device address (with
 * that device current); make that first call before any stream capture.
 * The address is kept for the life of the process and belongs to the
 * device's primary context: after cudaDeviceReset on that device it no
 * longer names the array, so do not call this entry point after a reset.
 * Sizes whose scratch (eacs_cell_fwd_workspace_size) exceeds the array are
 * rejected with EACS_ERR_WORKSPACE.  All calls share the one array per device
 * and it keeps the last call's contents (every byte a call reads it writes
 * first in that call), so calls that overlap on the GPU -- on different
 * streams or host threads of the same device -- race; serialise them.
 * Arguments and outputs are those of eacs_cell_fwd. */
EACS_API int eacs_cell_fwd_noalloc(const void* lam, const float* log_dt, const void* u,
                                   int u_dtype, const void* Bc, const void* Cc,
                                   const float* t, const float* D, const float* mean,
                                   const float* var, float eps, float eta, float var_eps,
                                   float dt_init, float dt_min, float dt_max,
                                   int robust, int robust_k, float spike_ratio,
                                   float eps_factor, int gate_mode, float temperature,
                                   float* y, float* gate, float* resid,
                                   int64_t B, int64_t L, int64_t H, int64_t N, void* stream);

/* One streaming frame of a MultiScaleEACS, inference (temporal_step,
 * cst_ssm/modules/streaming.py:45-85, with the branches' norm, _project and
 * proj_out, modules/eacs.py:261-267, and the module's fusion softmax and
 * out_norm, modules/multiscale.py:45-46, :177-179), in S + 3 launches:
 * the norms, input projections and fusion logits of all branches, each
 * branch's cell step (as eacs_stream_chunk with K = 1), each branch's proj_out
 * blended with the fusion weights plus the residual, and out_norm.  x (B,d)
 * float32 with B <= 8, t (B), valid (B) uint8 or NULL, cpi (B) or NULL; the
 * weights are the modules' float32 tensors: per branch the LayerNorm (d),
 * proj_u (H,d), proj_B and proj_C (2N,d) with biases, proj_out (d,H) with its
 * bias; the fusion layer (S,d), (S) and out_norm (d).  State in and out as
 * eacs_stream_chunk, per branch.  Outputs: y (B,d), the fusion weights (B,S),
 * and gate, resid, innov (S,B).  1 <= S <= 4. */
typedef struct {
    const float* ln_w; const float* ln_b; float ln_eps;       /* the branch's norm */
    const float* wu; const float* bu;                         /* proj_u (H,d), (H) */
    const float* wB; const float* bB;                         /* proj_B (2N,d), (2N) */
    const float* wC; const float* bC;                         /* proj_C (2N,d), (2N) */
    const float* wo; const float* bo;                         /* proj_out (d,H), (d) */
    const void* lam; const float* log_dt; const float* D; const float* mean; const float* var;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_modulation, temperature;
    int gate_mode;                                            /* 0 hard, 1 soft */
    int H, N;
    const void* h_in; const float* t_in; const float* u_in; const void* B_in; const void* C_in;
    const uint8_t* init_in;
    void* h_out; float* t_out; float* u_out; void* B_out; void* C_out; uint8_t* init_out;
} EacsFrameBranch;

EACS_API size_t eacs_stream_frame_workspace_size(const EacsFrameBranch* branches, int S, int64_t B,
                                                 int64_t d);
EACS_API int eacs_stream_frame(const float* x, const float* t, const uint8_t* valid, const float* cpi,
                               const EacsFrameBranch* branches, int S, const float* fusion_w,
                               const float* fusion_b, const float* out_norm_w, const float* out_norm_b,
                               float out_norm_eps, float* y, float* weights, float* gate, float* resid,
                               float* innov, void* workspace, size_t workspace_bytes, int64_t B,
                               int64_t d, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EACS_B200_H */
