// eacs_host.h -- host-side declarations shared by the translation units of
// libeacs_b200.so (kernels launchers and the C ABI in capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/eacs_b200.h"

namespace eacs {

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to EACS_ERR_CUDA with a message (EACS_OK when e == success).
int cuda_check(cudaError_t e, const char* what);

// Launch bookkeeping (capi.cu): count a launch; record the thread's optional
// timing events around the dominant kernel of a call.
void note_launch(int n = 1);
void mark_start(cudaStream_t s);
void mark_stop(cudaStream_t s);

// scan.cu
int scan_fwd(const void* a, const void* b, void* h, int64_t B, int64_t L, int64_t C,
             cudaStream_t stream);
int scan_bwd(const void* a, const void* h, const void* gh, void* ga, void* gb, int64_t B,
             int64_t L, int64_t C, cudaStream_t stream);
cudaError_t scan_read_status(int* out, cudaStream_t stream);

// Steps between the state checkpoints of the ungated training forward
// (eacs_ssm_train_fwd); the backward recomputes one such chunk at a time.
constexpr int kSsmCk = 8;

// cell.cu
struct CellCall {
    const void* lam;
    const float* log_dt;
    const void* u;
    int u_dtype;
    const void* Bc;
    const void* Cc;
    const float* t;
    const float* D;
    const float* mean;
    const float* var;
    float eps, eta, var_eps, dt_init, dt_min, dt_max;
    int robust, robust_k;
    float spike_ratio, eps_factor;
    int gate_mode;
    float temperature;
    float* y;
    float* gate;
    float* resid;
    void* workspace;
    size_t workspace_bytes;
    int64_t B, L, H, N;
    void* stats = nullptr;  // optional (B,L) float2 (||obs-pred||, ||obs||)
    // optional per-frame commits (hard gate; workspace cell_commits_workspace_size)
    void* commit_h = nullptr;  // (B,L,H,N) complex64
    float* commit_t = nullptr; // (B,L)
    float* commit_u = nullptr; // (B,L,H)
    void* commit_B = nullptr;  // (B,L,N) complex64
    void* commit_C = nullptr;
    // optional row state carried between time chunks (hard gate or soft gate,
    // cluster repair shapes): in = state before step 0 (nullptr: the initial
    // state), out = state after step L-1 (L a multiple of 4)
    const void* cin_h = nullptr;  // (B,H,N) complex64
    const float* cin_u = nullptr; // (B,H)
    const void* cin_B = nullptr;  // (B,N) complex64
    const void* cin_C = nullptr;
    const void* cin_row = nullptr;  // (B) float4: t_pi, spike, r_prev, -
    void* cout_h = nullptr;
    float* cout_u = nullptr;
    void* cout_B = nullptr;
    void* cout_C = nullptr;
    void* cout_row = nullptr;
    // optional training checkpoints (train_ckpt_layout): the state before
    // every ck_K-th step, as the training backward reads them
    void* ck_h = nullptr;    // [B][nK][H][N] complex64
    float* ck_u = nullptr;   // [B][nK][H]
    void* ck_row = nullptr;  // [B][nK] float4 (t_pi, -, -, -)
    void* ck_bc = nullptr;   // [B][nK][2][N] complex64 (B_pi, C_pi)
    int ck_K = 0, ck_nK = 0;
    // cells of this shape the caller runs at the same time on other streams
    // (this one included); it picks the speculative pass's layout
    int side_by_side = 1;
};
size_t cell_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
size_t cell_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
// true when the repair pass for (H, N) can resume rows from a carried state
bool cell_resumable(int64_t H, int64_t N);

// pipeline.cu: gated cell over host buffers, time chunks pipelined with the copies
struct CellHostCall {
    const void* lam;  // parameters: device pointers
    const float* log_dt;
    const float* D;
    const float* mean;
    const float* var;
    const void* u;    // sequences and outputs: host pointers (pinned for overlap)
    int u_dtype;
    const void* Bc;
    const void* Cc;
    const float* t;
    float eps, eta, var_eps, dt_init, dt_min, dt_max;
    int robust, robust_k;
    float spike_ratio, eps_factor;
    float* y;
    float* gate;
    float* resid;
    void* workspace;  // device
    size_t workspace_bytes;
    int64_t B, L, H, N, chunk;
};
size_t cell_host_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N, int64_t chunk);
int cell_fwd_host(const CellHostCall& c, cudaStream_t stream);
int cell_fwd(const CellCall& c, cudaStream_t stream);
int cell_fwd_noalloc(const CellCall& c, cudaStream_t stream);
// ckpt == nullptr: inference; otherwise also writes the state before every
// kSsmCk-th step to ckpt ([B][ceil(L/kSsmCk)][H][N] complex64).
int ssm_fwd(const void* lam, const float* log_dt, const float* t, const void* Bc,
            const void* Cc, const void* u, int u_dtype, const float* D, float* y, int64_t B,
            int64_t L, int64_t H, int64_t N, float dt_min, float dt_max, void* ckpt,
            size_t ckpt_bytes, cudaStream_t stream);
size_t ssm_ckpt_size(int64_t B, int64_t L, int64_t H, int64_t N);
cudaError_t cell_read_status(int* out, cudaStream_t stream);
int wait_selftest(int polls, cudaStream_t stream);

// LayerNorm + input projections (project.cu)
struct ProjectCall {
    const void* x;       // (M, d), x_dtype
    int x_dtype;
    const float* gamma;  // (d)
    const float* beta;
    float ln_eps;
    const void* weight;  // (w_rows, d), w_dtype: [proj_u; proj_B; proj_C; zero rows]
    int w_dtype;
    int64_t w_rows;
    const float* bias;   // (H + 4N)
    void* u;             // (M, H), u_dtype
    int u_dtype;
    void* Bc;            // (M, N) complex64
    void* Cc;
    int64_t M, d, H, N;
    void* workspace;     // project_workspace_size(M) bytes
    size_t workspace_bytes;
};
size_t project_workspace_size(int64_t M);
int project_fwd(const ProjectCall& c, cudaStream_t stream);
int zoh_kernels(const void* lam, const float* dt, void* dA, void* dBbar, int64_t M, int64_t H,
                int64_t N, cudaStream_t stream);

// query.cu: continuous-time queries over recorded commits
int query_index(const float* frame_t, const float* t_query, int* idx, int64_t B, int64_t L,
                int64_t Q, cudaStream_t stream);
int query_readout(const void* lam, const float* log_dt, const float* D, const void* commit_h,
                  const float* commit_t, const float* commit_u, const void* commit_B,
                  const void* commit_C, const float* t_query, const int* idx, float* y, int64_t B,
                  int64_t L, int64_t Q, int64_t H, int64_t N, float dt_min, float dt_max,
                  cudaStream_t stream);
// adjoint of query_readout: idx nondecreasing per row (a frame's queries
// contiguous); the commits' adjoints are overwritten (zero where no query
// reads a frame)
struct QueryBwdCall {
    const void* lam;
    const float* log_dt;
    const float* D;
    const void* commit_h;
    const float* commit_t;
    const float* commit_u;
    const void* commit_B;
    const void* commit_C;
    const float* t_query;
    const int* idx;
    const float* gy;       // (B,Q,H)
    void* g_commit_h;      // (B,L,H,N) complex64
    float* g_commit_t;     // (B,L)
    float* g_commit_u;     // (B,L,H)
    void* g_commit_B;      // (B,L,N) complex64
    void* g_commit_C;
    float* g_t_query;      // (B,Q) or null
    void* dlam;            // (H,N) complex64
    float* dlog;           // (H)
    float* dD;             // (H)
    void* workspace;
    size_t workspace_bytes;
    int64_t B, L, Q, H, N;
    float dt_min, dt_max;
};
size_t query_readout_bwd_workspace_size(int64_t B, int64_t L, int64_t Q, int64_t H, int64_t N);
int query_readout_bwd(const QueryBwdCall& c, cudaStream_t stream);
cudaError_t query_read_status(int* out, cudaStream_t stream);

// stream.cu: gated steps with explicit branch state
struct StreamCall {
    const void* lam;
    const float* log_dt;
    const float* D;
    const float* mean;
    const float* var;
    const void* u;
    int u_dtype;
    const void* Bc;
    const void* Cc;
    const float* t;
    const uint8_t* valid;
    const float* cpi;
    const void* h_in;
    const float* t_in;
    const float* u_in;
    const void* B_in;
    const void* C_in;
    const uint8_t* init_in;
    void* h_out;
    float* t_out;
    float* u_out;
    void* B_out;
    void* C_out;
    uint8_t* init_out;
    float* y;
    float* gate;
    float* resid;
    float* innov;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_modulation, temperature;
    int gate_mode;
    int64_t B, K, H, N;
};
int stream_chunk(const StreamCall& c, cudaStream_t stream);
// backward of one step (K = 1), float32 u; upstream pointers may be null (0)
struct StreamBwdCall {
    const void* lam;
    const float* log_dt;
    const float* D;
    const float* mean;
    const float* var;
    const float* u;        // (B,H)
    const void* Bc;        // (B,N) complex64
    const void* Cc;
    const float* t;        // (B)
    const uint8_t* valid;  // (B) or null
    const float* cpi;      // (B) or null
    const void* h_in;
    const float* t_in;
    const float* u_in;
    const void* B_in;
    const void* C_in;
    const uint8_t* init_in;
    const float* gate;     // (B) the forward's gate output (pins a hard gate) or null
    const float* gy;       // (B,H)
    const float* gg;       // (B)
    const float* gr;
    const float* gn;
    const void* gh;        // (B,H,N) complex64: the state out's adjoints
    const float* gt;
    const float* gu;
    const void* gB;
    const void* gC;
    float* du;
    void* dBc;
    void* dCc;
    float* dt;
    float* dcpi;           // or null
    void* dh_in;
    float* dt_in;
    float* du_in;
    void* dB_in;
    void* dC_in;
    void* dlam;
    float* dlog;
    float* dD;
    float* deps;
    void* workspace;
    size_t workspace_bytes;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_modulation, temperature;
    int gate_mode;  // 0 STE, 1 soft, 2 hard (no gradient through the gate)
    int64_t B, H, N;
};
size_t stream_step_bwd_workspace_size(int64_t B, int64_t H, int64_t N);
int stream_step_bwd(const StreamBwdCall& c, cudaStream_t stream);

// frame.cu: one streaming frame of a MultiScaleEACS (inference)
constexpr int kFrameMaxBranches = 4;
constexpr int kFrameMaxRows = 8;
using FrameBranch = EacsFrameBranch;
struct FrameCall {
    const float* x;
    const float* t;
    const uint8_t* valid;
    const float* cpi;
    const FrameBranch* br;
    int S;
    const float* wf;
    const float* bf;
    const float* out_w;
    const float* out_b;
    float out_eps;
    float* y;
    float* weights;
    float* gate;
    float* resid;
    float* innov;
    void* workspace;
    size_t workspace_bytes;
    int64_t B, d;
};
size_t stream_frame_workspace_size(const FrameBranch* br, int S, int64_t B, int64_t d);
int stream_frame(const FrameCall& c, cudaStream_t stream);

// fuse.cu: MultiScaleEACS branch epilogue
struct FuseCall {
    const void* x;
    const void* delta[8];
    int S;
    int dtype;
    const float* wf;
    const float* bf;
    const float* gamma;
    const float* beta;
    float ln_eps;
    void* y;
    float* w;
    int64_t rows;
    int d;
};
int branch_fuse(const FuseCall& c, cudaStream_t stream);

// train.cu
struct TrainBwdCall {
    const void* lam;
    const float* log_dt;
    const void* u;
    int u_dtype;
    const void* Bc;
    const void* Cc;
    const float* t;
    const float* D;
    const float* mean;
    const float* var;
    float eps, eta, var_eps, dt_init, dt_min, dt_max, temperature;
    const float* gates;
    const float* resid;
    const void* stats;
    const float* gy;
    const float* ggs;
    const float* grs;
    const float* gns;
    float* du;
    void* dBc;
    void* dCc;
    float* dt;
    void* dlam;
    float* dlog;
    float* dD;
    float* deps;
    void* workspace;
    size_t workspace_bytes;
    int64_t B, L, H, N;
    bool have_ckpt = false;  // the workspace already holds the forward's checkpoints
    // training through per-frame commits: the workspace holds the checkpoints
    // train_commits_replay wrote, and the upstream adjoints of the commits
    // (any may be null = zero) join the backward at their step
    bool commits = false;
    bool gate_const = false;     // the gates are constants (no gradient through r > eps)
    const void* gc_h = nullptr;  // (B,L,H,N) complex64
    const float* gc_t = nullptr; // (B,L)
    const float* gc_u = nullptr; // (B,L,H)
    const void* gc_B = nullptr;  // (B,L,N) complex64
    const void* gc_C = nullptr;
};
size_t train_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
// per-frame commits written by the replay of the training forward
struct CommitOut {
    void* h;   // (B,L,H,N) complex64
    float* t;  // (B,L)
    float* u;  // (B,L,H)
    void* B;   // (B,L,N) complex64
    void* C;
};
size_t train_commits_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
// Replays the gated forward with c.gates, writing the commits and the
// backward's checkpoints into c.workspace (train_commits_workspace_size).
int train_commits_replay(const TrainBwdCall& c, const CommitOut& out, cudaStream_t stream);
// Where the training backward's workspace keeps its checkpoints (fills c's
// ck_* fields); an EACS status code.
int train_ckpt_layout(int64_t B, int64_t L, int64_t H, int64_t N, void* workspace, size_t workspace_bytes,
                      CellCall* c);

// ssm_train.cu
struct SsmBwdCall {
    const void* lam;
    const float* log_dt;
    const float* t;
    const void* Bc;
    const void* Cc;
    const void* u;
    int u_dtype;
    const float* D;
    const float* gy;
    const void* ckpt;
    size_t ckpt_bytes;
    float* du;
    void* dBc;
    void* dCc;
    float* dt;
    void* dlam;
    float* dlog;
    float* dD;
    void* workspace;
    size_t workspace_bytes;
    int64_t B, L, H, N;
    float dt_min, dt_max;
};
size_t ssm_bwd_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N);
int ssm_bwd(const SsmBwdCall& c, cudaStream_t stream);
int train_bwd(const TrainBwdCall& c, cudaStream_t stream);
cudaError_t train_read_status(int* out, cudaStream_t stream);

}  // namespace eacs
