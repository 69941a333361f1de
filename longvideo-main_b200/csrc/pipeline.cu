// pipeline.cu -- the gated cell over host buffers, with the host<->device
// copies of time chunks overlapped with the cell of neighbouring chunks.
//
// A row's gated cell is resumable from a carried state (committed state,
// t_pi, u_pi, B_pi, C_pi, robust_guard counter), so a sequence of L frames can
// be run as chunks of `chunk` frames: chunk k's inputs are copied in on one
// stream while chunk k-1 runs on the caller's stream and chunk k-2's outputs
// are copied out on a third.  Two device slots per direction and two carry
// buffers (ping-pong); the dependencies are events:
//   copy-in k   waits  cell k-2   (input slot free)
//   cell k      waits  copy-in k, copy-out k-2 (output slot free)
//   copy-out k  waits  cell k
// Host rows are strided by L frames, so every copy is one cudaMemcpy2DAsync
// of B rows.  The results equal one eacs_cell_fwd call on the whole sequence
// bit for bit (the chain pass does the same operations in the same order).
#include <algorithm>
#include <mutex>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

size_t al(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t u_size(int dtype) { return dtype == EACS_DTYPE_F32 ? 4 : 2; }

int64_t chunk_len(int64_t L, int64_t chunk) {
    int64_t c = chunk > 0 ? chunk : 512;
    c = ((c + 31) / 32) * 32;  // full 32-step stages: the carried state is exact
    return std::min(c, ((L + 31) / 32) * 32);
}

struct PWs {
    size_t cell, carry[2], in[2], out[2], total;
    size_t c_h, c_u, c_B, c_C, c_row, carry_bytes;  // offsets inside a carry
    size_t i_u, i_B, i_C, i_t, in_bytes;            // inside an input slot
    size_t o_y, o_g, o_r, out_bytes;                // inside an output slot
};

PWs pws(int64_t B, int64_t Lc, int64_t H, int64_t N, int dtype) {
    PWs w{};
    w.c_h = 0;
    w.c_u = w.c_h + al(sizeof(float2) * B * H * N);
    w.c_B = w.c_u + al(sizeof(float) * B * H);
    w.c_C = w.c_B + al(sizeof(float2) * B * N);
    w.c_row = w.c_C + al(sizeof(float2) * B * N);
    w.carry_bytes = w.c_row + al(sizeof(float4) * B);
    w.i_u = 0;
    w.i_B = w.i_u + al(u_size(dtype) * B * Lc * H);
    w.i_C = w.i_B + al(sizeof(float2) * B * Lc * N);
    w.i_t = w.i_C + al(sizeof(float2) * B * Lc * N);
    w.in_bytes = w.i_t + al(sizeof(float) * B * Lc);
    w.o_y = 0;
    w.o_g = w.o_y + al(sizeof(float) * B * Lc * H);
    w.o_r = w.o_g + al(sizeof(float) * B * Lc);
    w.out_bytes = w.o_r + al(sizeof(float) * B * Lc);
    size_t o = 0;
    w.cell = o;
    o += al(cell_workspace_size(B, Lc, H, N));
    for (int k = 0; k < 2; ++k) { w.carry[k] = o; o += w.carry_bytes; }
    for (int k = 0; k < 2; ++k) { w.in[k] = o; o += w.in_bytes; }
    for (int k = 0; k < 2; ++k) { w.out[k] = o; o += w.out_bytes; }
    w.total = o;
    return w;
}

// Copy streams and events, one set per device, created on first use and kept
// for the life of the process; a mutex serialises the enqueueing of calls.
constexpr int kMaxDev = 64;
struct DevPipe {
    std::mutex mu;
    bool ready = false;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t start = nullptr, ev_in[2] = {}, ev_cell[2] = {}, ev_out[2] = {};
};
DevPipe g_pipe[kMaxDev];

cudaError_t pipe_init(DevPipe& p) {
    if (p.ready) return cudaSuccess;
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&p.s_in, cudaStreamNonBlocking)) != cudaSuccess) return e;
    if ((e = cudaStreamCreateWithFlags(&p.s_out, cudaStreamNonBlocking)) != cudaSuccess) return e;
    cudaEvent_t* evs[] = {&p.start, &p.ev_in[0], &p.ev_in[1], &p.ev_cell[0], &p.ev_cell[1],
                          &p.ev_out[0], &p.ev_out[1]};
    for (cudaEvent_t* ev : evs)
        if ((e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming)) != cudaSuccess) return e;
    p.ready = true;
    return cudaSuccess;
}

}  // namespace

size_t cell_host_workspace_size(int64_t B, int64_t L, int64_t H, int64_t N, int64_t chunk) {
    if (B <= 0 || L <= 0 || H <= 0 || N <= 0 || N > 64) return 0;
    return pws(B, chunk_len(L, chunk), H, N, EACS_DTYPE_F32).total;  // f32 u bounds every dtype
}

int cell_fwd_host(const CellHostCall& c, cudaStream_t stream) {
    const char* fn = "eacs_cell_fwd_host";
    if (c.B < 0 || c.L < 0 || c.H < 0 || c.N < 0) return fail(EACS_ERR_INVALID, "%s: negative size", fn);
    if (c.B == 0 || c.L == 0 || c.H == 0) return EACS_OK;
    if (c.N <= 0 || c.N > 64) return fail(EACS_ERR_UNSUPPORTED, "%s: N=%lld outside 1..64", fn, (long long)c.N);
    if (c.u_dtype != EACS_DTYPE_F32 && c.u_dtype != EACS_DTYPE_F16 && c.u_dtype != EACS_DTYPE_BF16)
        return fail(EACS_ERR_INVALID, "%s: unknown u dtype %d", fn, c.u_dtype);
    if (!c.lam || !c.log_dt || !c.D || !c.mean || !c.var || !c.u || !c.Bc || !c.Cc || !c.t || !c.y ||
        !c.gate || !c.resid)
        return fail(EACS_ERR_INVALID, "%s: null pointer argument", fn);
    if (!cell_resumable(c.H, c.N))
        return fail(EACS_ERR_UNSUPPORTED, "%s: H=%lld N=%lld has no resumable repair pass", fn,
                    (long long)c.H, (long long)c.N);
    const int64_t Lc = chunk_len(c.L, c.chunk);
    const PWs w = pws(c.B, Lc, c.H, c.N, c.u_dtype);
    const size_t need = cell_host_workspace_size(c.B, c.L, c.H, c.N, c.chunk);
    if (!c.workspace || c.workspace_bytes < need)
        return fail(EACS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, need,
                    c.workspace_bytes);
    int dev = 0;
    int rc = cuda_check(cudaGetDevice(&dev), fn);
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDev) return fail(EACS_ERR_UNSUPPORTED, "%s: device %d", fn, dev);
    DevPipe& p = g_pipe[dev];
    std::lock_guard<std::mutex> lock(p.mu);
    if ((rc = cuda_check(pipe_init(p), fn))) return rc;

    char* ws = static_cast<char*>(c.workspace);
    const size_t esz = u_size(c.u_dtype);
    const int64_t nch = (c.L + Lc - 1) / Lc;
    cudaError_t e;
#define EACS_TRY(x)                                         \
    do {                                                    \
        if ((e = (x)) != cudaSuccess) return cuda_check(e, fn); \
    } while (0)
    // the slots may still be in use by earlier work on the caller's stream
    EACS_TRY(cudaEventRecord(p.start, stream));
    EACS_TRY(cudaStreamWaitEvent(p.s_in, p.start, 0));
    for (int64_t k = 0; k < nch; ++k) {
        const int sl = static_cast<int>(k & 1);
        const int64_t l0 = k * Lc;
        const int64_t len = std::min(Lc, c.L - l0);
        char* in = ws + w.in[sl];
        char* out = ws + w.out[sl];
        // ---- copy in (host rows are L frames apart) ----
        if (k >= 2) EACS_TRY(cudaStreamWaitEvent(p.s_in, p.ev_cell[sl], 0));
        const char* uh = static_cast<const char*>(c.u);
        EACS_TRY(cudaMemcpy2DAsync(in + w.i_u, len * c.H * esz, uh + l0 * c.H * esz, c.L * c.H * esz,
                                   len * c.H * esz, c.B, cudaMemcpyHostToDevice, p.s_in));
        const char* bh = static_cast<const char*>(c.Bc);
        const char* ch = static_cast<const char*>(c.Cc);
        EACS_TRY(cudaMemcpy2DAsync(in + w.i_B, len * c.N * 8, bh + l0 * c.N * 8, c.L * c.N * 8,
                                   len * c.N * 8, c.B, cudaMemcpyHostToDevice, p.s_in));
        EACS_TRY(cudaMemcpy2DAsync(in + w.i_C, len * c.N * 8, ch + l0 * c.N * 8, c.L * c.N * 8,
                                   len * c.N * 8, c.B, cudaMemcpyHostToDevice, p.s_in));
        EACS_TRY(cudaMemcpy2DAsync(in + w.i_t, len * 4, c.t + l0, c.L * 4, len * 4, c.B,
                                   cudaMemcpyHostToDevice, p.s_in));
        EACS_TRY(cudaEventRecord(p.ev_in[sl], p.s_in));
        // ---- cell on the caller's stream ----
        EACS_TRY(cudaStreamWaitEvent(stream, p.ev_in[sl], 0));
        if (k >= 2) EACS_TRY(cudaStreamWaitEvent(stream, p.ev_out[sl], 0));
        CellCall cc{c.lam,   c.log_dt, in + w.i_u, c.u_dtype,  in + w.i_B, in + w.i_C,
                    reinterpret_cast<const float*>(in + w.i_t), c.D, c.mean, c.var,
                    c.eps,   c.eta,    c.var_eps,  c.dt_init,  c.dt_min,   c.dt_max,
                    c.robust, c.robust_k, c.spike_ratio, c.eps_factor, 0, 0.1f,
                    reinterpret_cast<float*>(out + w.o_y), reinterpret_cast<float*>(out + w.o_g),
                    reinterpret_cast<float*>(out + w.o_r), ws + w.cell,
                    w.carry[0] - w.cell, c.B, len, c.H, c.N};
        if (k > 0) {  // resume from the state chunk k-1 left
            char* ci = ws + w.carry[sl];
            cc.cin_h = ci + w.c_h;
            cc.cin_u = reinterpret_cast<const float*>(ci + w.c_u);
            cc.cin_B = ci + w.c_B;
            cc.cin_C = ci + w.c_C;
            cc.cin_row = ci + w.c_row;
        }
        if (k + 1 < nch) {
            char* co = ws + w.carry[sl ^ 1];
            cc.cout_h = co + w.c_h;
            cc.cout_u = reinterpret_cast<float*>(co + w.c_u);
            cc.cout_B = co + w.c_B;
            cc.cout_C = co + w.c_C;
            cc.cout_row = co + w.c_row;
        }
        if ((rc = cell_fwd(cc, stream))) return rc;
        EACS_TRY(cudaEventRecord(p.ev_cell[sl], stream));
        // ---- copy out ----
        EACS_TRY(cudaStreamWaitEvent(p.s_out, p.ev_cell[sl], 0));
        char* yh = reinterpret_cast<char*>(c.y);
        EACS_TRY(cudaMemcpy2DAsync(yh + l0 * c.H * 4, c.L * c.H * 4, out + w.o_y, len * c.H * 4,
                                   len * c.H * 4, c.B, cudaMemcpyDeviceToHost, p.s_out));
        EACS_TRY(cudaMemcpy2DAsync(c.gate + l0, c.L * 4, out + w.o_g, len * 4, len * 4, c.B,
                                   cudaMemcpyDeviceToHost, p.s_out));
        EACS_TRY(cudaMemcpy2DAsync(c.resid + l0, c.L * 4, out + w.o_r, len * 4, len * 4, c.B,
                                   cudaMemcpyDeviceToHost, p.s_out));
        EACS_TRY(cudaEventRecord(p.ev_out[sl], p.s_out));
    }
    // the caller's stream completes when the last outputs are on the host
    EACS_TRY(cudaStreamWaitEvent(stream, p.ev_out[(nch - 1) & 1], 0));
#undef EACS_TRY
    return EACS_OK;
}

}  // namespace eacs
