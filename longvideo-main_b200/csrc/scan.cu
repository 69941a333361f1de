// scan.cu -- materialised variable-step diagonal complex scan (sm_100a).
//
// Forward  h_l = a_l h_{l-1} + b_l                        (24 B per update)
// Backward s_l = g_l + conj(a_{l+1}) s_{l+1}, grad_b = s,
//          grad_a = s conj(h_{l-1})                       (40 B per update)
// over (B, L, C = H*N) complex64, replacing scan_fwd / scan_bwd of
// cst_ssm/ops/csrc/eacs_scan_cuda.cu:23-96.
//
// Both directions are HBM-bound streams.  A CTA owns CB consecutive chains of
// one batch row and walks L in chunks of T steps; one elected thread keeps S
// chunks in flight with 3-D TMA tile loads (box {CB, T, 1}) completing on
// per-stage mbarriers, so DRAM sees deep queues while each thread runs its
// chain's recurrence out of shared memory and streams results straight to
// global memory (a warp writes 256 contiguous bytes per step).  When TMA cannot
// address the tensors (odd C, misaligned base) a plain-load kernel is used.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "eacs_common.cuh"
#include "eacs_host.h"

namespace eacs {
namespace {

constexpr int kCB = 64;  // chains per CTA (2 warps)
constexpr int kT = 16;   // steps per chunk
constexpr int kSF = 4;   // forward stages in flight (2 tiles each)
constexpr int kSB = 3;   // backward stages in flight (3 tiles each)

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCB) scan_fwd_tma(const __grid_constant__ CUtensorMap ta,
                                                   const __grid_constant__ CUtensorMap tb,
                                                   float2* __restrict__ h, int L, int64_t C,
                                                   int nblk) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float2* sa = reinterpret_cast<float2*>(smem_raw);               // [kSF][kT][kCB]
    float2* sb = sa + kSF * kT * kCB;                               // [kSF][kT][kCB]
    uint64_t* bar = reinterpret_cast<uint64_t*>(sb + kSF * kT * kCB);  // [kSF]

    const int tid = threadIdx.x;
    const int b = blockIdx.x / nblk;
    const int c0 = (blockIdx.x % nblk) * kCB;
    const int nch = (L + kT - 1) / kT;
    constexpr uint32_t kBytes = 2u * kT * kCB * sizeof(float2);

    if (tid == 0) {
        prefetch_tmap(&ta);
        prefetch_tmap(&tb);
        for (int s = 0; s < kSF; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int s = 0; s < kSF && s < nch; ++s) {
            mbar_expect_tx(&bar[s], kBytes);
            tma_load_3d(sa + s * kT * kCB, &ta, &bar[s], c0, s * kT, b);
            tma_load_3d(sb + s * kT * kCB, &tb, &bar[s], c0, s * kT, b);
        }
    }
    const int64_t c = c0 + tid;
    const bool valid = c < C;
    float2 st = make_float2(0.f, 0.f);
    float2* hp = h + (static_cast<int64_t>(b) * L) * C + c;
    int ch = 0;
    for (; ch < nch; ++ch) {
        const int s = ch % kSF;
        const bool ok = mbar_wait(&bar[s], (ch / kSF) & 1);
        if (!__syncthreads_and(ok)) break;
        const float2* xa = sa + s * kT * kCB;
        const float2* xb = sb + s * kT * kCB;
        const int l0 = ch * kT;
        const int steps = min(kT, L - l0);
        if (steps == kT) {
#pragma unroll
            for (int i = 0; i < kT; ++i) {
                const float2 av = xa[i * kCB + tid];
                const float2 bv = xb[i * kCB + tid];
                st = cadd(cmul(av, st), bv);
                if (valid) __stcs(hp + static_cast<int64_t>(l0 + i) * C, st);
            }
        } else {
            for (int i = 0; i < steps; ++i) {
                const float2 av = xa[i * kCB + tid];
                const float2 bv = xb[i * kCB + tid];
                st = cadd(cmul(av, st), bv);
                if (valid) __stcs(hp + static_cast<int64_t>(l0 + i) * C, st);
            }
        }
        __syncthreads();
        if (tid == 0 && ch + kSF < nch) {
            mbar_expect_tx(&bar[s], kBytes);
            tma_load_3d(sa + s * kT * kCB, &ta, &bar[s], c0, (ch + kSF) * kT, b);
            tma_load_3d(sb + s * kT * kCB, &tb, &bar[s], c0, (ch + kSF) * kT, b);
        }
    }
    if (ch < nch && tid == 0) {
        // A wait expired: drain the loads still in flight (bounded) before exit.
        for (int k = ch; k < nch && k < ch + kSF; ++k) mbar_wait(&bar[k % kSF], (k / kSF) & 1);
    }
}

__global__ void scan_fwd_plain(const float2* __restrict__ a, const float2* __restrict__ b,
                               float2* __restrict__ h, int B, int L, int64_t C) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(B) * C) return;
    const int64_t bi = idx / C, c = idx % C;
    const int64_t base = bi * L * C + c;
    float2 st = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int l = 0; l < L; ++l) {
        const int64_t o = base + static_cast<int64_t>(l) * C;
        st = cadd(cmul(__ldg(a + o), st), __ldg(b + o));
        h[o] = st;
    }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCB) scan_bwd_tma(const __grid_constant__ CUtensorMap ta,
                                                   const __grid_constant__ CUtensorMap th,
                                                   const __grid_constant__ CUtensorMap tg,
                                                   float2* __restrict__ ga, float2* __restrict__ gb,
                                                   int L, int64_t C, int nblk) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float2* sa = reinterpret_cast<float2*>(smem_raw);  // [kSB][kT][kCB]
    float2* sh = sa + kSB * kT * kCB;                  // h rows l-1 (shifted by one)
    float2* sg = sh + kSB * kT * kCB;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sg + kSB * kT * kCB);

    const int tid = threadIdx.x;
    const int b = blockIdx.x / nblk;
    const int c0 = (blockIdx.x % nblk) * kCB;
    const int nch = (L + kT - 1) / kT;
    constexpr uint32_t kBytes = 3u * kT * kCB * sizeof(float2);

    auto issue = [&](int k, int s) {
        const int l0 = (nch - 1 - k) * kT;  // k-th chunk from the end
        mbar_expect_tx(&bar[s], kBytes);
        tma_load_3d(sa + s * kT * kCB, &ta, &bar[s], c0, l0, b);
        tma_load_3d(sh + s * kT * kCB, &th, &bar[s], c0, l0 - 1, b);  // row -1 reads as zero
        tma_load_3d(sg + s * kT * kCB, &tg, &bar[s], c0, l0, b);
    };
    if (tid == 0) {
        prefetch_tmap(&ta);
        prefetch_tmap(&th);
        prefetch_tmap(&tg);
        for (int s = 0; s < kSB; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int k = 0; k < kSB && k < nch; ++k) issue(k, k);

    const int64_t c = c0 + tid;
    const bool valid = c < C;
    float2 s_adj = make_float2(0.f, 0.f);
    const int64_t base = static_cast<int64_t>(b) * L * C + c;
    int k = 0;
    for (; k < nch; ++k) {
        const int s = k % kSB;
        const bool ok = mbar_wait(&bar[s], (k / kSB) & 1);
        if (!__syncthreads_and(ok)) break;
        const float2* xa = sa + s * kT * kCB;
        const float2* xh = sh + s * kT * kCB;
        const float2* xg = sg + s * kT * kCB;
        const int l0 = (nch - 1 - k) * kT;
        const int steps = min(kT, L - l0);
        for (int i = steps - 1; i >= 0; --i) {
            const float2 g = xg[i * kCB + tid];
            s_adj = cadd(s_adj, g);
            const float2 hp = xh[i * kCB + tid];
            const float2 gav = cmul(s_adj, make_float2(hp.x, -hp.y));
            if (valid) {
                const int64_t o = base + static_cast<int64_t>(l0 + i) * C;
                __stcs(gb + o, s_adj);
                __stcs(ga + o, gav);
            }
            const float2 av = xa[i * kCB + tid];
            s_adj = cmul(make_float2(av.x, -av.y), s_adj);
        }
        __syncthreads();
        if (tid == 0 && k + kSB < nch) issue(k + kSB, s);
    }
    if (k < nch && tid == 0)
        for (int j = k; j < nch && j < k + kSB; ++j) mbar_wait(&bar[j % kSB], (j / kSB) & 1);
}

__global__ void scan_bwd_plain(const float2* __restrict__ a, const float2* __restrict__ h,
                               const float2* __restrict__ gh, float2* __restrict__ ga,
                               float2* __restrict__ gb, int B, int L, int64_t C) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(B) * C) return;
    const int64_t bi = idx / C, c = idx % C;
    const int64_t base = bi * L * C + c;
    float2 s = make_float2(0.f, 0.f);
    for (int l = L - 1; l >= 0; --l) {
        const int64_t o = base + static_cast<int64_t>(l) * C;
        s = cadd(s, __ldg(gh + o));
        gb[o] = s;
        const float2 hp = l > 0 ? __ldg(h + o - C) : make_float2(0.f, 0.f);
        ga[o] = cmul(s, make_float2(hp.x, -hp.y));
        const float2 av = __ldg(a + o);
        s = cmul(make_float2(av.x, -av.y), s);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tensor map over a (B, L, C) tensor of 8-byte complex64 elements, box {CB, T, 1}.
bool make_map(CUtensorMap* m, const void* base, int64_t B, int64_t L, int64_t C) {
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(L),
                          static_cast<cuuint64_t>(B)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(C * 8), static_cast<cuuint64_t>(L * C * 8)};
    cuuint32_t box[3] = {kCB, kT, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool tma_ok(int64_t B, int64_t L, int64_t C, std::initializer_list<const void*> ptrs) {
    if ((C & 1) != 0) return false;                 // row stride C*8 must be a multiple of 16
    if (B > 65535 || L > (1LL << 31) - 1 || C > (1LL << 31) - 1) return false;
    for (const void* p : ptrs)
        if ((reinterpret_cast<uintptr_t>(p) & 15) != 0) return false;
    return get_encode() != nullptr;
}

}  // namespace

int scan_fwd(const void* a, const void* b, void* h, int64_t B, int64_t L, int64_t C,
             cudaStream_t stream) {
    if (B * L * C == 0) return EACS_OK;
    if (!a || !b || !h) return fail(EACS_ERR_INVALID, "eacs_scan_fwd: null pointer");
    if (L > (1LL << 31) - 1) return fail(EACS_ERR_UNSUPPORTED, "eacs_scan_fwd: L too large");
    if (tma_ok(B, L, C, {a, b, h})) {
        CUtensorMap ta, tb;
        if (make_map(&ta, a, B, L, C) && make_map(&tb, b, B, L, C)) {
            const int nblk = static_cast<int>((C + kCB - 1) / kCB);
            const size_t smem = 2 * kSF * kT * kCB * sizeof(float2) + kSF * sizeof(uint64_t);
            cudaFuncSetAttribute(scan_fwd_tma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
            const int64_t grid = B * nblk;
            if (grid <= 0x7fffffff) {
                mark_start(stream);
                scan_fwd_tma<<<static_cast<unsigned>(grid), kCB, smem, stream>>>(
                    ta, tb, static_cast<float2*>(h), static_cast<int>(L), C, nblk);
                mark_stop(stream);
                note_launch();
                return cuda_check(cudaGetLastError(), "eacs_scan_fwd (tma)");
            }
        }
    }
    const int64_t n = B * C;
    mark_start(stream);
    scan_fwd_plain<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        static_cast<const float2*>(a), static_cast<const float2*>(b), static_cast<float2*>(h),
        static_cast<int>(B), static_cast<int>(L), C);
    mark_stop(stream);
    note_launch();
    return cuda_check(cudaGetLastError(), "eacs_scan_fwd (plain)");
}

int scan_bwd(const void* a, const void* h, const void* gh, void* ga, void* gb, int64_t B,
             int64_t L, int64_t C, cudaStream_t stream) {
    if (B * L * C == 0) return EACS_OK;
    if (!a || !h || !gh || !ga || !gb) return fail(EACS_ERR_INVALID, "eacs_scan_bwd: null pointer");
    if (L > (1LL << 31) - 1) return fail(EACS_ERR_UNSUPPORTED, "eacs_scan_bwd: L too large");
    if (tma_ok(B, L, C, {a, h, gh, ga, gb})) {
        CUtensorMap ta, th, tg;
        if (make_map(&ta, a, B, L, C) && make_map(&th, h, B, L, C) && make_map(&tg, gh, B, L, C)) {
            const int nblk = static_cast<int>((C + kCB - 1) / kCB);
            const size_t smem = 3 * kSB * kT * kCB * sizeof(float2) + kSB * sizeof(uint64_t);
            cudaFuncSetAttribute(scan_bwd_tma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
            const int64_t grid = B * nblk;
            if (grid <= 0x7fffffff) {
                mark_start(stream);
                scan_bwd_tma<<<static_cast<unsigned>(grid), kCB, smem, stream>>>(
                    ta, th, tg, static_cast<float2*>(ga), static_cast<float2*>(gb),
                    static_cast<int>(L), C, nblk);
                mark_stop(stream);
                note_launch();
                return cuda_check(cudaGetLastError(), "eacs_scan_bwd (tma)");
            }
        }
    }
    const int64_t n = B * C;
    mark_start(stream);
    scan_bwd_plain<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        static_cast<const float2*>(a), static_cast<const float2*>(h),
        static_cast<const float2*>(gh), static_cast<float2*>(ga), static_cast<float2*>(gb),
        static_cast<int>(B), static_cast<int>(L), C);
    mark_stop(stream);
    note_launch();
    return cuda_check(cudaGetLastError(), "eacs_scan_bwd (plain)");
}

cudaError_t scan_read_status(int* out, cudaStream_t stream) { return read_clear_status(out, stream); }

}  // namespace eacs
