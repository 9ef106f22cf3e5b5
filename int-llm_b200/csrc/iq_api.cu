// iq_api.cu -- the C ABI of libiq.so (declared in include/iq.h).
// Single translation unit: the kernel headers are included here.
#include <mutex>
#include <algorithm>
#include <unordered_map>
#include <vector>
#include <cstring>
#include <cstdlib>
#include "iq_common.cuh"
#include "iq_fpmath.cuh"
#include "iq_matvec.cuh"
#include "iq_gemm.cuh"
#include "iq_planes.cuh"
#include "iq_tc_gemm.cuh"
#include "iq_planes_smem.cuh"
#include "iq_elem.cuh"
#include "iq_peak.cuh"

namespace iq {

static int g_last_cuda = 0;

int cuda_fail(cudaError_t e) {
    g_last_cuda = (int)e;
    if (e == cudaErrorMemoryAllocation) return IQ_ERR_OOM;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ||
        e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDevice)
        return IQ_ERR_UNSUPPORTED;
    return IQ_ERR_CUDA;
}

struct DevState {
    bool ready = false;
    DevInfo info;
    cudaStream_t stream = nullptr;
};
static std::mutex g_mu;
static DevState g_dev[64];
static int g_host_device = 0;

static int ensure_device(int dev) {
    if (dev < 0 || dev >= 64) return IQ_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_mu);
    DevState &d = g_dev[dev];
    if (d.ready) return IQ_OK;
    cudaDeviceProp p;
    IQ_CUDA(cudaGetDeviceProperties(&p, dev));
    d.info.sms = p.multiProcessorCount;
    d.info.smem_optin = (int)p.sharedMemPerBlockOptin;
    d.info.cc_major = p.major;
    d.info.cc_minor = p.minor;
    if (p.major != 10) return IQ_ERR_UNSUPPORTED;  // built for sm_100a only
    IQ_CUDA(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
    k_cordic_init<<<1, 1, 0, d.stream>>>();
    IQ_CHECK_LAUNCH();
    IQ_CUDA(cudaStreamSynchronize(d.stream));
    d.ready = true;
    return IQ_OK;
}

int ensure_device_pub(int dev) { return ensure_device(dev); }

static int cur_device(int *dev) {
    IQ_CUDA(cudaGetDevice(dev));
    return ensure_device(*dev);
}

const DevInfo &dev_info() {
    int d = 0;
    cudaGetDevice(&d);
    return g_dev[d].info;
}
cudaStream_t lib_stream() {
    int d = 0;
    cudaGetDevice(&d);
    return g_dev[d].stream;
}

// ------------------------------------------------------------ launchers

template <int WPR, int UNROLL, bool VEC, bool XSMEM>
static int launch_mv_t(int64_t *out, const int64_t *W, const int64_t *x, int M, int N, int add, cudaStream_t s) {
    auto kern = k_matvec<WPR, UNROLL, VEC, XSMEM>;
    size_t smem = XSMEM ? (size_t)N * sizeof(int64_t) : 0;
    // static shared memory counts against the 48 KB default too
    if (smem > 40 * 1024) IQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int occ = 0;
    IQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, smem));
    if (occ < 1) occ = 1;
    int rpc = 8 / WPR;
    int ctas_needed = (M + rpc - 1) / rpc;
    int grid = dev_info().sms * occ;
    if (grid > ctas_needed) grid = ctas_needed;
    kern<<<grid, 256, smem, s>>>(out, W, x, M, N, add);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

template <bool VEC, bool XSMEM>
static int launch_mv_v(int64_t *out, const int64_t *W, const int64_t *x, int M, int N, int add, cudaStream_t s) {
    // split rows over enough warps to fill the GPU: ~16 warps per SM
    int want = dev_info().sms * 16;
    static int force = getenv("IQ_MV_WPR") ? atoi(getenv("IQ_MV_WPR")) : 0;
    int wpr = force ? force : (M >= want ? 1 : M * 2 >= want ? 2 : M * 4 >= want ? 4 : 8);
    if (N < 64 * wpr) wpr = 1;
    switch (wpr) {
    case 1: return launch_mv_t<1, 8, VEC, XSMEM>(out, W, x, M, N, add, s);
    case 2: return launch_mv_t<2, 8, VEC, XSMEM>(out, W, x, M, N, add, s);
    case 4: return launch_mv_t<4, 8, VEC, XSMEM>(out, W, x, M, N, add, s);
    default: return launch_mv_t<8, 8, VEC, XSMEM>(out, W, x, M, N, add, s);
    }
}

int launch_matvec(int64_t *out, const int64_t *W, const int64_t *x, int M, int N, cudaStream_t s, int add = 0) {
    // 16-byte weight loads need an even row length and a 16-byte aligned base;
    // x is read as 16-byte pairs too, from shared memory (always aligned) or,
    // for long rows, from global memory (then x must be 16-byte aligned).
    bool xsmem = (size_t)N * 8 <= 96 * 1024;
    bool vec = ((N & 1) == 0) && (((uintptr_t)W & 15) == 0) && (xsmem || (((uintptr_t)x & 15) == 0));
    if (vec && xsmem) return launch_mv_v<true, true>(out, W, x, M, N, add, s);
    if (vec) return launch_mv_v<true, false>(out, W, x, M, N, add, s);
    if (xsmem) return launch_mv_v<false, true>(out, W, x, M, N, add, s);
    return launch_mv_v<false, false>(out, W, x, M, N, add, s);
}

int launch_gemm_add(int64_t *out, const int64_t *W, const int64_t *X, int rows, int M, int N, cudaStream_t s,
                    int add) {
    constexpr int BM = 64, BR = 32, BK = 32, TM = 4, TR = 2;
    dim3 grid((M + BM - 1) / BM, (rows + BR - 1) / BR);
    k_gemm<BM, BR, BK, TM, TR><<<grid, (BM / TM) * (BR / TR), 0, s>>>(out, W, X, rows, M, N, add);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

// ------------------------------------------------- byte-plane matvec

// Plane statistics of a matrix (see k_plane_count): top = bytes needed as a
// signed integer, low[b] = weights whose lowest nonzero byte is b. Synchronises s.
static int plane_stats(const int64_t *d_w, int64_t n, cudaStream_t s, int *top, unsigned long long low[8]) {
    unsigned long long *d = nullptr, h[9] = {1, 0, 0, 0, 0, 0, 0, 0, 0};
    IQ_CUDA(cudaMalloc(&d, sizeof(h)));
    cudaError_t e = cudaMemcpyAsync(d, h, sizeof(h), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        k_plane_count<<<(int)std::min<int64_t>((n + 255) / 256, (int64_t)dev_info().sms * 16), 256, 0, s>>>(d, d_w, n);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e);
    *top = (int)h[0];
    for (int b = 0; b < 8; b++) low[b] = h[1 + b];
    return IQ_OK;
}

// Number of byte planes a matrix needs when all are kept from plane 0.
static int count_planes(const int64_t *d_w, int64_t n, cudaStream_t s, int *np) {
    unsigned long long low[8];
    return plane_stats(d_w, n, s, np, low);
}

// Lowest stored plane: the p0 that saves the most bytes, counting each
// residual entry (4-byte column + 8-byte value + its share of row offsets)
// as 16 bytes against Mp*Kp bytes per dropped plane, among the p0 whose
// residual stays at most one entry per 2^density_log2 weights (the entries are
// added serially by the row's writer, so density costs latency: the matvec
// allows 1/1024; the GEMM's epilogue pays 32 strided loads per entry and holds
// its CTA meanwhile, so it allows 1/2^20).
// IQ_PLANE_P0 (0..7) in the environment caps it (0 = keep every plane).
static int choose_p0(int top, const unsigned long long low[8], int64_t plane_bytes, int density_log2) {
    static const int cap = getenv("IQ_PLANE_P0") ? atoi(getenv("IQ_PLANE_P0")) : 8;
    int best = 0;
    long double best_gain = 0, below = 0;
    for (int p0 = 1; p0 < top && p0 <= cap; p0++) {
        below += (long double)low[p0 - 1];
        const long double gain = (long double)p0 * plane_bytes - 16.0L * below;
        if (below * (long double)(1ull << density_log2) > (long double)plane_bytes) break;
        if (gain > best_gain) { best_gain = gain; best = p0; }
    }
    return best;
}

static void free_packed(Packed *P);

// Sparse residual of the plane window (see iq_planes.cuh): CSR over rows_pad
// rows of the weights' bits in `mask` (the bytes below p0); nnz entries, in
// column order per row. Synchronises s.
static int build_residual(const int64_t *d_w, int M, int N, int rows_pad, int nnz, uint64_t mask,
                          cudaStream_t s, int *res_ptr, int *res_col, int64_t *res_val) {
    std::vector<int> cnt(rows_pad + 1, 0);
    IQ_CUDA(cudaMemsetAsync(res_ptr, 0, (size_t)(rows_pad + 1) * sizeof(int), s));
    const int g = std::min((M + 7) / 8, dev_info().sms * 16);
    k_res_count<<<g, 256, 0, s>>>(res_ptr, d_w, M, N, mask);
    IQ_CHECK_LAUNCH();
    IQ_CUDA(cudaMemcpyAsync(cnt.data(), res_ptr, (size_t)rows_pad * sizeof(int), cudaMemcpyDeviceToHost, s));
    IQ_CUDA(cudaStreamSynchronize(s));
    int run = 0;  // exclusive scan on the host
    for (int r = 0; r <= rows_pad; r++) { int c = r < rows_pad ? cnt[r] : 0; cnt[r] = run; run += c; }
    if (run != nnz) return IQ_ERR_STATE;
    IQ_CUDA(cudaMemcpyAsync(res_ptr, cnt.data(), (size_t)(rows_pad + 1) * sizeof(int), cudaMemcpyHostToDevice, s));
    k_res_fill<<<g, 256, 0, s>>>(res_col, res_val, res_ptr, d_w, M, N, mask);
    IQ_CHECK_LAUNCH();
    IQ_CUDA(cudaStreamSynchronize(s));  // cnt is a host buffer that goes out of scope
    return IQ_OK;
}

// Weights the bf16 form cannot hold (its residual entries). Synchronises s.
static int bf_residual_count(const int64_t *d_w, int64_t n, cudaStream_t s, unsigned long long *cnt) {
    unsigned long long *d = nullptr;
    IQ_CUDA(cudaMalloc(&d, sizeof(unsigned long long)));
    cudaError_t e = cudaMemsetAsync(d, 0, sizeof(unsigned long long), s);
    if (e == cudaSuccess) {
        k_bf_count<<<(int)std::min<int64_t>((n + 255) / 256, (int64_t)dev_info().sms * 16), 256, 0, s>>>(d, d_w, n);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(cnt, d, sizeof(unsigned long long), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e);
    return IQ_OK;
}

// The matvec form: the bf16 form (2 bytes per weight) when it holds all but
// at most one weight in 1024 exactly, the activations can be staged
// (Kp <= 12784) and it is smaller than the plane window; else the window.
// IQ_MV_FORMAT=planes|bf16 forces one (bf16 only where it applies).
// want: -1 = choose, IQ_FMT_PLANES or IQ_FMT_BF16 = that form (bf16: any
// weights, however many residual entries; IQ_ERR_UNSUPPORTED when N is too
// long to stage the activations).
static int pack_weights(const int64_t *d_w, int M, int N, cudaStream_t s, Packed *P, int want = -1) {
    P->M = M; P->N = N;
    P->Mp = (M + 15) / 16 * 16;
    P->Kp = (N + 31) / 32 * 32;
    int top = 8;
    unsigned long long low[8];
    int rc = plane_stats(d_w, (int64_t)M * N, s, &top, low);
    if (rc) return rc;
    P->p0 = choose_p0(top, low, (int64_t)P->Mp * P->Kp, 10);
    P->np = top - P->p0;
    P->nnz = 0;
    for (int b = 0; b < P->p0; b++) P->nnz += (int)low[b];
    P->fmt = IQ_FMT_PLANES;
    static const char *force_env = getenv("IQ_MV_FORMAT");
    const char *force = want == IQ_FMT_PLANES ? "planes" : want == IQ_FMT_BF16 ? "bf16" : force_env;
    const bool allow_bf = !(force && !strcmp(force, "planes"));
    const bool fits = 8 * ((int64_t)P->Kp + 16) <= 100 * 1024;
    if (want == IQ_FMT_BF16 && !fits) return IQ_ERR_UNSUPPORTED;
    if (allow_bf && fits) {
        unsigned long long nbf = 0;
        if ((rc = bf_residual_count(d_w, (int64_t)M * N, s, &nbf))) return rc;
        const int64_t cells = (int64_t)P->Mp * P->Kp;
        const bool sparse = (long double)nbf * 1024.0L <= (long double)cells;
        const long double bytes_bf = 2.0L * cells + 16.0L * nbf, bytes_pl = (long double)P->np * cells + 16.0L * P->nnz;
        if (want == IQ_FMT_BF16 || (sparse && (bytes_bf < bytes_pl || (force && !strcmp(force, "bf16"))))) {
            P->fmt = IQ_FMT_BF16;
            P->np = 3;
            P->p0 = 3;
            P->nnz = (int)nbf;
        }
    }
    if (P->fmt == IQ_FMT_BF16) {
        cudaError_t e = cudaMalloc(&P->planes, (size_t)P->Mp * P->Kp * 2);
        if (e == cudaSuccess) e = cudaMalloc(&P->rowsum, (size_t)P->Mp * 16);
        if (e == cudaSuccess && P->nnz > 0) {
            e = cudaMalloc(&P->res_ptr, (size_t)(P->Mp + 1) * sizeof(int));
            if (e == cudaSuccess) e = cudaMalloc(&P->res_col, (size_t)P->nnz * sizeof(int));
            if (e == cudaSuccess) e = cudaMalloc(&P->res_val, (size_t)P->nnz * sizeof(int64_t));
        }
        if (e != cudaSuccess) { free_packed(P); return cuda_fail(e); }
        const int KT = P->Kp / 32;
        const int64_t total = (int64_t)(P->Mp / 16) * KT * 32;
        k_pack_bf<<<(int)std::min<int64_t>((total + 255) / 256, (int64_t)dev_info().sms * 32), 256, 0, s>>>(
            P->planes, d_w, M, N, KT, total);
        IQ_CHECK_LAUNCH();
        k_bf_row_sums<<<std::min(P->Mp / 8 + 1, dev_info().sms * 16), 256, 0, s>>>(P->rowsum, d_w, M, N, P->Mp);
        IQ_CHECK_LAUNCH();
        if (P->nnz > 0 && (rc = build_residual(d_w, M, N, P->Mp, P->nnz, 0ull, s, P->res_ptr, P->res_col,
                                                P->res_val))) {
            free_packed(P);
            return rc;
        }
        return IQ_OK;
    }
    const uint64_t mask = P->p0 ? (~0ull >> (64 - 8 * P->p0)) : 0ull;
    size_t nbytes = (size_t)P->Mp * P->Kp * P->np;
    cudaError_t e = cudaMalloc(&P->planes, nbytes);
    if (e == cudaSuccess) e = cudaMalloc(&P->rowsum, (size_t)P->Mp * 16);
    if (e == cudaSuccess && P->nnz > 0) {
        e = cudaMalloc(&P->res_ptr, (size_t)(P->Mp + 1) * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&P->res_col, (size_t)P->nnz * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&P->res_val, (size_t)P->nnz * sizeof(int64_t));
    }
    if (e != cudaSuccess) { free_packed(P); return cuda_fail(e); }
    const int KT = P->Kp / 32;
    int64_t total = (int64_t)(P->Mp / 16) * KT * 32;
    int64_t blocks = (total + 255) / 256;
    k_pack_planes<<<(int)std::min<int64_t>(blocks, (int64_t)dev_info().sms * 32), 256, 0, s>>>(
        P->planes, d_w, M, N, KT, total, P->np, P->p0);
    IQ_CHECK_LAUNCH();
    k_row_sums<<<std::min(P->Mp / 8 + 1, dev_info().sms * 16), 256, 0, s>>>(P->rowsum, d_w, M, N, P->Mp, mask);
    IQ_CHECK_LAUNCH();
    if (P->nnz > 0 && (rc = build_residual(d_w, M, N, P->Mp, P->nnz, mask, s, P->res_ptr, P->res_col, P->res_val))) {
        free_packed(P);
        return rc;
    }
    return IQ_OK;
}

static PackedRes packed_res(const Packed &P) {
    return PackedRes{P.p0, P.fmt == IQ_FMT_BF16 ? 1 : 0, P.rowsum, P.res_ptr, P.res_col, P.res_val};
}

static void free_packed(Packed *P) {
    if (P->planes) cudaFree(P->planes);
    if (P->rowsum) cudaFree(P->rowsum);
    if (P->res_ptr) cudaFree(P->res_ptr);
    if (P->res_col) cudaFree(P->res_col);
    if (P->res_val) cudaFree(P->res_val);
    P->planes = nullptr;
    P->rowsum = nullptr;
    P->res_ptr = P->res_col = nullptr;
    P->res_val = nullptr;
    P->nnz = 0;
}

// racc: RowAcc scratch with >= M zeroed entries (zero again on completion).

typedef void (*PlanesKernel)(int64_t *, const uint4 *, const PackedRes, const int64_t *, int, int, int, int,
                             RowAcc *, const int64_t *);
template <bool XS>
static PlanesKernel planes_kernel(int np) {
    switch (np) {
    case 1: return k_matvec_planes<1, XS>;
    case 2: return k_matvec_planes<2, XS>;
    case 3: return k_matvec_planes<3, XS>;
    case 4: return k_matvec_planes<4, XS>;
    case 5: return k_matvec_planes<5, XS>;
    case 6: return k_matvec_planes<6, XS>;
    case 7: return k_matvec_planes<7, XS>;
    default: return k_matvec_planes<8, XS>;
    }
}

typedef void (*RowsKernel)(int64_t *, const uint4 *, const PackedRes, const int64_t *, int, int, int, int,
                           const int64_t *);
// Once per device and plane count: allow the largest staged-digit buffer
// (the 48 KB default covers static + dynamic shared memory together) and
// record the occupancy at that size.
template <int NP, bool BF = false>
static int rows_setup(RowsKernel *k, int *occ) {
    static int occs[64] = {0};
    int dev = 0;
    IQ_CUDA(cudaGetDevice(&dev));
    *k = k_matvec_rows<NP, BF>;
    if (dev >= 0 && dev < 64 && occs[dev]) { *occ = occs[dev]; return IQ_OK; }
    const int smax = 100 * 1024;
    IQ_CUDA(cudaFuncSetAttribute(*k, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    IQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, *k, 256, smax));
    if (*occ < 1) *occ = 1;
    if (dev >= 0 && dev < 64) occs[dev] = *occ;
    return IQ_OK;
}

// Row-owned matvec (k_matvec_rows). When one wave of CTAs covers every row
// tile, the cluster size S is the largest of 1, 2, 4, 8 with rows * S CTAs
// still one wave and at least two column tiles per warp; otherwise S = 1 and
// one wave of CTAs loops over the row tiles. IQ_ERR_UNSUPPORTED = use the
// stream-K kernel.
// The bf16-form row-owned matvec with the weight slice bulk-copied into shared
// memory (k_matvec_rows_smem): used when one wave of CTAs, each holding one
// row tile's column range, fits; cluster size = the smallest S in 1, 2, 4, 8
// that fits (IQ_MV_SMEM=0 disables it; IQ_MV_SMEM_S forces S).
static int launch_matvec_rows_smem(int64_t *out, const Packed &P, const int64_t *x, cudaStream_t s, int add,
                                   const int64_t *nrm_w) {
    static const int enabled = getenv("IQ_MV_SMEM") ? atoi(getenv("IQ_MV_SMEM")) : 1;
    static const int s_force = getenv("IQ_MV_SMEM_S") ? atoi(getenv("IQ_MV_SMEM_S")) : 0;
    if (!enabled || P.fmt != IQ_FMT_BF16) return IQ_ERR_UNSUPPORTED;
    static int smem_max[64] = {0};   // per device: the dynamic shared memory the kernel may use
    int dev = 0;
    IQ_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return IQ_ERR_UNSUPPORTED;
    if (!smem_max[dev]) {
        int optin = 0;
        cudaFuncAttributes fa;
        IQ_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        IQ_CUDA(cudaFuncGetAttributes(&fa, k_matvec_rows_smem));
        const int lim = optin - (int)fa.sharedSizeBytes;
        IQ_CUDA(cudaFuncSetAttribute(k_matvec_rows_smem, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
        smem_max[dev] = lim;
    }
    const int RT = P.Mp / 16, KT = P.Kp / 32;
    const size_t xbytes = ((size_t)8 * (P.Kp + 16) + 127) / 128 * 128;
    for (int S = 1; S <= 8; S *= 2) {
        if (s_force && S != s_force) continue;
        const int per = (KT + S - 1) / S;
        const size_t smem = xbytes + (size_t)per * 1024;
        if (smem > (size_t)smem_max[dev]) continue;
        int occ = 0;
        IQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_matvec_rows_smem, 256, smem));
        if (occ < 1 || (int64_t)RT * S > (int64_t)dev_info().sms * occ) continue;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)S;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.gridDim = dim3((unsigned)(RT * S));
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = S > 1 ? 2 : 1;
        IQ_CUDA(cudaLaunchKernelEx(&cfg, k_matvec_rows_smem, out, (const uint4 *)P.planes, packed_res(P), x, P.M,
                                   P.N, P.Kp, add, nrm_w, (int)xbytes));
        IQ_CHECK_LAUNCH();
        return IQ_OK;
    }
    // a few row tiles per CTA (up to 3 per SM): a ring of whole-row-tile slots
    // per CTA (measured: 2048 -> 5632 at 10.9 us against 14.7 for the two-wave
    // row-owned kernel; beyond that stream-K wins, e.g. the 2048 -> 32000 LM
    // head at 35 us against 53)
    static const int pipe_on = getenv("IQ_MV_PIPE") ? atoi(getenv("IQ_MV_PIPE")) : 1;
    if (!pipe_on || RT > 3 * dev_info().sms) return IQ_ERR_UNSUPPORTED;
    static int pmax[64] = {0};
    if (!pmax[dev]) {
        int optin = 0;
        cudaFuncAttributes fa;
        IQ_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        IQ_CUDA(cudaFuncGetAttributes(&fa, k_matvec_rows_pipe));
        pmax[dev] = optin - (int)fa.sharedSizeBytes;
        IQ_CUDA(cudaFuncSetAttribute(k_matvec_rows_pipe, cudaFuncAttributeMaxDynamicSharedMemorySize, pmax[dev]));
    }
    const size_t tile = (size_t)KT * 1024;
    int stages = 3;
    while (stages > 2 && xbytes + stages * tile > (size_t)pmax[dev]) stages--;
    if (xbytes + stages * tile > (size_t)pmax[dev]) return IQ_ERR_UNSUPPORTED;
    const size_t smem = xbytes + stages * tile;
    const int grid = std::min(RT, dev_info().sms);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    IQ_CUDA(cudaLaunchKernelEx(&cfg, k_matvec_rows_pipe, out, (const uint4 *)P.planes, packed_res(P), x, P.M, P.N,
                               P.Kp, add, nrm_w, (int)xbytes, stages));
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

int launch_matvec_rows(int64_t *out, const Packed &P, const int64_t *x, cudaStream_t s, int add,
                       const int64_t *nrm_w, size_t smem) {
    {
        const int rc = launch_matvec_rows_smem(out, P, x, s, add, nrm_w);
        if (rc != IQ_ERR_UNSUPPORTED) return rc;
    }
    // IQ_MV_ROWS: 0 = stream-K only, 1 = row-owned when one wave covers the
    // rows, 2 (default) = row-owned also up to two waves (CTAs loop over tiles)
    static const int mode = getenv("IQ_MV_ROWS") ? atoi(getenv("IQ_MV_ROWS")) : 2;
    if (mode == 0) return IQ_ERR_UNSUPPORTED;
    RowsKernel kern = nullptr;
    int occ = 0, rc = IQ_OK;
    switch (P.fmt == IQ_FMT_BF16 ? 0 : P.np) {
    case 0: rc = rows_setup<3, true>(&kern, &occ); break;
    case 1: rc = rows_setup<1>(&kern, &occ); break;
    case 2: rc = rows_setup<2>(&kern, &occ); break;
    case 3: rc = rows_setup<3>(&kern, &occ); break;
    case 4: rc = rows_setup<4>(&kern, &occ); break;
    case 5: rc = rows_setup<5>(&kern, &occ); break;
    case 6: rc = rows_setup<6>(&kern, &occ); break;
    case 7: rc = rows_setup<7>(&kern, &occ); break;
    default: rc = rows_setup<8>(&kern, &occ); break;
    }
    if (rc) return rc;
    const int64_t slots = (int64_t)dev_info().sms * (occ < 1 ? 1 : occ);
    const int RT = P.Mp / 16, KT = P.Kp / 32;
    // beyond two waves the stream-K kernel's even split wins (measured: 1.2 waves
    // row-owned +2%, 6.8 waves -4%)
    static const int waves = getenv("IQ_MV_ROWS_WAVES") ? atoi(getenv("IQ_MV_ROWS_WAVES")) : 2;
    if (RT > slots && (mode < 2 || RT > (int64_t)waves * slots)) return IQ_ERR_UNSUPPORTED;
    int S = 1;
    static const int s_env = getenv("IQ_MV_CLUSTER") ? atoi(getenv("IQ_MV_CLUSTER")) : 0;
    if (s_env > 0) {   // forced cluster size (measurement aid)
        while (S < s_env && (int64_t)RT * S * 2 <= 2 * slots) S *= 2;
    } else {
        while (S < 8 && (int64_t)RT * S * 2 <= slots && KT >= 2 * 8 * S * 2) S *= 2;
    }
    const int64_t grid = RT > slots ? slots : (int64_t)RT * S;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)S;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = S > 1 ? 2 : 1;
    IQ_CUDA(cudaLaunchKernelEx(&cfg, kern, out, (const uint4 *)P.planes, packed_res(P), x, P.M, P.N, P.Kp, add,
                               nrm_w));
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

// nrm_w != nullptr: x is un-normalised and rmsnorm with weights nrm_w is fused
// into the digit staging; returns IQ_ERR_UNSUPPORTED if x is too long to stage.
int launch_matvec_planes(int64_t *out, const Packed &P, const int64_t *x, cudaStream_t s, int add, RowAcc *racc,
                         const int64_t *nrm_w = nullptr) {
    size_t smem = (size_t)8 * (P.Kp + 16);
    bool xs = smem <= 100 * 1024;
    if (nrm_w && !xs) return IQ_ERR_UNSUPPORTED;
    if (xs) {
        int rc = launch_matvec_rows(out, P, x, s, add, nrm_w, smem);
        if (rc != IQ_ERR_UNSUPPORTED) return rc;
    }
    if (P.fmt == IQ_FMT_BF16 && !xs) return IQ_ERR_STATE;  // packing guarantees staged activations
    PlanesKernel kern = P.fmt == IQ_FMT_BF16 ? k_matvec_planes<3, true, true>
                        : xs ? planes_kernel<true>(P.np) : planes_kernel<false>(P.np);
    if (!xs) smem = 0;
    // static shared memory counts against the 48 KB default too
    if (smem > 40 * 1024) IQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int occ = 0;
    IQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, smem));
    if (occ < 1) occ = 1;
    int64_t units = (int64_t)(P.Mp / 16) * (P.Kp / 32);
    int64_t grid = (int64_t)dev_info().sms * occ;
    int64_t need = (units + 7) / 8;
    if (grid > need) grid = need;
    if (grid < 1) grid = 1;
    // launched with programmatic stream serialisation (see k_matvec_planes)
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    IQ_CUDA(cudaLaunchKernelEx(&cfg, kern, out, (const uint4 *)P.planes, packed_res(P), x, P.M, P.N, P.Kp, add,
                               racc, nrm_w));
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

// Library-owned RowAcc scratch per (device, stream), grown on demand outside
// stream capture. Launches on one stream are ordered, so they share it safely.
struct ScratchKey {
    int dev; cudaStream_t s;
    bool operator==(const ScratchKey &o) const { return dev == o.dev && s == o.s; }
};
struct ScratchHash {
    size_t operator()(const ScratchKey &k) const { return std::hash<void *>()((void *)k.s) ^ (size_t)k.dev; }
};
struct ScratchBuf { RowAcc *p = nullptr; size_t cap = 0; };
static std::mutex g_scr_mu;
static std::unordered_map<ScratchKey, ScratchBuf, ScratchHash> g_scr;

int stream_scratch(cudaStream_t s, size_t rows, RowAcc **out) {
    int dev = 0;
    IQ_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_scr_mu);
    ScratchBuf &b = g_scr[ScratchKey{dev, s}];
    if (b.cap < rows) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        IQ_CUDA(cudaStreamIsCapturing(s, &cs));
        if (cs != cudaStreamCaptureStatusNone) return IQ_ERR_STATE;  // grow before capturing
        size_t n = rows < 65536 ? 65536 : rows;
        RowAcc *p = nullptr;
        if (b.p) { IQ_CUDA(cudaStreamSynchronize(s)); cudaFree(b.p); b.p = nullptr; b.cap = 0; }
        IQ_CUDA(cudaMalloc(&p, n * sizeof(RowAcc)));
        IQ_CUDA(cudaMemsetAsync(p, 0, n * sizeof(RowAcc), s));
        b.p = p;
        b.cap = n;
    }
    *out = b.p;
    return IQ_OK;
}

// ------------------------------------------------ tcgen05 GEMM (rows >= 2)

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);
static PFN_encodeTiled g_encode = nullptr;

static int get_encoder() {
    if (g_encode) return IQ_OK;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    IQ_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) return IQ_ERR_UNSUPPORTED;
    g_encode = (PFN_encodeTiled)fn;
    return IQ_OK;
}

// 2-D map over a [rows][cols] byte matrix, box {128 bytes, box_rows}, 128-byte swizzle
static int encode_u8_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    int rc = get_encoder();
    if (rc) return rc;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? IQ_OK : IQ_ERR_CUDA;
}

struct PackedTC {
    int M = 0, K = 0, Mpad = 0, Kpad = 0, np = 8, p0 = 0, nnz = 0;
    uint8_t *planes = nullptr;   // [np][Mpad][Kpad]: bytes p0 .. p0+np-1
    int64_t *rowsum = nullptr;   // [Mpad][2] (128-bit sum of w_hi)
    int *res_ptr = nullptr, *res_col = nullptr;  // sparse residual (CSR over Mpad rows)
    int64_t *res_val = nullptr;
    CUtensorMap mapA;
};

static void free_packed_tc(PackedTC *P) {
    if (P->planes) cudaFree(P->planes);
    if (P->rowsum) cudaFree(P->rowsum);
    if (P->res_ptr) cudaFree(P->res_ptr);
    if (P->res_col) cudaFree(P->res_col);
    if (P->res_val) cudaFree(P->res_val);
    P->planes = nullptr;
    P->rowsum = nullptr;
    P->res_ptr = P->res_col = nullptr;
    P->res_val = nullptr;
    P->nnz = 0;
}

static PackedRes packed_res(const PackedTC &P) {
    return PackedRes{P.p0, 0, P.rowsum, P.res_ptr, P.res_col, P.res_val};
}

static int pack_weights_tc(const int64_t *d_w, int M, int K, cudaStream_t s, PackedTC *P) {
    if (K > 32768) return IQ_ERR_UNSUPPORTED;  // int32 partials exact up to 33025 terms
    P->M = M; P->K = K;
    P->Mpad = (M + TC_BM - 1) / TC_BM * TC_BM;
    P->Kpad = (K + TC_BK - 1) / TC_BK * TC_BK;
    int top = 8;
    unsigned long long low[8];
    int rc = plane_stats(d_w, (int64_t)M * K, s, &top, low);
    if (rc) return rc;
    P->p0 = choose_p0(top, low, (int64_t)P->Mpad * P->Kpad, 20);
    P->np = top - P->p0;
    P->nnz = 0;
    for (int b = 0; b < P->p0; b++) P->nnz += (int)low[b];
    const uint64_t mask = P->p0 ? (~0ull >> (64 - 8 * P->p0)) : 0ull;
    size_t n = (size_t)P->Mpad * P->Kpad;
    cudaError_t e = cudaMalloc(&P->planes, (size_t)P->np * n);
    if (e == cudaSuccess) e = cudaMalloc(&P->rowsum, (size_t)P->Mpad * 16);
    if (e == cudaSuccess && P->nnz > 0) {
        e = cudaMalloc(&P->res_ptr, (size_t)(P->Mpad + 1) * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&P->res_col, (size_t)P->nnz * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&P->res_val, (size_t)P->nnz * sizeof(int64_t));
    }
    if (e != cudaSuccess) { free_packed_tc(P); return cuda_fail(e); }
    k_pack_rowplanes<<<(int)std::min<size_t>((n + 255) / 256, (size_t)dev_info().sms * 64), 256, 0, s>>>(
        P->planes, d_w, M, K, P->Mpad, P->Kpad, P->np, P->p0);
    IQ_CHECK_LAUNCH();
    k_row_sums<<<std::min(P->Mpad / 8 + 1, dev_info().sms * 16), 256, 0, s>>>(P->rowsum, d_w, M, K, P->Mpad,
                                                                            mask);
    IQ_CHECK_LAUNCH();
    if (P->nnz > 0 &&
        (rc = build_residual(d_w, M, K, P->Mpad, P->nnz, mask, s, P->res_ptr, P->res_col, P->res_val))) {
        free_packed_tc(P);
        return rc;
    }
    rc = encode_u8_map(&P->mapA, P->planes, (uint64_t)P->np * P->Mpad, (uint64_t)P->Kpad, TC_BM);
    if (rc) { free_packed_tc(P); return rc; }
    return IQ_OK;
}

// Byte scratch per (device, stream) for the digit matrix, grown outside capture.
struct ByteScratch { uint8_t *p = nullptr; size_t cap = 0; };
static std::mutex g_bs_mu;
static std::unordered_map<ScratchKey, ByteScratch, ScratchHash> g_bs;

static int stream_bytes(cudaStream_t s, size_t bytes, uint8_t **out) {
    int dev = 0;
    IQ_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_bs_mu);
    ByteScratch &b = g_bs[ScratchKey{dev, s}];
    if (b.cap < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        IQ_CUDA(cudaStreamIsCapturing(s, &cs));
        if (cs != cudaStreamCaptureStatusNone) return IQ_ERR_STATE;
        if (b.p) { IQ_CUDA(cudaStreamSynchronize(s)); cudaFree(b.p); b.p = nullptr; b.cap = 0; }
        IQ_CUDA(cudaMalloc(&b.p, bytes));
        b.cap = bytes;
    }
    *out = b.p;
    return IQ_OK;
}

// Split-K factor for decode-sized batches: the ks in 1..16 (each split keeping >= IQ_GEMM_MINKB K blocks,
// default 8: the per-plane epilogue fold is a fixed cost per CTA) that
// minimises waves x K blocks per split, i.e. the time of the longest SM with
// one CTA per SM; ties go to the smaller ks (less partial traffic).
static int gemm_ksplit(const PackedTC &P, int R) {
    static const int minkb = getenv("IQ_GEMM_MINKB") ? std::max(1, atoi(getenv("IQ_GEMM_MINKB"))) : 8;
    const int Rpad = (R + TC_BR - 1) / TC_BR * TC_BR;
    const int tiles = (P.Mpad / TC_BM) * (Rpad / TC_BR), KBall = P.Kpad / TC_BK, sms = dev_info().sms;
    // a full wave of tiles at prefill-sized batches: the partials' traffic outweighs
    // the balance (measured: config-2 down 0.146 -> 0.184 ms at ks = 4); two or
    // more waves: the tile count already balances
    if ((tiles >= sms && Rpad > 128) || tiles >= 2 * sms) return 1;
    int best = 1;
    long best_cost = (long)((tiles + sms - 1) / sms) * KBall;
    for (int ks = 2; ks <= 16 && KBall / ks >= minkb; ks++) {
        const long cost = (long)((tiles * ks + sms - 1) / sms) * ((KBall + ks - 1) / ks);
        if (cost * 20 < best_cost * 19) { best = ks; best_cost = cost; }   // > 5% better
    }
    return best;
}
// bytes of split-K partial scratch launch_gemm_tc needs for (P, R)
size_t gemm_tc_part_bytes(const PackedTC &P, int R) {
    const int ks = gemm_ksplit(P, R);
    if (ks <= 1) return 0;
    const size_t Rpad = (size_t)(R + TC_BR - 1) / TC_BR * TC_BR;
    return (size_t)ks * Rpad * P.Mpad * 16;
}

// out[r][i] (+)= rows of matmul_vec for X [R][K]; digits: >= Rpad*8*Kpad bytes scratch;
// part: >= gemm_tc_part_bytes(P, R) bytes (unused when no split-K is needed)
int launch_gemm_tc(int64_t *out, const PackedTC &P, const int64_t *X, int R, cudaStream_t s, int add,
                   uint8_t *digits, int64_t *part) {
    const int Rpad = (R + TC_BR - 1) / TC_BR * TC_BR;
    int64_t n = (int64_t)Rpad * P.Kpad;
    k_x_digits<<<(int)std::min<int64_t>((n + 255) / 256, (int64_t)dev_info().sms * 64), 256, 0, s>>>(
        digits, X, R, P.K, Rpad, P.Kpad);
    IQ_CHECK_LAUNCH();
    CUtensorMap mapB;
    int rc = encode_u8_map(&mapB, digits, (uint64_t)Rpad * 8, (uint64_t)P.Kpad, TC_BR * 8);
    if (rc) return rc;
    IQ_CUDA(cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
    const int ks = part ? gemm_ksplit(P, R) : 1;
    dim3 grid(Rpad / TC_BR, P.Mpad / TC_BM, ks);
    k_gemm_tc<<<grid, TC_THREADS, TC_SMEM, s>>>(P.mapA, mapB, out, packed_res(P), X, P.K, P.M, R, P.Mpad, P.Kpad, add,
                                         part, Rpad, P.np);
    IQ_CHECK_LAUNCH();
    if (ks > 1) {
        int64_t n = (int64_t)R * P.M;
        k_gemm_reduce<<<(int)std::min<int64_t>((n + 255) / 256, (int64_t)dev_info().sms * 16), 256, 0, s>>>(
            out, part, packed_res(P), X, P.K, P.M, R, P.Mpad, Rpad, ks, add);
        IQ_CHECK_LAUNCH();
    }
    return IQ_OK;
}

// Reads and clears the device status word after a synchronisation point.
int take_dev_error() {
    int v = 0;
    IQ_CUDA(cudaMemcpyFromSymbol(&v, g_iq_err, sizeof(int)));
    if (v) {
        int z = 0;
        IQ_CUDA(cudaMemcpyToSymbol(g_iq_err, &z, sizeof(int)));
    }
    return v;
}

// ------------------------------------------------------- weight cache
//
// The drop-in iq_matmul_vec receives host matrices. Each is uploaded, packed
// and cached on first use. The reference's weights never change after load
// when they are mmap'd or cached (llama_int.c:2464, --cache-layers), but its
// default streaming path reads every layer into fresh malloc'd buffers and
// frees them after the layer (llama_int.c:2840-2872, mgw_stream_load_layer /
// free_layer_weights): a later call can pass a different matrix at the same
// address. So an entry is trusted only while the matrix's content still
// matches what was uploaded:
//   IQ_WCHECK_SAMPLED (default): a 64-bit fingerprint of 1,152 fixed
//     positions (the first and last 64 values and 1,024 spread over the
//     matrix) is recomputed on every call (microseconds); a mismatch uploads
//     the new content;
//   IQ_WCHECK_FULL: a hash of every value is recomputed on every call (host
//     memory bandwidth), and entries are also found by content, so a layer
//     re-read into a new buffer reuses its packed copy without an upload;
//   IQ_WCHECK_NONE: the address alone (weights known to be immutable).
// Entries are evicted least recently used beyond a byte limit of device memory.

struct WEntry {
    Packed P;
    int M = 0, N = 0, dev = 0;
    uint64_t fp_sampled = 0, fp_full = 0;
    bool has_full = false;
    uint64_t last_use = 0;
    int64_t bytes = 0;
};
static std::mutex g_wmu;
static std::unordered_map<uint64_t, WEntry> g_wents;              // id -> entry
static std::unordered_map<const void *, uint64_t> g_wptr;          // host pointer -> id
static std::unordered_map<uint64_t, uint64_t> g_wcontent;          // content key -> id (FULL mode)
static uint64_t g_wnext = 1, g_wclock = 0;
static int g_wcheck = 1;                                           // IQ_WCHECK_SAMPLED
static int64_t g_wlimit = (int64_t)64 << 30, g_wbytes = 0;

static inline uint64_t mix64(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h *= 0xBF58476D1CE4E5B9ull;
    return h ^ (h >> 31);
}

static uint64_t fingerprint_sampled(const int64_t *w, int M, int N) {
    const uint64_t n = (uint64_t)M * (uint64_t)N;
    uint64_t h = mix64(0x6A09E667F3BCC909ull, n);
    const uint64_t edge = n < 64 ? n : 64;
    for (uint64_t i = 0; i < edge; i++) h = mix64(h, (uint64_t)w[i]);
    for (uint64_t i = 0; i < edge; i++) h = mix64(h, (uint64_t)w[n - 1 - i]);
    uint64_t r = 0x243F6A8885A308D3ull;
    for (int k = 0; k < 1024; k++) {
        r = r * 6364136223846793005ull + 1442695040888963407ull;
        const uint64_t i = (uint64_t)(((unsigned __int128)(r >> 11) * n) >> 53);
        h = mix64(h, (uint64_t)w[i]);
    }
    return h;
}

// Every value, four independent lanes (multiply-xor, then a final mix).
static uint64_t fingerprint_full(const int64_t *w, int M, int N) {
    const uint64_t n = (uint64_t)M * (uint64_t)N;
    uint64_t h0 = 0x9E3779B97F4A7C15ull, h1 = 0xC2B2AE3D27D4EB4Full, h2 = 0x165667B19E3779F9ull,
             h3 = 0xD6E8FEB86659FD93ull;
    const uint64_t K0 = 0xFF51AFD7ED558CCDull;
    uint64_t i = 0;
    for (; i + 4 <= n; i += 4) {
        h0 = (h0 ^ (uint64_t)w[i]) * K0;
        h1 = (h1 ^ (uint64_t)w[i + 1]) * K0;
        h2 = (h2 ^ (uint64_t)w[i + 2]) * K0;
        h3 = (h3 ^ (uint64_t)w[i + 3]) * K0;
        h0 ^= h0 >> 29; h1 ^= h1 >> 29; h2 ^= h2 >> 29; h3 ^= h3 >> 29;
    }
    for (; i < n; i++) h0 = mix64(h0, (uint64_t)w[i]);
    return mix64(mix64(mix64(mix64(n, h0), h1), h2), h3);
}

static uint64_t content_key(uint64_t full, int M, int N, int dev) {
    return mix64(mix64(mix64(full, (uint64_t)M), (uint64_t)N), (uint64_t)dev);
}

static void wcache_drop(uint64_t id) {
    auto it = g_wents.find(id);
    if (it == g_wents.end()) return;
    if (it->second.has_full) {
        auto c = g_wcontent.find(content_key(it->second.fp_full, it->second.M, it->second.N, it->second.dev));
        if (c != g_wcontent.end() && c->second == id) g_wcontent.erase(c);
    }
    g_wbytes -= it->second.bytes;
    free_packed(&it->second.P);
    g_wents.erase(it);
    for (auto p = g_wptr.begin(); p != g_wptr.end();)
        p = p->second == id ? g_wptr.erase(p) : std::next(p);
}

// Least recently used entries out until `extra` more bytes fit the limit.
static void wcache_make_room(int64_t extra) {
    while (!g_wents.empty() && g_wbytes + extra > g_wlimit) {
        uint64_t oldest = 0, t = UINT64_MAX;
        for (auto &kv : g_wents)
            if (kv.second.last_use < t) { t = kv.second.last_use; oldest = kv.first; }
        wcache_drop(oldest);
    }
}

static int weight_upload(const int64_t *w, int M, int N, int dev, WEntry *en) {
    size_t bytes = (size_t)M * N * sizeof(int64_t);
    int64_t *d = nullptr;
    IQ_CUDA(cudaMalloc(&d, bytes));
    cudaError_t e = cudaMemcpy(d, w, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { cudaFree(d); return cuda_fail(e); }
    en->M = M; en->N = N; en->dev = dev;
    int rc = pack_weights(d, M, N, 0, &en->P);
    e = cudaDeviceSynchronize();
    cudaFree(d);
    if (rc) return rc;
    if (e != cudaSuccess) { free_packed(&en->P); return cuda_fail(e); }
    en->bytes = packed_bytes(en->P);
    return IQ_OK;
}

// Finds (or uploads) the packed copy of host matrix w [M][N] on dev.
static int weight_lookup(const int64_t *w, int M, int N, int dev, Packed **pp) {
    std::lock_guard<std::mutex> lk(g_wmu);
    const int mode = g_wcheck;
    const uint64_t fs = mode == 1 ? fingerprint_sampled(w, M, N) : 0;
    const uint64_t ff = mode == 2 ? fingerprint_full(w, M, N) : 0;
    auto pit = g_wptr.find(w);
    if (pit != g_wptr.end()) {
        auto eit = g_wents.find(pit->second);
        if (eit != g_wents.end()) {
            WEntry &e = eit->second;
            const bool same = e.M == M && e.N == N && e.dev == dev &&
                              (mode == 0 || (mode == 1 && e.fp_sampled == fs) ||
                               (mode == 2 && e.has_full && e.fp_full == ff));
            if (same) {
                e.last_use = ++g_wclock;
                *pp = &e.P;
                return IQ_OK;
            }
            // the address now holds another matrix: forget the old entry
            // (its packed copy stays findable by content in FULL mode)
            if (!e.has_full) wcache_drop(pit->second);
            else g_wptr.erase(pit);
        } else {
            g_wptr.erase(pit);
        }
    }
    if (mode == 2) {  // the same content under another address
        auto c = g_wcontent.find(content_key(ff, M, N, dev));
        if (c != g_wcontent.end() && g_wents.count(c->second)) {
            WEntry &e = g_wents[c->second];
            e.last_use = ++g_wclock;
            g_wptr[w] = c->second;
            *pp = &e.P;
            return IQ_OK;
        }
    }
    WEntry en;
    int rc = weight_upload(w, M, N, dev, &en);
    if (rc) return rc;
    wcache_make_room(en.bytes);
    en.fp_sampled = fingerprint_sampled(w, M, N);
    en.fp_full = mode == 2 ? ff : 0;
    en.has_full = mode == 2;
    en.last_use = ++g_wclock;
    const uint64_t id = g_wnext++;
    g_wbytes += en.bytes;
    g_wents[id] = en;
    g_wptr[w] = id;
    if (en.has_full) g_wcontent[content_key(ff, M, N, dev)] = id;
    *pp = &g_wents[id].P;
    return IQ_OK;
}

}  // namespace iq

using namespace iq;

// ------------------------------------------------------------ C ABI

extern "C" {

IQ_API const char *iq_status_str(int s) {
    switch (s) {
    case IQ_OK: return "ok";
    case IQ_ERR_ARG: return "invalid argument";
    case IQ_ERR_CUDA: return "CUDA error";
    case IQ_ERR_OOM: return "out of memory";
    case IQ_ERR_NCCL: return "NCCL error";
    case IQ_ERR_TIMEOUT: return "timeout";
    case IQ_ERR_RANGE: return "out of range";
    case IQ_ERR_STATE: return "invalid state";
    case IQ_ERR_UNSUPPORTED: return "unsupported device";
    default: return "unknown status";
    }
}

IQ_API int iq_last_cuda_error(void) { return g_last_cuda; }
IQ_API int iq_version(void) { return 100; }

IQ_API int iq_set_device(int device) {
    int n = 0;
    IQ_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return IQ_ERR_ARG;
    g_host_device = device;
    IQ_CUDA(cudaSetDevice(device));
    return ensure_device(device);
}

IQ_API int iq_weight_register(const int64_t *weight, int M, int N) {
    if (!weight || M <= 0 || N <= 0) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(g_host_device));
    int rc = ensure_device(g_host_device);
    if (rc) return rc;
    Packed *d;
    return weight_lookup(weight, M, N, g_host_device, &d);
}

IQ_API int iq_weight_unregister(const int64_t *weight) {
    std::lock_guard<std::mutex> lk(g_wmu);
    auto it = g_wptr.find(weight);
    if (it == g_wptr.end()) return IQ_ERR_STATE;
    wcache_drop(it->second);
    return IQ_OK;
}

IQ_API int iq_weight_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_wmu);
    for (auto &kv : g_wents) free_packed(&kv.second.P);
    g_wents.clear();
    g_wptr.clear();
    g_wcontent.clear();
    g_wbytes = 0;
    return IQ_OK;
}

IQ_API int iq_weight_check_mode(int mode) {
    if (mode < IQ_WCHECK_NONE || mode > IQ_WCHECK_FULL) return IQ_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_wmu);
    g_wcheck = mode;
    return IQ_OK;
}

IQ_API int iq_weight_cache_limit(int64_t bytes) {
    if (bytes < 0) return IQ_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_wmu);
    g_wlimit = bytes;
    wcache_make_room(0);
    return IQ_OK;
}

IQ_API int iq_weight_cache_stats(int *entries, int64_t *device_bytes) {
    if (!entries || !device_bytes) return IQ_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_wmu);
    *entries = (int)g_wents.size();
    *device_bytes = g_wbytes;
    return IQ_OK;
}

namespace iq {
// Per-device staging buffers for the host-pointer drop-in (grown on demand).
struct Staging { int64_t *d_in = nullptr, *d_out = nullptr; size_t cap_in = 0, cap_out = 0; };
static Staging g_stage[64];
static std::mutex g_stage_mu;

static int stage_grow(int64_t **p, size_t *cap, size_t need) {
    if (*cap >= need) return IQ_OK;
    if (*p) cudaFree(*p);
    *p = nullptr; *cap = 0;
    size_t n = need < 4096 ? 4096 : need;
    IQ_CUDA(cudaMalloc(p, n * sizeof(int64_t)));
    *cap = n;
    return IQ_OK;
}
}  // namespace iq

IQ_API int iq_matmul_vec(int64_t *out, const int64_t *weight, const int64_t *in, int M, int N) {
    if (!out || !weight || !in || M <= 0 || N <= 0) return IQ_ERR_ARG;
    int dev = g_host_device;
    IQ_CUDA(cudaSetDevice(dev));
    int rc = ensure_device(dev);
    if (rc) return rc;
    Packed *dw = nullptr;
    rc = weight_lookup(weight, M, N, dev, &dw);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_stage_mu);
    Staging &st = g_stage[dev];
    if ((rc = stage_grow(&st.d_in, &st.cap_in, (size_t)N))) return rc;
    if ((rc = stage_grow(&st.d_out, &st.cap_out, (size_t)M))) return rc;
    cudaStream_t s = g_dev[dev].stream;
    IQ_CUDA(cudaMemcpyAsync(st.d_in, in, (size_t)N * 8, cudaMemcpyHostToDevice, s));
    RowAcc *racc = nullptr;
    if ((rc = stream_scratch(s, (size_t)dw->Mp, &racc))) return rc;
    if ((rc = launch_matvec_planes(st.d_out, *dw, st.d_in, s, 0, racc))) return rc;
    IQ_CUDA(cudaMemcpyAsync(out, st.d_out, (size_t)M * 8, cudaMemcpyDeviceToHost, s));
    IQ_CUDA(cudaStreamSynchronize(s));
    return IQ_OK;
}

IQ_API int iq_matvec_dev(int64_t *d_out, const int64_t *d_w, const int64_t *d_in, int M, int N, void *stream) {
    if (!d_out || !d_w || !d_in || M <= 0 || N <= 0) return IQ_ERR_ARG;
    if (d_out == d_in) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    return launch_matvec(d_out, d_w, d_in, M, N, pick(stream));
}

IQ_API int iq_gemm_dev(int64_t *d_out, const int64_t *d_w, const int64_t *d_X, int rows, int M, int N, void *stream) {
    if (!d_out || !d_w || !d_X || rows <= 0 || M <= 0 || N <= 0) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    if (rows == 1) return launch_matvec(d_out, d_w, d_X, M, N, pick(stream));
    return launch_gemm_add(d_out, d_w, d_X, rows, M, N, pick(stream), 0);
}

IQ_API int iq_fp_dev(int fn, const int64_t *d_x, const int64_t *d_y, int64_t *d_out, int64_t n, void *stream) {
    if (!d_x || !d_out || n < 0 || fn < 0 || fn > IQ_FN_EXP_DYADIC) return IQ_ERR_ARG;
    if ((fn == IQ_FN_MUL || fn == IQ_FN_DIV || fn == IQ_FN_EXP_DYADIC) && !d_y) return IQ_ERR_ARG;
    if (n == 0) return IQ_OK;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    int64_t blocks = (n + 255) / 256;
    int cap = dev_info().sms * 8;
    k_fp_eval<<<(int)(blocks < cap ? blocks : cap), 256, 0, pick(stream)>>>(fn, d_x, d_y, d_out, n);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

IQ_API int iq_rmsnorm_dev(int64_t *d_out, const int64_t *d_x, const int64_t *d_w, int rows, int dim, void *stream) {
    if (!d_out || !d_x || !d_w || rows <= 0 || dim <= 0) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    k_rmsnorm<<<rows, 256, 0, pick(stream)>>>(d_out, d_x, d_w, dim);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

IQ_API int iq_softmax_dev(int64_t *d_x, int rows, int n, void *stream) {
    if (!d_x || rows <= 0 || n <= 0) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    k_softmax<<<rows, 256, 0, pick(stream)>>>(d_x, n);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

struct iq_packed { Packed P; int dev; };

// Accessor for iq_noalloc.cu (the packed handle's layout stays private here).
const Packed *iq_packed_inner(const iq_packed *w, int *dev) {
    *dev = w->dev;
    return &w->P;
}

IQ_API int iq_pack_weights_fmt_dev(const int64_t *d_w, int M, int N, int fmt, void *stream, iq_packed **out) {
    if (!d_w || !out || M <= 0 || N <= 0 || fmt < -1 || fmt > IQ_FMT_BF16) return IQ_ERR_ARG;
    *out = nullptr;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    iq_packed *p = new iq_packed();
    p->dev = dev;
    if ((rc = pack_weights(d_w, M, N, pick(stream), &p->P, fmt))) { delete p; return rc; }
    *out = p;
    return IQ_OK;
}

IQ_API int iq_pack_weights_dev(const int64_t *d_w, int M, int N, void *stream, iq_packed **out) {
    return iq_pack_weights_fmt_dev(d_w, M, N, -1, stream, out);
}

IQ_API int iq_packed_free(iq_packed *p) {
    if (!p) return IQ_ERR_ARG;
    cudaDeviceSynchronize();
    free_packed(&p->P);
    delete p;
    return IQ_OK;
}

IQ_API int iq_packed_info(const iq_packed *p, int *np, int *p0, int *residual_entries) {
    if (!p || !np || !p0 || !residual_entries) return IQ_ERR_ARG;
    *np = p->P.np;
    *p0 = p->P.p0;
    *residual_entries = p->P.nnz;
    return IQ_OK;
}

IQ_API int iq_packed_format(const iq_packed *p, int *fmt) {
    if (!p || !fmt) return IQ_ERR_ARG;
    *fmt = p->P.fmt;
    return IQ_OK;
}

IQ_API int iq_packed_bytes(const iq_packed *p, int64_t *bytes) {
    if (!p || !bytes) return IQ_ERR_ARG;
    *bytes = packed_bytes(p->P);
    return IQ_OK;
}

IQ_API int iq_matvec_packed_dev(int64_t *d_out, const iq_packed *w, const int64_t *d_in, void *stream) {
    if (!d_out || !w || !d_in || d_out == d_in) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    if (dev != w->dev) return IQ_ERR_ARG;
    cudaStream_t s = pick(stream);
    RowAcc *racc = nullptr;
    if ((rc = stream_scratch(s, (size_t)w->P.Mp, &racc))) return rc;
    return launch_matvec_planes(d_out, w->P, d_in, s, 0, racc);
}

struct iq_packed_tc { PackedTC P; int dev; };

IQ_API int iq_pack_weights_tc_dev(const int64_t *d_w, int M, int N, void *stream, iq_packed_tc **out) {
    if (!d_w || !out || M <= 0 || N <= 0) return IQ_ERR_ARG;
    *out = nullptr;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    iq_packed_tc *p = new iq_packed_tc();
    p->dev = dev;
    if ((rc = pack_weights_tc(d_w, M, N, pick(stream), &p->P))) { delete p; return rc; }
    *out = p;
    return IQ_OK;
}

IQ_API int iq_packed_tc_info(const iq_packed_tc *p, int *np, int *p0, int *residual_entries) {
    if (!p || !np || !p0 || !residual_entries) return IQ_ERR_ARG;
    *np = p->P.np;
    *p0 = p->P.p0;
    *residual_entries = p->P.nnz;
    return IQ_OK;
}

IQ_API int iq_packed_tc_free(iq_packed_tc *p) {
    if (!p) return IQ_ERR_ARG;
    cudaDeviceSynchronize();
    free_packed_tc(&p->P);
    delete p;
    return IQ_OK;
}

IQ_API int iq_gemm_tc_dev(int64_t *d_out, const iq_packed_tc *w, const int64_t *d_X, int rows, void *stream) {
    if (!d_out || !w || !d_X || rows <= 0 || (const void *)d_out == (const void *)d_X) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    if (dev != w->dev) return IQ_ERR_ARG;
    cudaStream_t s = pick(stream);
    const size_t Rpad = (size_t)(rows + TC_BR - 1) / TC_BR * TC_BR;
    // one byte scratch: the digit matrix, then (16-byte aligned) the split-K partials
    const size_t dbytes = (Rpad * 8 * (size_t)w->P.Kpad + 255) / 256 * 256;
    const size_t pbytes = gemm_tc_part_bytes(w->P, rows);
    uint8_t *dg = nullptr;
    if ((rc = stream_bytes(s, dbytes + pbytes, &dg))) return rc;
    return launch_gemm_tc(d_out, w->P, d_X, rows, s, 0, dg, pbytes ? (int64_t *)(dg + dbytes) : nullptr);
}

IQ_API int iq_device_status(void) {
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    IQ_CUDA(cudaDeviceSynchronize());
    return take_dev_error();
}

IQ_API int iq_bench_i8_peak(int iters, double *tops, float *ms) {
    if (iters < 4 || iters > (1 << 24) || !tops || !ms) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    const int smem = 49152 + 1024 + 64;
    IQ_CUDA(cudaFuncSetAttribute(k_i8_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int *d = nullptr, h = 0;
    IQ_CUDA(cudaMalloc(&d, sizeof(int)));
    cudaStream_t s = lib_stream();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const int grid = dev_info().sms;
    cudaMemsetAsync(d, 0, sizeof(int), s);
    k_i8_peak<<<grid, 128, smem, s>>>(iters / 4, d);   // warm-up
    cudaEventRecord(e0, s);
    k_i8_peak<<<grid, 128, smem, s>>>(iters, d);
    cudaEventRecord(e1, s);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, d, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    float t = 0;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e);
    if (h != 2 * grid) return take_dev_error() ? IQ_ERR_TIMEOUT : IQ_ERR_STATE;
    *ms = t;
    *tops = 2.0 * 128 * 256 * 32 * 4.0 * iters * grid / (t * 1e-3) / 1e12;
    return IQ_OK;
}

IQ_API int iq_wait_selftest(int64_t limit_ns) {
    if (limit_ns < 0 || limit_ns > 100000000) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    int *d = nullptr, h = -1;
    IQ_CUDA(cudaMalloc(&d, sizeof(int)));
    k_wait_selftest<<<1, 32, 0, lib_stream()>>>((uint64_t)limit_ns, d);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, d, sizeof(int), cudaMemcpyDeviceToHost, lib_stream());
    if (e == cudaSuccess) e = cudaStreamSynchronize(lib_stream());
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e);
    return h == 0 ? IQ_OK : IQ_ERR_STATE;  // the wait must have given up
}

}  // extern "C"
