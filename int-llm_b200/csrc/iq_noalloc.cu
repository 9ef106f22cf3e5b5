// iq_noalloc.cu -- a matvec entry point that allocates no memory.
//
// Who needs it: callers that may not allocate GPU memory at the moment they
// call us -- e.g. code running under an external memory budget or custom
// allocator that forbids cudaMalloc outside its own pool, real-time loops where
// an allocation's implicit synchronisation is unacceptable, or a host process
// that has handed all free device memory to another component. The regular
// iq_matvec_packed_dev grows a per-stream scratch buffer with cudaMalloc on
// first use; this variant uses a fixed array that lives in the library image.
//
// The split-row scratch (one 32-byte RowAcc per output row) is the file-scope
// device array g_noalloc_rows below: IQ_NOALLOC_MAX_ROWS entries (1 MiB),
// held by every GPU that loads the library until the process exits. In host
// code its name is only a host-side stand-in, so the kernel gets the real
// device address, fetched once per device by cudaGetSymbolAddress.
#include <mutex>
#include "iq_common.cuh"
#include "iq_planes.cuh"

#define IQ_NOALLOC_MAX_ROWS 32768

namespace iq {

static __device__ __align__(256) RowAcc g_noalloc_rows[IQ_NOALLOC_MAX_ROWS];

int launch_matvec_planes(int64_t *out, const Packed &P, const int64_t *x, cudaStream_t s, int add, RowAcc *racc,
                         const int64_t *nrm_w);
int ensure_device_pub(int dev);

static std::mutex g_noalloc_mu;
static RowAcc *g_noalloc_ptr[64];

// Per-device set-up, run by the first call on each device (with that device
// current): look up the array's device address and clear it. Both steps are
// plain runtime calls that allocate nothing.
static int noalloc_setup(int dev, RowAcc **out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        RowAcc *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void **)&p, g_noalloc_rows);
        if (e != cudaSuccess) return cuda_fail(e);
        e = cudaMemset(p, 0, sizeof(g_noalloc_rows));
        if (e != cudaSuccess) return cuda_fail(e);
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e);
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return IQ_OK;
}

}  // namespace iq

using namespace iq;

struct iq_packed;  // defined in iq_api.cu
const Packed *iq_packed_inner(const iq_packed *w, int *dev);

extern "C" IQ_API int iq_matvec_packed_noalloc_dev(int64_t *d_out, const iq_packed *w, const int64_t *d_in,
                                                    void *stream) {
    if (!d_out || !w || !d_in || d_out == d_in) return IQ_ERR_ARG;
    int wdev = -1;
    const Packed *P = iq_packed_inner(w, &wdev);
    int dev = 0;
    IQ_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || dev != wdev) return IQ_ERR_ARG;  // checked first, as iq_matvec_packed_dev does
    if (P->Mp > IQ_NOALLOC_MAX_ROWS) return IQ_ERR_RANGE;  // more rows than the fixed scratch holds
    int rc = ensure_device_pub(dev);  // device properties + library stream; no memory allocation
    if (rc) return rc;
    RowAcc *rows = nullptr;
    rc = noalloc_setup(dev, &rows);
    if (rc) return rc;
    // The kernel leaves every entry it touched at zero again when it completes,
    // so the shared array is ready for the next call.
    return launch_matvec_planes(d_out, *P, d_in, stream ? (cudaStream_t)stream : lib_stream(), 0, rows);
}
