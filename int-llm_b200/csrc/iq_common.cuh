// iq_common.cuh -- shared definitions for the sm_100a Q16.48 library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/iq.h"

#define IQ_Q 48
#define IQ_ONE ((int64_t)1 << IQ_Q)

typedef __int128 i128;
typedef unsigned __int128 u128;

namespace iq {

// Records the CUDA error and maps it to an iq_status.
int cuda_fail(cudaError_t e);

#define IQ_CUDA(call)                                   \
    do {                                                \
        cudaError_t _e = (call);                        \
        if (_e != cudaSuccess) return ::iq::cuda_fail(_e); \
    } while (0)

#define IQ_CHECK_LAUNCH() IQ_CUDA(cudaGetLastError())

struct DevInfo {
    int sms = 0;
    int smem_optin = 0;
    int cc_major = 0, cc_minor = 0;
};
const DevInfo &dev_info();  // for the current device
cudaStream_t lib_stream();  // the library's own stream on the current device
inline cudaStream_t pick(void *s) { return s ? (cudaStream_t)s : lib_stream(); }

}  // namespace iq
