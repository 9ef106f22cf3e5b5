/*
 * iq_matvec_shim.h -- the source-level drop-in of libiq.so into int-llm's
 * llama_int.c. Force-include it (`-include iq_matvec_shim.h`) into a copy of
 * llama_int.c whose definition of `static void matmul_vec(...)` (line 1014)
 * is renamed `matmul_vec_cpu`: every call site (llama_int.c:1387-1389, 1532,
 * 1547-1548, 1553, 2880) then calls iq_matmul_vec with the same arguments.
 * The reference has no error path in matmul_vec (it returns void), so a
 * failing call is reported and ends the process, as the reference does on
 * allocation failure (llama_int.c:460-477).
 */
#ifndef IQ_MATVEC_SHIM_H
#define IQ_MATVEC_SHIM_H
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include "iq.h"

static inline void matmul_vec(int64_t *out, const int64_t *weight, const int64_t *in, int M, int N) {
    int rc = iq_matmul_vec(out, weight, in, M, N);
    if (rc != IQ_OK) {
        fprintf(stderr, "iq_matmul_vec(M=%d, N=%d): %s\n", M, N, iq_status_str(rc));
        exit(1);
    }
}
#endif
