// Entry points for the library's own tests.  Exported from libtikun_cuda.so
// but not part of the public ABI (include/tikun_cuda.h).
#pragma once

#include <stdint.h>

#include "../../include/tikun_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* D[b] = alpha * P[b] * Q[b]^T for half-precision row-major P (M x K), Q
 * (N x K), D (M x N); fmt 0 = f16, 1 = bf16.  Synchronous. */
TK_API int tk_testing_gemm_tn(const void* P, const void* Q, void* D, int batch, int M, int N,
                              int K, int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt,
                              void* stream);

/* Launches a kernel whose mbarrier wait can never complete; the bounded wait
 * gives up after limit_ms (1..2000), the kernel returns and the call reports
 * TK_ERR_DEVICE.  Exercises the failure path without faulting the GPU. */
TK_API int tk_testing_bounded_wait(int limit_ms, void* stream);

/* Device memory the library holds on the current device through its own
 * allocations: the scratch pool's reserved bytes plus the status word (0 when
 * neither was ever created).  Creates nothing. */
TK_API int tk_testing_library_device_bytes(uint64_t* bytes_out);

#ifdef __cplusplus
}
#endif
