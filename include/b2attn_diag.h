/*
 * b2attn diagnostics — not part of the attention ABI, no counterpart in the
 * reference. Used by the GPU tests to check the tensor-core operand layouts
 * in isolation.
 */
#ifndef B2ATTN_DIAG_H
#define B2ATTN_DIAG_H

#include "b2attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * One 128x128x128 bf16 tcgen05 MMA (single CTA) with fp32 output c [128][128].
 * a: [128][128] bf16 row-major (M x K).
 * b_mn_major = 0: b is [N][K] row-major and c = a * b^T.
 * b_mn_major = 1: b is [K][N] row-major and c = a * b.
 * b_mn_major = 2: as 1, with a read by the MMA from tensor memory.
 * Returns 0 or a negative B2A_ERR_* code.
 */
B2A_API int b2a_diag_umma_gemm(const void* a, const void* b, float* c, int b_mn_major, void* stream);

/*
 * Launch one CTA that waits on an mbarrier nothing arrives on, with the same
 * bounded wait the kernels use but a limit of `limit_cycles` (1 .. 4e9). The
 * wait runs out, sets the abort path and the device error word, and the
 * kernel exits; b2a_get_device_error then reports B2A_ERR_DEVICE_TIMEOUT.
 * Used by the GPU tests to check failure reporting without a GPU fault.
 */
B2A_API int b2a_diag_wait_timeout(long long limit_cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2ATTN_DIAG_H */
