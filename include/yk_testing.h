/*
 * yk_testing.h -- test hooks of libyk.so.  Not part of the reference-facing
 * boundary (no reference counterpart): they run one internal kernel in
 * isolation so GPU tests can localise a failure.
 */
#pragma once
#include <stdint.h>

#include "yk.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Y[m_tok x n_out] (fp32, host) = X[m_tok x K] * W[n_out x K]^T through the
 * tcgen05 GEMM; W and X are host bf16 bit patterns.  splits > 0 forces the
 * split-K factor (0 = the heuristic). */
yk_status ykt_gemm_bf16(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K, int32_t m_tok,
                        int32_t splits, float* Y);

#ifdef __cplusplus
}
#endif
