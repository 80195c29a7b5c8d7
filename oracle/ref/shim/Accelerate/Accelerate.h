/*
 * Stand-in for macOS Accelerate, test infrastructure only: the reference CPU
 * path (cpu_reference.hpp:437-458,515-551) calls cblas_sgemm for its batched
 * MLPs. This provides the row-major subset it uses. Each output element is an
 * in-order sum over k (then alpha*acc + beta*C), parallel over output rows with
 * OpenMP. Accelerate's summation order is not specified, so MLP outputs of the
 * reference are compared with tolerances, never bitwise.
 */
#pragma once
#include <cstddef>
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

inline void cblas_sgemm(const CBLAS_ORDER order, const CBLAS_TRANSPOSE ta, const CBLAS_TRANSPOSE tb,
                        const int M, const int N, const int K, const float alpha,
                        const float* A, const int lda, const float* B, const int ldb,
                        const float beta, float* C, const int ldc) {
    (void)order; /* callers only use CblasRowMajor */
    const bool at = ta != CblasNoTrans, bt = tb != CblasNoTrans;
#pragma omp parallel for schedule(static) if (size_t(M) * size_t(N) * size_t(K) > (1u << 16))
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) {
                const float a = at ? A[size_t(k) * lda + m] : A[size_t(m) * lda + k];
                const float b = bt ? B[size_t(n) * ldb + k] : B[size_t(k) * ldb + n];
                acc += a * b;
            }
            float* c = C + size_t(m) * ldc + n;
            *c = beta == 0.0f ? alpha * acc : alpha * acc + beta * *c;
        }
    }
}
