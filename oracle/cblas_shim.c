/*
 * Plain-C cblas_sgemv / cblas_sdot / openblas_set_num_threads, used to link
 * the reference engine only when no OpenBLAS library is found.  Results then
 * follow this file's summation order, not OpenBLAS's; the build labels such a
 * baseline "reference + naive BLAS shim".  Test infrastructure only.
 */
#include "cblas/cblas.h"

void openblas_set_num_threads(int n) { (void)n; }

void cblas_sgemv(const CBLAS_ORDER order, const CBLAS_TRANSPOSE trans, const int m, const int n,
                 const float alpha, const float *a, const int lda, const float *x, const int incx,
                 const float beta, float *y, const int incy) {
    (void)order; /* main.c only passes CblasRowMajor */
    if (trans == CblasNoTrans) {
        for (int i = 0; i < m; i++) {
            float s = 0.0f;
            for (int j = 0; j < n; j++) s += a[(long)i * lda + j] * x[(long)j * incx];
            y[(long)i * incy] = alpha * s + (beta != 0.0f ? beta * y[(long)i * incy] : 0.0f);
        }
    } else {
        for (int j = 0; j < n; j++) y[(long)j * incy] = (beta != 0.0f ? beta * y[(long)j * incy] : 0.0f);
        for (int i = 0; i < m; i++) {
            const float xi = alpha * x[(long)i * incx];
            for (int j = 0; j < n; j++) y[(long)j * incy] += a[(long)i * lda + j] * xi;
        }
    }
}

float cblas_sdot(const int n, const float *x, const int incx, const float *y, const int incy) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[(long)i * incx] * y[(long)i * incy];
    return s;
}
