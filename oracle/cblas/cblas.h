/*
 * Prototype-only CBLAS header for building the reference engine
 * (gemma4-4b/cpu-blas/main.c includes <cblas.h>, main.c:29-33) against the
 * OpenBLAS shared library bundled in the Python environment, which ships
 * without headers.  Only what main.c uses is declared: the two enums and
 * cblas_sgemv / cblas_sdot (standard CBLAS values and 32-bit int interface).
 * Test infrastructure only.
 */
#ifndef G4_ORACLE_CBLAS_H
#define G4_ORACLE_CBLAS_H
typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 } CBLAS_TRANSPOSE;
void cblas_sgemv(const CBLAS_ORDER order, const CBLAS_TRANSPOSE trans, const int m, const int n,
                 const float alpha, const float *a, const int lda, const float *x, const int incx,
                 const float beta, float *y, const int incy);
float cblas_sdot(const int n, const float *x, const int incx, const float *y, const int incy);
#endif
