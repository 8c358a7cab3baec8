/* Minimal CBLAS declarations (the standard C interface to the BLAS, as
 * published by netlib) for compiling the reference's CPU path against the
 * OpenBLAS shared library present in this image, which ships no headers.
 * Test infrastructure only. */
#ifndef ORACLE_SHIM_CBLAS_H
#define ORACLE_SHIM_CBLAS_H
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
typedef enum CBLAS_ORDER CBLAS_ORDER;
typedef enum CBLAS_TRANSPOSE CBLAS_TRANSPOSE;
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE transa, enum CBLAS_TRANSPOSE transb,
                 int m, int n, int k, float alpha, const float *a, int lda, const float *b,
                 int ldb, float beta, float *c, int ldc);
#ifdef __cplusplus
}
#endif
#endif
