/*
 * cblas.h - minimal CBLAS prototypes for building the gemma3.c reference as a
 * test oracle.  TEST INFRASTRUCTURE ONLY: nothing in the shipped library
 * includes this file.
 *
 * The reference includes <cblas.h> under USE_BLAS (gemma3_kernels.h:14-16) and
 * calls exactly four routines: cblas_sdot / cblas_saxpy (gemma3_kernels.c:562,587),
 * cblas_sgemv (gemma3_kernels.c:48) and cblas_sgemm (gemma3_kernels.c:28,
 * gemma3_transformer.c:624-751).  No system cblas.h is installed in this image,
 * so the standard CBLAS enum values and these four signatures are declared
 * here; the symbols resolve against the OpenBLAS 0.3.15 shared library that
 * ships inside the Python environment.
 */
#ifndef ORACLE_MIN_CBLAS_H
#define ORACLE_MIN_CBLAS_H
#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

float cblas_sdot(const int n, const float *x, const int incx,
                 const float *y, const int incy);
void cblas_saxpy(const int n, const float alpha, const float *x, const int incx,
                 float *y, const int incy);
void cblas_sgemv(const enum CBLAS_ORDER order, const enum CBLAS_TRANSPOSE trans,
                 const int m, const int n, const float alpha, const float *a,
                 const int lda, const float *x, const int incx, const float beta,
                 float *y, const int incy);
void cblas_sgemm(const enum CBLAS_ORDER order, const enum CBLAS_TRANSPOSE ta,
                 const enum CBLAS_TRANSPOSE tb, const int m, const int n,
                 const int k, const float alpha, const float *a, const int lda,
                 const float *b, const int ldb, const float beta, float *c,
                 const int ldc);

#ifdef __cplusplus
}
#endif
#endif
