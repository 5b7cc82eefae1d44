/* The part of the standard CBLAS interface that the reference's BLAS
 * backend calls (cblas_sgemm with row-major storage). The image has
 * OpenBLAS as a shared library without its header, so oracle/Makefile
 * compiles against this declaration and links that library. */
#ifndef AZ_CBLAS_SHIM_H
#define AZ_CBLAS_SHIM_H
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
typedef int blasint;
void cblas_sgemm(const enum CBLAS_ORDER order, const enum CBLAS_TRANSPOSE transA,
                 const enum CBLAS_TRANSPOSE transB, const blasint M, const blasint N, const blasint K,
                 const float alpha, const float* A, const blasint lda, const float* B, const blasint ldb,
                 const float beta, float* C, const blasint ldc);
#ifdef __cplusplus
}
#endif
#endif
