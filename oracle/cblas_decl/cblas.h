/* Minimal CBLAS declarations so the reference's cpu/jl_transform.cpp compiles
 * against the OpenBLAS shared library shipped in this image (no BLAS headers
 * are installed). Only the one routine that file calls is declared.
 * Test infrastructure: used by oracle/Makefile for oracle/_ref only. */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float* a, int lda,
                 const float* b, int ldb, float beta, float* c, int ldc);
#ifdef __cplusplus
}
#endif
