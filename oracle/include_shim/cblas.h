/* Minimal CBLAS declarations (the standard public CBLAS API) so that the reference's
 * src/core/blas.cpp compiles against the OpenBLAS shared library shipped in this image.
 * Test infrastructure only: used by oracle/Makefile when it builds oracle/_ref. */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
typedef enum CBLAS_ORDER CBLAS_LAYOUT;
void cblas_sgemm(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE, int, int, int,
                 float, const float*, int, const float*, int, float, float*, int);
void openblas_set_num_threads(int);
char* openblas_get_corename(void);
#ifdef __cplusplus
}
#endif
