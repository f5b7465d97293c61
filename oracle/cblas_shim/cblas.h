/* Minimal stand-in for the two OpenBLAS entry points that the reference's
 * gqa_attention.c (src/mojollama/kernels/gqa_attention.c:19,107,113,129) uses.
 * OpenBLAS is not installed in this image, so the oracle build links this
 * header and cblas_shim.c instead.  Test infrastructure only: nothing in the
 * product links it.  Plain row-major / column-major SGEMM with the standard
 * CBLAS argument meaning; no blocking, no threading. */
#ifndef MLQ_ORACLE_CBLAS_SHIM_H
#define MLQ_ORACLE_CBLAS_SHIM_H

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float *a, int lda,
                 const float *b, int ldb, float beta, float *c, int ldc);
void openblas_set_num_threads(int n);

#endif
