/*
 * cblas.h — minimal CBLAS shim used only to build the reference C sources
 * into the test oracle (oracle/_ref).  It declares the one routine the
 * reference calls, cblas_sgemm, and forwards it to the ILP64 OpenBLAS
 * build that numpy ships (symbol scipy_cblas_sgemm64_), because no
 * OpenBLAS development package is installed on these machines.
 *
 * TEST INFRASTRUCTURE ONLY.
 */
#ifndef ORACLE_CBLAS_SHIM_H
#define ORACLE_CBLAS_SHIM_H
#include <stdint.h>

enum CBLAS_ORDER     { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void scipy_cblas_sgemm64_(int order, int transa, int transb,
                          int64_t m, int64_t n, int64_t k, float alpha,
                          const float *a, int64_t lda, const float *b,
                          int64_t ldb, float beta, float *c, int64_t ldc);

static inline void cblas_sgemm(enum CBLAS_ORDER order,
                               enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                               int m, int n, int k, float alpha,
                               const float *a, int lda, const float *b, int ldb,
                               float beta, float *c, int ldc) {
    scipy_cblas_sgemm64_((int)order, (int)ta, (int)tb, m, n, k, alpha,
                         a, lda, b, ldb, beta, c, ldc);
}
#endif
