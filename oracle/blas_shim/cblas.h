/* Minimal cblas.h for building the reference with -DUSE_BLAS against the OpenBLAS
 * that numpy bundles (ILP64, symbols prefixed scipy_ and suffixed 64_).  Only the two
 * routines the reference calls are declared.  TEST INFRASTRUCTURE ONLY. */
#ifndef JD_CBLAS_SHIM_H
#define JD_CBLAS_SHIM_H
#include <stdint.h>
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void scipy_cblas_sgemv64_(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, int64_t, int64_t, float, const float *, int64_t,
                          const float *, int64_t, float, float *, int64_t);
void scipy_cblas_sgemm64_(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE, int64_t, int64_t, int64_t, float,
                          const float *, int64_t, const float *, int64_t, float, float *, int64_t);
#define cblas_sgemv scipy_cblas_sgemv64_
#define cblas_sgemm scipy_cblas_sgemm64_
#endif
