/* Test infrastructure only.  The reference's CMake build links a vendored
 * scipy-openblas32; that wheel is absent here, and its only user (DPA4) is off
 * the SOAP path.  This header declares the two prefixed symbols the reference
 * includes through cpp/include/mdescriptor/detail/blas.hpp:6,25,38 so that the
 * reference `_native` module links for the golden-fixture generator.  The
 * prefixed LAPACKE SVD that ACE declares itself gets a failing stand-in in
 * cblas_shim.cpp. */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void scipy_openblas_set_num_threads(int threads);
void scipy_cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE trans_a,
                       enum CBLAS_TRANSPOSE trans_b, int m, int n, int k, float alpha,
                       const float* a, int lda, const float* b, int ldb, float beta, float* c,
                       int ldc);
#ifdef __cplusplus
}
#endif
