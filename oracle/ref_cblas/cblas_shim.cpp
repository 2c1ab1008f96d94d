// Test infrastructure only: plain row-major sgemm behind the prefixed names
// declared in cblas.h (no-transpose only, which is all DPA4 asks for).
#include "cblas.h"

extern "C" void scipy_openblas_set_num_threads(int) {}

extern "C" void scipy_cblas_sgemm(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE,
                                  int m, int n, int k, float alpha, const float* a, int lda,
                                  const float* b, int ldb, float beta, float* c, int ldc) {
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float sum = 0.0F;
            for (int p = 0; p < k; ++p) sum += a[i * lda + p] * b[p * ldb + j];
            c[i * ldc + j] = alpha * sum + (beta == 0.0F ? 0.0F : beta * c[i * ldc + j]);
        }
    }
}

// ACE (cpp/src/standalone/ace.cpp:28) declares a prefixed LAPACKE SVD.  ACE is
// off the SOAP path; the stand-in reports failure so ACE raises its own
// "ACE LAPACK SVD failed" error instead of returning wrong numbers.
extern "C" int scipy_LAPACKE_dgesdd(int, char, int, int, double*, int, double*, double*, int,
                                    double*, int) {
    return -1;
}
