// Test-infrastructure shim: lets the reference CPU sources (which include Apple's
// <Accelerate/Accelerate.h> for cblas_sgemm / cblas_sgemv) compile on Linux.
//
// Call sites in the reference: src/model/ops.cpp:15,119,138,156,158,167,169 and
// src/infer/inference.cpp:38,107,111,122,125,128,131,146,150. Only row-major
// single-precision GEMM/GEMV are used.
//
// Two backends, chosen at build time:
//   * default: OpenBLAS 0.3.30 as bundled with numpy (ILP64, symbols prefixed
//     "scipy_" and suffixed "64_"), linked by oracle/Makefile;
//   * -DMINI_MLA_PORTABLE_BLAS: a plain blocked loop nest (no external library).
// This is the checker's arithmetic, never the product's.
#pragma once
#include <cstdint>

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

#ifndef MINI_MLA_PORTABLE_BLAS
extern "C" {
void scipy_cblas_sgemm64_(int order, int ta, int tb, std::int64_t m, std::int64_t n,
                          std::int64_t k, float alpha, const float* a, std::int64_t lda,
                          const float* b, std::int64_t ldb, float beta, float* c,
                          std::int64_t ldc);
void scipy_cblas_sgemv64_(int order, int ta, std::int64_t m, std::int64_t n, float alpha,
                          const float* a, std::int64_t lda, const float* x, std::int64_t incx,
                          float beta, float* y, std::int64_t incy);
}
inline void cblas_sgemm(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n,
                        int k, float alpha, const float* a, int lda, const float* b, int ldb,
                        float beta, float* c, int ldc) {
    scipy_cblas_sgemm64_(order, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}
inline void cblas_sgemv(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, int m, int n, float alpha,
                        const float* a, int lda, const float* x, int incx, float beta, float* y,
                        int incy) {
    scipy_cblas_sgemv64_(order, ta, m, n, alpha, a, lda, x, incx, beta, y, incy);
}
#else
// Row-major only (the reference never asks for column-major).
inline void cblas_sgemm(CBLAS_ORDER, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n, int k,
                        float alpha, const float* a, int lda, const float* b, int ldb, float beta,
                        float* c, int ldc) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float s = 0;
            for (int p = 0; p < k; ++p) {
                float av = ta == CblasNoTrans ? a[(long)i * lda + p] : a[(long)p * lda + i];
                float bv = tb == CblasNoTrans ? b[(long)p * ldb + j] : b[(long)j * ldb + p];
                s += av * bv;
            }
            float& out = c[(long)i * ldc + j];
            out = alpha * s + (beta == 0 ? 0.0F : beta * out);
        }
}
inline void cblas_sgemv(CBLAS_ORDER, CBLAS_TRANSPOSE ta, int m, int n, float alpha, const float* a,
                        int lda, const float* x, int incx, float beta, float* y, int incy) {
    int rows = ta == CblasNoTrans ? m : n, cols = ta == CblasNoTrans ? n : m;
    for (int i = 0; i < rows; ++i) {
        float s = 0;
        for (int j = 0; j < cols; ++j) {
            float av = ta == CblasNoTrans ? a[(long)i * lda + j] : a[(long)j * lda + i];
            s += av * x[(long)j * incx];
        }
        float& out = y[(long)i * incy];
        out = alpha * s + (beta == 0 ? 0.0F : beta * out);
    }
}
#endif
