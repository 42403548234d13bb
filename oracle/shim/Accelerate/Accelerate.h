/*
 * Test infrastructure (oracle only; never linked into the product library).
 *
 * Minimal stand-in for Apple's <Accelerate/Accelerate.h>, just large enough to
 * compile the reference's core/cpu_ops.cpp unmodified on Linux.  It provides the
 * 13 vDSP / vForce / CBLAS routines that file calls, written as plain loops
 * following Apple's and the CBLAS documented argument order:
 *
 *   vDSP_vneg   C = -A
 *   vvexpf      y = exp(x)
 *   vDSP_vsadd  C = A + *B           (scalar B)
 *   vDSP_vdiv   C = A / B            (note: divisor B is the FIRST argument)
 *   vDSP_svesq  *C = sum(A^2)
 *   vDSP_vsmul  C = A * *B           (scalar B)
 *   vDSP_vmul   C = A * B
 *   vDSP_vsub   C = A - B            (note: subtrahend B is the FIRST argument)
 *   vDSP_dotpr  *C = sum(A * B)
 *   cblas_sgemv y = alpha*op(A)*x + beta*y   (beta == 0 => y not read)
 *   cblas_sscal x = alpha*x
 *   cblas_sger  A = A + alpha*x*y^T
 *   cblas_saxpy y = alpha*x + y
 *
 * Reductions run in ascending index order; oracle/anelm_oracle.c restates the
 * same loops so the two agree bit for bit when both are built with
 * -ffp-contract=off.
 */
#ifndef ANELM_ORACLE_ACCELERATE_SHIM_H
#define ANELM_ORACLE_ACCELERATE_SHIM_H

#include <math.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

static inline void vDSP_vneg(const float* A, vDSP_Stride IA, float* C, vDSP_Stride IC, vDSP_Length N) {
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = -A[n * IA];
}

static inline void vvexpf(float* y, const float* x, const int* n) {
    for (int i = 0; i < *n; i++) y[i] = expf(x[i]);
}

static inline void vDSP_vsadd(const float* A, vDSP_Stride IA, const float* B, float* C,
                              vDSP_Stride IC, vDSP_Length N) {
    const float b = *B;
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = A[n * IA] + b;
}

static inline void vDSP_vdiv(const float* B, vDSP_Stride IB, const float* A, vDSP_Stride IA,
                             float* C, vDSP_Stride IC, vDSP_Length N) {
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = A[n * IA] / B[n * IB];
}

static inline void vDSP_svesq(const float* A, vDSP_Stride IA, float* C, vDSP_Length N) {
    float s = 0.0f;
    for (vDSP_Length n = 0; n < N; n++) s += A[n * IA] * A[n * IA];
    *C = s;
}

static inline void vDSP_vsmul(const float* A, vDSP_Stride IA, const float* B, float* C,
                              vDSP_Stride IC, vDSP_Length N) {
    const float b = *B;
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = A[n * IA] * b;
}

static inline void vDSP_vmul(const float* A, vDSP_Stride IA, const float* B, vDSP_Stride IB,
                             float* C, vDSP_Stride IC, vDSP_Length N) {
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = A[n * IA] * B[n * IB];
}

static inline void vDSP_vsub(const float* B, vDSP_Stride IB, const float* A, vDSP_Stride IA,
                             float* C, vDSP_Stride IC, vDSP_Length N) {
    for (vDSP_Length n = 0; n < N; n++) C[n * IC] = A[n * IA] - B[n * IB];
}

static inline void vDSP_dotpr(const float* A, vDSP_Stride IA, const float* B, vDSP_Stride IB,
                              float* C, vDSP_Length N) {
    float s = 0.0f;
    for (vDSP_Length n = 0; n < N; n++) s += A[n * IA] * B[n * IB];
    *C = s;
}

/* Row-major only (the reference never passes CblasColMajor). */
static inline void cblas_sgemv(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE trans, int M, int N,
                               float alpha, const float* A, int lda, const float* X, int incX,
                               float beta, float* Y, int incY) {
    (void)order;
    if (trans == CblasNoTrans) {
        for (int i = 0; i < M; i++) {
            float s = 0.0f;
            for (int j = 0; j < N; j++) s += A[(size_t)i * lda + j] * X[j * incX];
            Y[i * incY] = (beta == 0.0f) ? alpha * s : alpha * s + beta * Y[i * incY];
        }
    } else {
        for (int j = 0; j < N; j++) {
            float s = 0.0f;
            for (int i = 0; i < M; i++) s += A[(size_t)i * lda + j] * X[i * incX];
            Y[j * incY] = (beta == 0.0f) ? alpha * s : alpha * s + beta * Y[j * incY];
        }
    }
}

static inline void cblas_sscal(int N, float alpha, float* X, int incX) {
    for (int n = 0; n < N; n++) X[(size_t)n * incX] *= alpha;
}

static inline void cblas_sger(enum CBLAS_ORDER order, int M, int N, float alpha, const float* X,
                              int incX, const float* Y, int incY, float* A, int lda) {
    (void)order;
    for (int i = 0; i < M; i++) {
        const float ax = alpha * X[i * incX];
        for (int j = 0; j < N; j++) A[(size_t)i * lda + j] += ax * Y[j * incY];
    }
}

static inline void cblas_saxpy(int N, float alpha, const float* X, int incX, float* Y, int incY) {
    for (int n = 0; n < N; n++) Y[(size_t)n * incY] += alpha * X[(size_t)n * incX];
}

#ifdef __cplusplus
}
#endif

#endif /* ANELM_ORACLE_ACCELERATE_SHIM_H */
