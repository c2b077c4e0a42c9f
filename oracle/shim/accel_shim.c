/*
 * TEST INFRASTRUCTURE ONLY. Linux implementations of the two Accelerate
 * entry points the reference's kernel.c uses, for oracle/_ref.
 *
 * BNNSMatMul (gemm_bf16, c/src/kernel.c:190-228): C[M,N] = A[M,K] . W[N,K]^T
 * with A fp32 and W bf16. Apple's arithmetic is closed; this shim defines it
 * as the project's canonical router dot (oracle_router_dot in moe_oracle.c:
 * exact products, fp64 sums in a fixed order, one rounding to fp32).
 *
 * cblas_sgemm (gemm_fp32, kernel.c:181-186): forwarded to the OpenBLAS that
 * ships inside numpy (ILP64 symbol scipy_cblas_sgemm64_) when it can be
 * found with dlopen, else a plain fp32 loop. QMOE_OPENBLAS names the library
 * file explicitly.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include <Accelerate/Accelerate.h>

#include <dlfcn.h>
#include <glob.h>
#include <stdlib.h>
#include <string.h>

#include "../oracle.h"

size_t BNNSMatMulWorkspaceSize(bool transA, bool transB, float alpha,
                               const BNNSNDArrayDescriptor *A,
                               const BNNSNDArrayDescriptor *B,
                               const BNNSNDArrayDescriptor *C,
                               const void *params) {
    (void)transA; (void)transB; (void)alpha; (void)A; (void)B; (void)C; (void)params;
    return 0;
}

int BNNSMatMul(bool transA, bool transB, float alpha,
               const BNNSNDArrayDescriptor *A, const BNNSNDArrayDescriptor *B,
               const BNNSNDArrayDescriptor *C, void *workspace,
               const void *params) {
    (void)workspace; (void)params;
    /* the only form kernel.c uses: A [M,K] fp32, B [N,K] bf16, transB */
    if (transA || !transB || alpha != 1.0f) return -1;
    if (A->data_type != BNNSDataTypeFloat32 || B->data_type != BNNSDataTypeBFloat16 ||
        C->data_type != BNNSDataTypeFloat32)
        return -1;
    size_t K = A->size[0], M = A->size[1], N = B->size[1];
    if (B->size[0] != K || C->size[0] != N || C->size[1] != M) return -1;
    const float *a = (const float *)A->data;
    const uint16_t *w = (const uint16_t *)B->data;
    float *c = (float *)C->data;
    for (size_t m = 0; m < M; m++)
        for (size_t n = 0; n < N; n++)
            c[m * C->stride[1] + n] =
                oracle_router_dot(a + m * A->stride[1], w + n * B->stride[1], (int)K);
    return 0;
}

typedef void (*sgemm64_fn)(int, int, int, int64_t, int64_t, int64_t, float,
                           const float *, int64_t, const float *, int64_t,
                           float, float *, int64_t);
typedef void (*setthreads_fn)(int);

static sgemm64_fn g_sgemm;
static setthreads_fn g_setthreads;
static int g_probed;

static void probe_openblas(void) {
    if (g_probed) return;
    g_probed = 1;
    const char *env = getenv("QMOE_OPENBLAS");
    void *h = NULL;
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        /* numpy's bundled OpenBLAS beside the running interpreter */
        const char *pats[] = {
            "/opt/prime-rl/.venv/lib/python3*/site-packages/numpy.libs/libscipy_openblas64_*.so",
            "/usr/lib/python3/dist-packages/numpy.libs/libscipy_openblas64_*.so",
        };
        for (size_t i = 0; i < sizeof(pats) / sizeof(pats[0]) && !h; i++) {
            glob_t gl;
            if (glob(pats[i], 0, NULL, &gl) == 0 && gl.gl_pathc > 0)
                h = dlopen(gl.gl_pathv[0], RTLD_NOW | RTLD_LOCAL);
            globfree(&gl);
        }
    }
    if (!h) return;
    g_sgemm = (sgemm64_fn)dlsym(h, "scipy_cblas_sgemm64_");
    g_setthreads = (setthreads_fn)dlsym(h, "scipy_openblas_set_num_threads64_");
}

void ref_set_threads(int threads) {
    probe_openblas();
    if (g_setthreads && threads > 0) g_setthreads(threads);
}

int ref_blas_available(void) {
    probe_openblas();
    return g_sgemm != NULL;
}

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float *A, int lda, const float *B, int ldb, float beta,
                 float *C, int ldc) {
    probe_openblas();
    if (g_sgemm) {
        g_sgemm((int)order, (int)ta, (int)tb, M, N, K, alpha, A, lda, B, ldb,
                beta, C, ldc);
        return;
    }
    /* fallback: the row-major NoTrans x Trans form kernel.c uses */
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            float acc = 0;
            for (int k = 0; k < K; k++) {
                float a = ta == CblasNoTrans ? A[(size_t)m * lda + k] : A[(size_t)k * lda + m];
                float b = tb == CblasTrans ? B[(size_t)n * ldb + k] : B[(size_t)k * ldb + n];
                acc += a * b;
            }
            C[(size_t)m * ldc + n] = alpha * acc + (beta != 0.0f ? beta * C[(size_t)m * ldc + n] : 0.0f);
        }
}
