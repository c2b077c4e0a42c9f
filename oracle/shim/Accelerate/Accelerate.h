/*
 * TEST INFRASTRUCTURE ONLY. Stand-in for Apple's <Accelerate/Accelerate.h>,
 * declaring just the entry points the reference's c/src/kernel.c calls
 * (cblas_sgemm at kernel.c:181-186; BNNSMatMul and BNNSMatMulWorkspaceSize at
 * kernel.c:190-228) so that the reference compiles unmodified on Linux for
 * oracle/_ref. Implemented in oracle/shim/accel_shim.c.
 */
#ifndef QMOE_ACCEL_SHIM_H
#define QMOE_ACCEL_SHIM_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float *A, int lda, const float *B, int ldb, float beta,
                 float *C, int ldc);

typedef enum {
    BNNSDataLayoutRowMajorMatrix = 0x10000,
} BNNSDataLayout;

typedef enum {
    BNNSDataTypeFloat32 = 0x10020,
    BNNSDataTypeBFloat16 = 0x10010,
} BNNSDataType;

typedef struct {
    BNNSDataLayout layout;
    size_t size[8];
    size_t stride[8];
    void *data;
    BNNSDataType data_type;
} BNNSNDArrayDescriptor;

size_t BNNSMatMulWorkspaceSize(bool transA, bool transB, float alpha,
                               const BNNSNDArrayDescriptor *A,
                               const BNNSNDArrayDescriptor *B,
                               const BNNSNDArrayDescriptor *C,
                               const void *params);

int BNNSMatMul(bool transA, bool transB, float alpha,
               const BNNSNDArrayDescriptor *A, const BNNSNDArrayDescriptor *B,
               const BNNSNDArrayDescriptor *C, void *workspace,
               const void *params);

#endif
