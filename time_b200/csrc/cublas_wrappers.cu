// cublas_wrappers.cu -- libcublaswrap's reference-compatible part: the 17
// cbw* entry points (csrc/cublas_wrappers.h:51-67) as plain cuBLAS/cuBLASLt
// calls.  Status mapping follows csrc/cublas_wrappers.cu:7-18.  The MoE expert
// GEMM lives in moe_gemm.cu (cbwFp8BlockScaledGroupedGemm).
#include <cublas_v2.h>
#include <cublasLt.h>
#include <cuda_fp16.h>
#include <cstdio>

#include "cublas_wrappers.h"

namespace {

cbwStatus_t to_cbw(cublasStatus_t e) {
    switch (e) {
        case CUBLAS_STATUS_SUCCESS: return CBW_SUCCESS;
        case CUBLAS_STATUS_NOT_INITIALIZED: return CBW_ERROR_NOT_INITIALIZED;
        case CUBLAS_STATUS_ALLOC_FAILED: return CBW_ERROR_ALLOC_FAILED;
        case CUBLAS_STATUS_INVALID_VALUE: return CBW_ERROR_INVALID_VALUE;
        case CUBLAS_STATUS_EXECUTION_FAILED: return CBW_ERROR_EXECUTION_FAILED;
        case CUBLAS_STATUS_NOT_SUPPORTED: return CBW_ERROR_NOT_SUPPORTED;
        default: return CBW_ERROR_INTERNAL;
    }
}

cbwStatus_t report(cublasStatus_t e, const char* what) {
    if (e != CUBLAS_STATUS_SUCCESS) std::fprintf(stderr, "%s failed: %d\n", what, static_cast<int>(e));
    return to_cbw(e);
}

cublasOperation_t op(cbwOperation_t o) {
    return o == CBW_OP_T ? CUBLAS_OP_T : (o == CBW_OP_C ? CUBLAS_OP_C : CUBLAS_OP_N);
}

cudaDataType_t dtype(cbwDataType_t t) {
    switch (t) {
        case CBW_R_16F: return CUDA_R_16F;
        case CBW_R_64F: return CUDA_R_64F;
        case CBW_R_16BF: return CUDA_R_16BF;
        case CBW_R_8F_E4M3: return CUDA_R_8F_E4M3;
        case CBW_R_8F_E5M2: return CUDA_R_8F_E5M2;
        default: return CUDA_R_32F;
    }
}

cublasComputeType_t ctype(cbwComputeType_t t) {
    switch (t) {
        case CBW_COMPUTE_16F: return CUBLAS_COMPUTE_16F;
        case CBW_COMPUTE_64F: return CUBLAS_COMPUTE_64F;
        case CBW_COMPUTE_32F_FAST_16F: return CUBLAS_COMPUTE_32F_FAST_16F;
        case CBW_COMPUTE_32F_FAST_TF32: return CUBLAS_COMPUTE_32F_FAST_TF32;
        default: return CUBLAS_COMPUTE_32F;
    }
}

}  // namespace

extern "C" {

cbwStatus_t cbwCreate(cbwHandle_t* handle) {
    cublasHandle_t h = nullptr;
    cublasStatus_t e = cublasCreate(&h);
    *handle = (e == CUBLAS_STATUS_SUCCESS) ? static_cast<cbwHandle_t>(h) : nullptr;
    return report(e, "cublasCreate");
}

cbwStatus_t cbwDestroy(cbwHandle_t handle) {
    if (!handle) return CBW_SUCCESS;
    return to_cbw(cublasDestroy(static_cast<cublasHandle_t>(handle)));
}

cbwStatus_t cbwSetStream(cbwHandle_t handle, cwStream_t stream) {
    return to_cbw(cublasSetStream(static_cast<cublasHandle_t>(handle), static_cast<cudaStream_t>(stream)));
}

cbwStatus_t cbwSgemm(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k,
                     const float* alpha, const float* A, int lda, const float* B, int ldb, const float* beta, float* C,
                     int ldc) {
    return report(cublasSgemm(static_cast<cublasHandle_t>(handle), op(transa), op(transb), m, n, k, alpha, A, lda, B, ldb,
                              beta, C, ldc), "cublasSgemm");
}

cbwStatus_t cbwHgemm(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k,
                     const void* alpha, const void* A, int lda, const void* B, int ldb, const void* beta, void* C, int ldc) {
    return report(cublasHgemm(static_cast<cublasHandle_t>(handle), op(transa), op(transb), m, n, k,
                              static_cast<const __half*>(alpha), static_cast<const __half*>(A), lda,
                              static_cast<const __half*>(B), ldb, static_cast<const __half*>(beta),
                              static_cast<__half*>(C), ldc), "cublasHgemm");
}

cbwStatus_t cbwSgemmBatched(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k,
                            const float* alpha, const float** Aarray, int lda, const float** Barray, int ldb,
                            const float* beta, float** Carray, int ldc, int batchCount) {
    return report(cublasSgemmBatched(static_cast<cublasHandle_t>(handle), op(transa), op(transb), m, n, k, alpha, Aarray,
                                     lda, Barray, ldb, beta, Carray, ldc, batchCount), "cublasSgemmBatched");
}

cbwStatus_t cbwSgemmStridedBatched(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k,
                                   const float* alpha, const float* A, int lda, long long strideA, const float* B, int ldb,
                                   long long strideB, const float* beta, float* C, int ldc, long long strideC,
                                   int batchCount) {
    return report(cublasSgemmStridedBatched(static_cast<cublasHandle_t>(handle), op(transa), op(transb), m, n, k, alpha, A,
                                            lda, strideA, B, ldb, strideB, beta, C, ldc, strideC, batchCount),
                  "cublasSgemmStridedBatched");
}

cbwStatus_t cbwLtCreate(cbwLtHandle_t* handle) {
    cublasLtHandle_t h = nullptr;
    cublasStatus_t e = cublasLtCreate(&h);
    *handle = (e == CUBLAS_STATUS_SUCCESS) ? static_cast<cbwLtHandle_t>(h) : nullptr;
    return report(e, "cublasLtCreate");
}

cbwStatus_t cbwLtDestroy(cbwLtHandle_t handle) {
    if (!handle) return CBW_SUCCESS;
    return to_cbw(cublasLtDestroy(static_cast<cublasLtHandle_t>(handle)));
}

cbwStatus_t cbwLtMatmulDescCreate(cbwLtMatmulDesc_t* desc, cbwComputeType_t computeType, cbwDataType_t scaleType) {
    cublasLtMatmulDesc_t d = nullptr;
    cublasStatus_t e = cublasLtMatmulDescCreate(&d, ctype(computeType), dtype(scaleType));
    *desc = (e == CUBLAS_STATUS_SUCCESS) ? static_cast<cbwLtMatmulDesc_t>(d) : nullptr;
    return to_cbw(e);
}

cbwStatus_t cbwLtMatmulDescDestroy(cbwLtMatmulDesc_t desc) {
    if (!desc) return CBW_SUCCESS;
    return to_cbw(cublasLtMatmulDescDestroy(static_cast<cublasLtMatmulDesc_t>(desc)));
}

cbwStatus_t cbwLtMatrixLayoutCreate(cbwLtMatrixLayout_t* layout, cbwDataType_t type, uint64_t rows, uint64_t cols,
                                    int64_t ld) {
    cublasLtMatrixLayout_t l = nullptr;
    cublasStatus_t e = cublasLtMatrixLayoutCreate(&l, dtype(type), rows, cols, ld);
    *layout = (e == CUBLAS_STATUS_SUCCESS) ? static_cast<cbwLtMatrixLayout_t>(l) : nullptr;
    return to_cbw(e);
}

cbwStatus_t cbwLtMatrixLayoutDestroy(cbwLtMatrixLayout_t layout) {
    if (!layout) return CBW_SUCCESS;
    return to_cbw(cublasLtMatrixLayoutDestroy(static_cast<cublasLtMatrixLayout_t>(layout)));
}

cbwStatus_t cbwLtMatmulPreferenceCreate(cbwLtMatmulPreference_t* pref) {
    cublasLtMatmulPreference_t p = nullptr;
    cublasStatus_t e = cublasLtMatmulPreferenceCreate(&p);
    *pref = (e == CUBLAS_STATUS_SUCCESS) ? static_cast<cbwLtMatmulPreference_t>(p) : nullptr;
    return to_cbw(e);
}

cbwStatus_t cbwLtMatmulPreferenceDestroy(cbwLtMatmulPreference_t pref) {
    if (!pref) return CBW_SUCCESS;
    return to_cbw(cublasLtMatmulPreferenceDestroy(static_cast<cublasLtMatmulPreference_t>(pref)));
}

cbwStatus_t cbwLtMatmul(cbwLtHandle_t ltHandle, cbwLtMatmulDesc_t computeDesc, const void* alpha, const void* A,
                        cbwLtMatrixLayout_t Adesc, const void* B, cbwLtMatrixLayout_t Bdesc, const void* beta,
                        const void* C, cbwLtMatrixLayout_t Cdesc, void* D, cbwLtMatrixLayout_t Ddesc, cwStream_t stream) {
    cublasLtMatmulPreference_t pref = nullptr;
    cublasStatus_t e = cublasLtMatmulPreferenceCreate(&pref);
    if (e != CUBLAS_STATUS_SUCCESS) return to_cbw(e);
    cublasLtMatmulHeuristicResult_t heur = {};
    int found = 0;
    e = cublasLtMatmulAlgoGetHeuristic(static_cast<cublasLtHandle_t>(ltHandle), static_cast<cublasLtMatmulDesc_t>(computeDesc),
                                       static_cast<cublasLtMatrixLayout_t>(Adesc), static_cast<cublasLtMatrixLayout_t>(Bdesc),
                                       static_cast<cublasLtMatrixLayout_t>(Cdesc), static_cast<cublasLtMatrixLayout_t>(Ddesc),
                                       pref, 1, &heur, &found);
    if (e != CUBLAS_STATUS_SUCCESS || found == 0) {
        cublasLtMatmulPreferenceDestroy(pref);
        std::fprintf(stderr, "cublasLtMatmulAlgoGetHeuristic failed\n");
        return e != CUBLAS_STATUS_SUCCESS ? to_cbw(e) : CBW_ERROR_NOT_SUPPORTED;
    }
    e = cublasLtMatmul(static_cast<cublasLtHandle_t>(ltHandle), static_cast<cublasLtMatmulDesc_t>(computeDesc), alpha, A,
                       static_cast<cublasLtMatrixLayout_t>(Adesc), B, static_cast<cublasLtMatrixLayout_t>(Bdesc), beta, C,
                       static_cast<cublasLtMatrixLayout_t>(Cdesc), D, static_cast<cublasLtMatrixLayout_t>(Ddesc), &heur.algo,
                       nullptr, 0, static_cast<cudaStream_t>(stream));
    cublasLtMatmulPreferenceDestroy(pref);
    return report(e, "cublasLtMatmul");
}

const char* cbwGetErrorString(cbwStatus_t status) {
    switch (status) {
        case CBW_SUCCESS: return "Success";
        case CBW_ERROR_NOT_INITIALIZED: return "Not initialized";
        case CBW_ERROR_ALLOC_FAILED: return "Allocation failed";
        case CBW_ERROR_INVALID_VALUE: return "Invalid value";
        case CBW_ERROR_EXECUTION_FAILED: return "Execution failed";
        case CBW_ERROR_INTERNAL: return "Internal error";
        case CBW_ERROR_NOT_SUPPORTED: return "Not supported";
        default: return "Unknown error";
    }
}

}  // extern "C"
