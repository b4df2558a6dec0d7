/*
 * cublas_wrappers.h -- GEMM shim (libcublaswrap.so), drop-in for the
 * reference engine's csrc/cublas_wrappers.h.
 *
 * The 17 cbw* entry points, enums and handle typedefs are the binary
 * interface the engine links (csrc/cublas_wrappers.h:12-67) and are kept as
 * declared there.  They remain thin cuBLAS/cuBLASLt calls (plain library
 * GEMMs; the engine uses only cbwSgemm, src/terra/engine.t:1275-1366).
 *
 * New: cbwFp8BlockScaledGroupedGemm, the hand-written sm_100a grouped expert
 * GEMM (TMA + tcgen05/TMEM) that replaces the reference's per-slot
 * "launch_fp8_dequantize + cbwSgemm" sequence (engine.t:1321-1346).
 */
#ifndef CUBLAS_WRAPPERS_H
#define CUBLAS_WRAPPERS_H

#include <stdint.h>
#include <stddef.h>
#include "cuda_wrappers.h"

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/cublas_wrappers.h:12-20 */
typedef enum {
    CBW_SUCCESS = 0,
    CBW_ERROR_NOT_INITIALIZED = 1,
    CBW_ERROR_ALLOC_FAILED = 3,
    CBW_ERROR_INVALID_VALUE = 7,
    CBW_ERROR_EXECUTION_FAILED = 13,
    CBW_ERROR_INTERNAL = 14,
    CBW_ERROR_NOT_SUPPORTED = 15
} cbwStatus_t;

/* csrc/cublas_wrappers.h:22-26 */
typedef enum {
    CBW_OP_N = 0,
    CBW_OP_T = 1,
    CBW_OP_C = 2
} cbwOperation_t;

/* csrc/cublas_wrappers.h:28-35 */
typedef enum {
    CBW_R_16F = 0,
    CBW_R_32F = 1,
    CBW_R_64F = 2,
    CBW_R_16BF = 3,
    CBW_R_8F_E4M3 = 4,
    CBW_R_8F_E5M2 = 5
} cbwDataType_t;

/* csrc/cublas_wrappers.h:37-43 */
typedef enum {
    CBW_COMPUTE_16F = 0,
    CBW_COMPUTE_32F = 1,
    CBW_COMPUTE_64F = 2,
    CBW_COMPUTE_32F_FAST_16F = 3,
    CBW_COMPUTE_32F_FAST_TF32 = 4
} cbwComputeType_t;

/* csrc/cublas_wrappers.h:45-49 */
typedef void* cbwHandle_t;
typedef void* cbwLtHandle_t;
typedef void* cbwLtMatmulDesc_t;
typedef void* cbwLtMatrixLayout_t;
typedef void* cbwLtMatmulPreference_t;

/* csrc/cublas_wrappers.h:51 */ cbwStatus_t cbwCreate(cbwHandle_t* handle);
/* csrc/cublas_wrappers.h:52 */ cbwStatus_t cbwDestroy(cbwHandle_t handle);
/* csrc/cublas_wrappers.h:53 */ cbwStatus_t cbwSetStream(cbwHandle_t handle, cwStream_t stream);
/* csrc/cublas_wrappers.h:54 */ cbwStatus_t cbwSgemm(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k, const float* alpha, const float* A, int lda, const float* B, int ldb, const float* beta, float* C, int ldc);
/* csrc/cublas_wrappers.h:55 */ cbwStatus_t cbwHgemm(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k, const void* alpha, const void* A, int lda, const void* B, int ldb, const void* beta, void* C, int ldc);
/* csrc/cublas_wrappers.h:56 */ cbwStatus_t cbwSgemmBatched(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k, const float* alpha, const float** Aarray, int lda, const float** Barray, int ldb, const float* beta, float** Carray, int ldc, int batchCount);
/* csrc/cublas_wrappers.h:57 */ cbwStatus_t cbwSgemmStridedBatched(cbwHandle_t handle, cbwOperation_t transa, cbwOperation_t transb, int m, int n, int k, const float* alpha, const float* A, int lda, long long strideA, const float* B, int ldb, long long strideB, const float* beta, float* C, int ldc, long long strideC, int batchCount);
/* csrc/cublas_wrappers.h:58 */ cbwStatus_t cbwLtCreate(cbwLtHandle_t* handle);
/* csrc/cublas_wrappers.h:59 */ cbwStatus_t cbwLtDestroy(cbwLtHandle_t handle);
/* csrc/cublas_wrappers.h:60 */ cbwStatus_t cbwLtMatmulDescCreate(cbwLtMatmulDesc_t* desc, cbwComputeType_t computeType, cbwDataType_t scaleType);
/* csrc/cublas_wrappers.h:61 */ cbwStatus_t cbwLtMatmulDescDestroy(cbwLtMatmulDesc_t desc);
/* csrc/cublas_wrappers.h:62 */ cbwStatus_t cbwLtMatrixLayoutCreate(cbwLtMatrixLayout_t* layout, cbwDataType_t type, uint64_t rows, uint64_t cols, int64_t ld);
/* csrc/cublas_wrappers.h:63 */ cbwStatus_t cbwLtMatrixLayoutDestroy(cbwLtMatrixLayout_t layout);
/* csrc/cublas_wrappers.h:64 */ cbwStatus_t cbwLtMatmulPreferenceCreate(cbwLtMatmulPreference_t* pref);
/* csrc/cublas_wrappers.h:65 */ cbwStatus_t cbwLtMatmulPreferenceDestroy(cbwLtMatmulPreference_t pref);
/* csrc/cublas_wrappers.h:66 */ cbwStatus_t cbwLtMatmul(cbwLtHandle_t ltHandle, cbwLtMatmulDesc_t computeDesc, const void* alpha, const void* A, cbwLtMatrixLayout_t Adesc, const void* B, cbwLtMatrixLayout_t Bdesc, const void* beta, const void* C, cbwLtMatrixLayout_t Cdesc, void* D, cbwLtMatrixLayout_t Ddesc, cwStream_t stream);
/* csrc/cublas_wrappers.h:67 */ const char* cbwGetErrorString(cbwStatus_t status);

/* ------------------------------------------------------------------------
 * Grouped block-scaled FP8 expert GEMM (new; replaces engine.t:1321-1346).
 *
 * For every group g (an expert) with count[g] rows starting at row
 * start[g] of the activation matrix A:
 *   acc[r][n] = sum_kb  a_scale[kb][r] * w_scale[g][n/128][kb]
 *                       * sum_{k in kb} A[r][k] * W[g][n][k]
 * with A, W in e4m3 (K-major rows), 128-wide K blocks, fp32 accumulation.
 *
 * mode CBW_GEMM_GATED_SWIGLU: W[g] holds 2N rows (gate rows [0,N), up rows
 *   [N,2N)); the output is h = silu(gate) * up, quantised per 128 columns:
 *   out_q[r][n] (e4m3) and out_scale[n/128][r] (fp32) -- the input format of
 *   the down projection.  Rows in [count, round_up(count,16)) are zeroed.
 * mode CBW_GEMM_DOWN_BF16: W[g] holds N rows; out[r][n] = bf16(acc).
 * Either mode may be or-ed with CBW_GEMM_SMALL_TILES (tiles of at most 32
 * rows and a deeper weight ring: the decode form) or CBW_GEMM_FULL_TILES;
 * without either, small tiles are used when rows <= 32 * num_groups.  The
 * full form has three variants with bit-identical results: token-major tiles
 * (128 rows x 256 weight rows per instruction -- the gate and up rows of 128
 * output columns, or 256 down rows; the down mode needs N % 256 == 0), one SM
 * per tile (128 weight rows x up to 128 rows), and pairs of SMs (tcgen05
 * cta_group::2, 256 weight rows x up to 128 rows; needs K % 256 == 0 and,
 * for the down mode, N % 256 == 0).  By default both modes run token-major;
 * a down projection with N % 256 != 0 runs on one SM (one plane) or in
 * 32-token tiles (two planes).  CBW_GEMM_TOKEN_TILES, CBW_GEMM_ONE_SM_TILES or
 * CBW_GEMM_PAIR_TILES (instead of FULL) picks one.
 * The decode form adds a row's K blocks in a different order from the full
 * form, so its results differ from the full form's in the last bits.
 *
 * CBW_GEMM_ACT_X2 (or-ed in; no counterpart in the reference): two-term
 * activations.  A holds two e4m3 planes, hi at a and lo at a + rows*K bytes,
 * with one scale: A = a_scale * (decode(hi) + decode(lo)), lo being the e4m3
 * rounding of the residual (x/scale - decode(hi)).  Each K block's tensor-core
 * partial covers both planes (twice the MMA work) and carries about 7
 * significant bits of every activation instead of 4.  The gated mode then
 * writes its output in the same two-plane form (hi at out, lo at
 * out + rows*N); the down mode reads it.  The full down form runs token-major
 * or on CTA pairs (both need N % 256 == 0) or else in 32-token tiles.
 *
 * Requirements: K % 128 == 0, N % 128 == 0, start[g] % 16 == 0, every
 * segment [start, start + round_up(count,16)) inside [0, rows), a_ld (the
 * scale leading dimension) % 4 == 0 and >= rows, 16-byte aligned pointers.
 * count/start are device arrays; the kernel reads them (no host sync).
 * error_word: device int set non-zero if a device-side wait timed out.
 */
typedef enum {
    CBW_GEMM_GATED_SWIGLU = 0,
    CBW_GEMM_DOWN_BF16 = 1,
    CBW_GEMM_SMALL_TILES = 0x10,
    CBW_GEMM_FULL_TILES = 0x20,
    CBW_GEMM_ONE_SM_TILES = 0x40,
    CBW_GEMM_PAIR_TILES = 0x80,
    CBW_GEMM_TOKEN_TILES = 0x30,
    CBW_GEMM_ACT_X2 = 0x100
} cbwGemmMode_t;

typedef struct {
    int mode;                  /* cbwGemmMode_t */
    int num_groups;            /* G */
    int K;                     /* reduction size, % 128 == 0 */
    int N;                     /* output columns (I for gated, H for down) */
    int rows;                  /* rows of A / outputs */
    const void* a;             /* [rows][K] e4m3 */
    const float* a_scale;      /* [K/128][a_ld] */
    int a_ld;
    const void* w;             /* [G][N or 2N][K] e4m3 */
    const float* w_scale;      /* [G][(N or 2N)/128][K/128] */
    const int32_t* count;      /* [G] device */
    const int32_t* start;      /* [G] device */
    void* out;                 /* gated: [rows][N] e4m3; down: [rows][N] bf16 */
    float* out_scale;          /* gated: [N/128][out_ld]; down: unused */
    int out_ld;
} cbwGroupedGemmArgs;

cbwStatus_t cbwFp8BlockScaledGroupedGemm(const cbwGroupedGemmArgs* args, int* error_word,
                                         cwStream_t stream);

/* Extension (no reference counterpart): the down projection with one output
 * address per row, the expert-parallel return fused into the GEMM.
 * row_out: device array [rows] of bf16 row addresses (N * 2 bytes each,
 * 16-byte aligned), nullptr for rows that go to args->out as usual; an
 * address may lie in another GPU's memory (peer mapping).  Every storing
 * thread fences at system scope before the grid ends, so a flag raised by the
 * next launch on the stream orders all rows before it.  Only the token-major
 * down form takes row addresses: CBW_ERROR_NOT_SUPPORTED (nothing launched)
 * when the mode or the shape selects another form. */
cbwStatus_t cbwFp8BlockScaledGroupedGemmRowOut(const cbwGroupedGemmArgs* args, void* const* row_out,
                                               int* error_word, cwStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CUBLAS_WRAPPERS_H */
