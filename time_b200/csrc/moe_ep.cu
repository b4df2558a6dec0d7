// moe_ep.cu -- the data movement of the expert-parallel MoE FFN block.
//
// Expert parallelism follows the spec's sharding (src/futhark/kernels.fut:
// 612-617 all_to_all, 640-647 shard_experts): rank r owns the routed experts
// [r*E/ep, (r+1)*E/ep) plus a replica of the shared expert, and its own slice
// of the tokens.  One forward on rank r:
//
//   1. RMSNorm + 1x128 FP8 quantisation and the router on its own tokens.
//   2. moe_permute_padded(pad = 1) over all E experts: the (token, slot) pairs
//      in a dense order sorted by global expert, stable in pair order.  The
//      pairs for rank d are then the contiguous block of experts d*E/ep ..
//      (d+1)*E/ep - 1.
//   3. moe_ep_pack_rows: one packed row per pair (FP8 values + their 1x128
//      scales; the dispatch sends exactly the bytes the single-GPU path feeds
//      its GEMM, so the expert outputs are bit-identical).
//   4. Counts all-to-all (E/ep int32 per peer) and one read-back to the host,
//      which NCCL's send/recv need for their sizes; moe_ep_plan_host turns the
//      counts into per-peer row counts and offsets.
//   5. Dispatch all-to-all of the packed rows.
//   6. moe_ep_recv_plan + moe_ep_gather: the received rows, source rank by
//      source rank, become the local experts' 16-aligned row segments (the same
//      within-expert order as the single-GPU permutation, because rank s owns
//      global tokens [s*T_r, (s+1)*T_r)), followed by the shared expert's rows
//      taken from this rank's own tokens.
//   7. The two grouped GEMMs.
//   8. moe_ep_pack_y: expert outputs back into received-row order; combine
//      all-to-all (bf16 rows) returns them to the tokens' owners in their send
//      order, where the combine adds them exactly as on one GPU.
//
// Packed row (moe_ep_row_bytes(H) bytes, a multiple of 16): H e4m3 bytes, then
// H/128 fp32 scales, then zero padding.
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_layer.h"

namespace {

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// One warp per row: 16-byte copies of the FP8 values, one lane per scale.
__global__ void __launch_bounds__(256)
ep_pack_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int xs_ld,
                    const int32_t* __restrict__ row_token, const int32_t* __restrict__ num_rows, int row_capacity,
                    int H, uint8_t* __restrict__ packed, size_t row_bytes) {
    const int R = min(*num_rows, row_capacity);
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    const int nblk = H / 128;
    const int nscale_padded = (nblk * 4 + 15) / 16 * 4;   // row_bytes == H + 4 * nscale_padded
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        const int t = row_token[r];
        uint8_t* dst = packed + static_cast<size_t>(r) * row_bytes;
        const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
        for (int i = lane; i < vec; i += 32) reinterpret_cast<int4*>(dst)[i] = src[i];
        float* ds = reinterpret_cast<float*>(dst + H);
        for (int b = lane; b < nblk; b += 32) ds[b] = xs[static_cast<size_t>(b) * xs_ld + t];
        // zero the padding after the scales so the transferred bytes are defined
        for (int b = nblk + lane; b < nscale_padded; b += 32) ds[b] = 0.0f;
    }
}

// Single block.  recv_counts[s][j] = rows rank s sent for local expert j.
// Builds the GEMM row layout (16-aligned segments, source-major inside each
// expert) and the two index maps between received rows and GEMM rows.
constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads)
ep_recv_plan_kernel(const int32_t* __restrict__ recv_counts, int ep, int epr, int T_local, int num_shared,
                    int32_t* __restrict__ counts, int32_t* __restrict__ seg_start, int32_t* __restrict__ total_rows,
                    int32_t* __restrict__ row_src, int32_t* __restrict__ recv_dst, int row_capacity,
                    int recv_capacity, int* __restrict__ error_word) {
    extern __shared__ int sh[];
    const int G = epr + num_shared;
    const int P = ep * epr;
    int* cnt = sh;              // [ep*epr] copy of recv_counts
    int* src_base = cnt + P;    // [ep*epr] first received row of (s, j)
    int* dst_base = src_base + P;  // [ep*epr] first GEMM row of (s, j)
    int* start = dst_base + P;  // [G]
    __shared__ int s_total, s_recv;
    const int tid = threadIdx.x;
    for (int i = tid; i < P; i += kPlanThreads) cnt[i] = recv_counts[i];
    __syncthreads();
    if (tid == 0) {
        // tiny serial scans (ep*epr <= 1024 entries)
        int run = 0;
        for (int s = 0; s < ep; ++s)
            for (int j = 0; j < epr; ++j) { src_base[s * epr + j] = run; run += cnt[s * epr + j]; }
        s_recv = run;
        int row = 0;
        for (int j = 0; j < epr; ++j) {
            start[j] = row;
            int r = row;
            for (int s = 0; s < ep; ++s) { dst_base[s * epr + j] = r; r += cnt[s * epr + j]; }
            row += (r - row + 15) / 16 * 16;
        }
        for (int g = epr; g < G; ++g) { start[g] = row; row += (T_local + 15) / 16 * 16; }
        s_total = row;
    }
    __syncthreads();
    const int R = s_total;
    if (R > row_capacity || s_recv > recv_capacity) {
        for (int g = tid; g < G; g += kPlanThreads) { counts[g] = 0; seg_start[g] = 0; }
        if (tid == 0) { *total_rows = 0; if (error_word) atomicExch(error_word, 2); }
        return;
    }
    for (int g = tid; g < G; g += kPlanThreads) {
        int c = T_local;
        if (g < epr) { c = 0; for (int s = 0; s < ep; ++s) c += cnt[s * epr + g]; }
        counts[g] = c;
        seg_start[g] = start[g];
    }
    if (tid == 0) *total_rows = R;
    for (int r = tid; r < R; r += kPlanThreads) row_src[r] = -1;
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    for (int pj = warp; pj < P; pj += kPlanThreads / 32) {
        const int n = cnt[pj], sb = src_base[pj], db = dst_base[pj];
        for (int q = lane; q < n; q += 32) {
            row_src[db + q] = sb + q;
            recv_dst[sb + q] = db + q;
        }
    }
    for (int g = epr; g < G; ++g)
        for (int t = tid; t < T_local; t += kPlanThreads) row_src[start[g] + t] = -(t + 2);
}

// GEMM rows from the received packed rows (row_src >= 0), this rank's own
// quantised tokens (row_src = -(t+2), the shared expert), or zeros (-1).
__global__ void __launch_bounds__(256)
ep_gather_kernel(const uint8_t* __restrict__ packed, size_t row_bytes, const uint8_t* __restrict__ xq,
                 const float* __restrict__ xs, int xs_ld, const int32_t* __restrict__ row_src,
                 const int32_t* __restrict__ total_rows, int row_capacity, int H, uint8_t* __restrict__ xp,
                 float* __restrict__ xps, int xps_ld) {
    const int R = min(*total_rows, row_capacity);
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    const int nblk = H / 128;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        const int v = row_src[r];
        int4* dst = reinterpret_cast<int4*>(xp + static_cast<size_t>(r) * H);
        if (v >= 0) {
            const uint8_t* src = packed + static_cast<size_t>(v) * row_bytes;
            for (int i = lane; i < vec; i += 32) dst[i] = reinterpret_cast<const int4*>(src)[i];
            const float* ss = reinterpret_cast<const float*>(src + H);
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = ss[b];
        } else if (v <= -2) {
            const int t = -v - 2;
            const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
            for (int i = lane; i < vec; i += 32) dst[i] = src[i];
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = xs[static_cast<size_t>(b) * xs_ld + t];
        } else {
            const int4 z = make_int4(0, 0, 0, 0);
            for (int i = lane; i < vec; i += 32) dst[i] = z;
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = 0.0f;
        }
    }
}

// ysend[i] = y[recv_dst[i]] (bf16 rows), i < n.
__global__ void __launch_bounds__(256)
ep_pack_y_kernel(const uint8_t* __restrict__ y, const int32_t* __restrict__ recv_dst, int n, size_t row_bytes,
                 uint8_t* __restrict__ ysend) {
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = static_cast<int>(row_bytes / 16);
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n; i += nwarps) {
        const int4* src = reinterpret_cast<const int4*>(y + static_cast<size_t>(recv_dst[i]) * row_bytes);
        int4* dst = reinterpret_cast<int4*>(ysend + static_cast<size_t>(i) * row_bytes);
        for (int c = lane; c < vec; c += 32) dst[c] = src[c];
    }
}

inline int grid_for_rows(int rows) {
    int blocks = (rows + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    return blocks < 1 ? 1 : blocks;
}

}  // namespace

extern "C" {

size_t moe_ep_row_bytes(int H) {
    if (H <= 0 || H % 128) return 0;
    const size_t raw = static_cast<size_t>(H) + static_cast<size_t>(H / 128) * 4;
    return (raw + 15) / 16 * 16;
}

moe_status_t moe_ep_plan_host(int ep_size, int experts_per_rank, const int32_t* send_expert_counts,
                              const int32_t* recv_counts, size_t* send_rows, size_t* send_offsets,
                              size_t* recv_rows, size_t* recv_offsets, size_t* send_total, size_t* recv_total) {
    if (ep_size <= 0 || experts_per_rank <= 0 || !send_expert_counts || !recv_counts || !send_rows || !send_offsets ||
        !recv_rows || !recv_offsets)
        return MOE_ERR_INVALID_ARGUMENT;
    size_t so = 0, ro = 0;
    for (int p = 0; p < ep_size; ++p) {
        size_t sn = 0, rn = 0;
        for (int j = 0; j < experts_per_rank; ++j) {
            const int32_t a = send_expert_counts[p * experts_per_rank + j];
            const int32_t b = recv_counts[p * experts_per_rank + j];
            if (a < 0 || b < 0) return MOE_ERR_INVALID_ARGUMENT;
            sn += static_cast<size_t>(a);
            rn += static_cast<size_t>(b);
        }
        send_rows[p] = sn;
        send_offsets[p] = so;
        recv_rows[p] = rn;
        recv_offsets[p] = ro;
        so += sn;
        ro += rn;
    }
    if (send_total) *send_total = so;
    if (recv_total) *recv_total = ro;
    return MOE_OK;
}

moe_status_t moe_ep_pack_rows(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                              const int32_t* num_rows, int row_capacity, int H, void* packed, cwStream_t stream) {
    const size_t rb = moe_ep_row_bytes(H);
    if (!rb || !xq || !xs || !row_token || !num_rows || !packed || row_capacity < 0) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(xq) || !aligned16(packed)) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    ep_pack_rows_kernel<<<grid_for_rows(row_capacity), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(xq), xs, xs_ld, row_token, num_rows, row_capacity, H,
        static_cast<uint8_t*>(packed), rb);
    return launch_status();
}

moe_status_t moe_ep_recv_plan(const int32_t* recv_counts, int ep_size, int experts_per_rank, int T_local,
                              int num_shared, int32_t* counts, int32_t* seg_start, int32_t* total_rows,
                              int32_t* row_src, int32_t* recv_dst, int row_capacity, int recv_capacity,
                              int* error_word, cwStream_t stream) {
    if (!recv_counts || !counts || !seg_start || !total_rows || !row_src || !recv_dst) return MOE_ERR_INVALID_ARGUMENT;
    if (ep_size <= 0 || experts_per_rank <= 0 || ep_size * experts_per_rank > 1024 || T_local < 0 || num_shared < 0 ||
        num_shared > 1 || row_capacity < 0 || recv_capacity < 0)
        return MOE_ERR_INVALID_ARGUMENT;
    const int P = ep_size * experts_per_rank;
    const size_t smem = static_cast<size_t>(3 * P + experts_per_rank + num_shared) * sizeof(int);
    ep_recv_plan_kernel<<<1, kPlanThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        recv_counts, ep_size, experts_per_rank, T_local, num_shared, counts, seg_start, total_rows, row_src,
        recv_dst, row_capacity, recv_capacity, error_word);
    return launch_status();
}

moe_status_t moe_ep_gather(const void* packed, const void* xq, const float* xs, int xs_ld, const int32_t* row_src,
                           const int32_t* total_rows, int row_capacity, int H, void* xp, float* xps, int xps_ld,
                           cwStream_t stream) {
    const size_t rb = moe_ep_row_bytes(H);
    if (!rb || !packed || !xq || !xs || !row_src || !total_rows || !xp || !xps || row_capacity < 0 ||
        xps_ld < row_capacity)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(packed) || !aligned16(xq) || !aligned16(xp)) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    ep_gather_kernel<<<grid_for_rows(row_capacity), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(packed), rb, static_cast<const uint8_t*>(xq), xs, xs_ld, row_src, total_rows,
        row_capacity, H, static_cast<uint8_t*>(xp), xps, xps_ld);
    return launch_status();
}

moe_status_t moe_ep_pack_y(const void* y_bf16, const int32_t* recv_dst, int n, int H, void* ysend_bf16,
                           cwStream_t stream) {
    if (!y_bf16 || !recv_dst || !ysend_bf16 || n < 0 || H <= 0 || H % 8) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(y_bf16) || !aligned16(ysend_bf16)) return MOE_ERR_INVALID_ARGUMENT;
    if (n == 0) return MOE_OK;
    ep_pack_y_kernel<<<grid_for_rows(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(y_bf16), recv_dst, n, static_cast<size_t>(H) * 2,
        static_cast<uint8_t*>(ysend_bf16));
    return launch_status();
}

}  // extern "C"
