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
// H/128 fp32 scales, then zero padding.  Two-term activations add the lo
// plane's H bytes after the hi plane's (moe_ep_row_bytes(H) + H bytes).
//
// Peer-memory exchange (moe_layer_set_peer_buffers): the same protocol with no
// NCCL and no host synchronisation.  Every rank owns a symmetric buffer that
// all ranks have mapped (NVLink peer memory):
//   flags [3][kMaxEpRanks] u32   counts / dispatch / combine epochs, one per source
//   table [ep][E + ep] i32       every rank's per-expert send counts, then its
//                                row counts per destination rank
//   recv  [recv_cap][rb]         packed rows dispatched to this rank: one per
//                                (source token, this rank), source-major
//   pmap  [recv_cap] i32         per received pair (source-major, the sender's
//                                expert order): its row in recv
//   yrecv [T*k][H] bf16          expert outputs returned to this rank
// Per forward (epoch e = 1, 2, ..., counted on the device): ep_counts_kernel writes this rank's
// counts into every table and raises flags[0][me] = e on every rank, waits for
// all ranks' flags, then derives the whole exchange plan on the device;
// ep_dispatch_kernel packs each token that has a pair for a destination
// straight into that destination's recv buffer, once however many of the
// token's experts live there (ep_unique_kernel numbers those tokens), and
// writes every pair's row index into the destination's pmap, so the receiving
// gather builds the same expert segments from fewer transferred rows; ep_signal_wait_kernel raises flags[1][me] and waits for every
// source; each expert output row then goes into its token owner's yrecv --
// copied there by ep_combine_send_kernel after the GEMM, or (optional,
// token-major down form) stored there by the down GEMM's own epilogue, which
// ep_return_rows_kernel gives every row's address -- and flags[2] closes the
// step.  Writers fence
// (system scope) before a release store of the flag; waiters acquire.  Every
// wait is a bounded spin of one thread (error word 3 on timeout).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "sm100.cuh"
#include "moe_layer.h"
#include "moe_ep_peer.h"

namespace {

using namespace tb;

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// vidx[p] = slot_of_expert[idx[p]] for valid expert ids, -1 otherwise.
__global__ void ep_remap_kernel(const int32_t* __restrict__ idx, int P, int E, const int32_t* __restrict__ slot_of,
                                int32_t* __restrict__ vidx) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x) {
        const int e = idx[p];
        vidx[p] = (e >= 0 && e < E) ? slot_of[e] : -1;
    }
}

// One warp per row: 16-byte copies of the FP8 values, one lane per scale.
__global__ void __launch_bounds__(256)
ep_pack_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int xs_ld,
                    const int32_t* __restrict__ row_token, const int32_t* __restrict__ num_rows, int row_capacity,
                    int H, uint8_t* __restrict__ packed, size_t row_bytes, const uint8_t* __restrict__ xq_lo) {
    const int R = min(*num_rows, row_capacity);
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    const int nblk = H / 128;
    const int nscale_padded = (nblk * 4 + 15) / 16 * 4;   // row_bytes == planes * H + 4 * nscale_padded
    const int planes = xq_lo ? 2 : 1;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        const int t = row_token[r];
        uint8_t* dst = packed + static_cast<size_t>(r) * row_bytes;
        const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
        for (int i = lane; i < vec; i += 32) reinterpret_cast<int4*>(dst)[i] = src[i];
        if (xq_lo) {
            const int4* slo = reinterpret_cast<const int4*>(xq_lo + static_cast<size_t>(t) * H);
            for (int i = lane; i < vec; i += 32) reinterpret_cast<int4*>(dst + H)[i] = slo[i];
        }
        float* ds = reinterpret_cast<float*>(dst + static_cast<size_t>(planes) * H);
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
                 float* __restrict__ xps, int xps_ld, const uint8_t* __restrict__ xq_lo, uint8_t* __restrict__ xp_lo,
                 const int32_t* __restrict__ pmap = nullptr, int pmap_bound = 0) {
    const int R = min(*total_rows, row_capacity);
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    const int nblk = H / 128;
    const int planes = xp_lo ? 2 : 1;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        int v = row_src[r];
        if (pmap && v >= 0) {               // received pair -> its (token, this rank) row
            v = v < pmap_bound ? pmap[v] : -1;
            if (v < 0 || v >= pmap_bound) v = -1;   // cannot happen for a well-formed exchange: a zero row
        }
        int4* dst = reinterpret_cast<int4*>(xp + static_cast<size_t>(r) * H);
        int4* dlo = xp_lo ? reinterpret_cast<int4*>(xp_lo + static_cast<size_t>(r) * H) : nullptr;
        if (v >= 0) {
            const uint8_t* src = packed + static_cast<size_t>(v) * row_bytes;
            for (int i = lane; i < vec; i += 32) dst[i] = reinterpret_cast<const int4*>(src)[i];
            if (dlo)
                for (int i = lane; i < vec; i += 32) dlo[i] = reinterpret_cast<const int4*>(src + H)[i];
            const float* ss = reinterpret_cast<const float*>(src + static_cast<size_t>(planes) * H);
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = ss[b];
        } else if (v <= -2) {
            const int t = -v - 2;
            const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
            for (int i = lane; i < vec; i += 32) dst[i] = src[i];
            if (dlo) {
                const int4* slo = reinterpret_cast<const int4*>(xq_lo + static_cast<size_t>(t) * H);
                for (int i = lane; i < vec; i += 32) dlo[i] = slo[i];
            }
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = xs[static_cast<size_t>(b) * xs_ld + t];
        } else {
            const int4 z = make_int4(0, 0, 0, 0);
            for (int i = lane; i < vec; i += 32) dst[i] = z;
            if (dlo)
                for (int i = lane; i < vec; i += 32) dlo[i] = z;
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

// ---------------------------------------------------------------- peer memory

constexpr int kMaxEpRanks = 64;
enum { kFlagCounts = 0, kFlagDispatch = 1, kFlagCombine = 2 };
// plan[] layout (int32, device): per rank d (kPlanStride entries): soff,
// srows (my pairs for d, in my send order), roff_in (where my pairs land in
// d's pair positions), recv_off, rrows (pairs from d), ysoff (where d's
// outputs for my experts land in d's send order), usoff, usrows (my rows for
// d: tokens with a pair there), uoff_in (where my rows land in d's recv);
// then stot, rtot, utot.
enum {
    kPlanSoff = 0, kPlanSrows = 1, kPlanRoffIn = 2, kPlanRecvOff = 3, kPlanRrows = 4, kPlanYsoff = 5,
    kPlanUsoff = 6, kPlanUsrows = 7, kPlanUoffIn = 8, kPlanStride = 9
};

struct EpPeers {
    uint8_t* base[kMaxEpRanks];   // rank r's symmetric buffer as mapped in this process
    int ep, me, E, epr;
    size_t off_flags, off_table, off_recv, off_pmap, off_yrecv;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ uint32_t* flag_ptr(const EpPeers& P, int rank, int phase, int src) {
    return reinterpret_cast<uint32_t*>(P.base[rank] + P.off_flags) + phase * kMaxEpRanks + src;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread: raise this rank's flag for `phase` on every rank, then wait
// until every source has raised its flag here.  False on timeout.
__device__ bool signal_and_wait(const EpPeers& P, int phase, uint32_t epoch) {
    __threadfence_system();
    for (int d = 0; d < P.ep; ++d) st_release_sys(flag_ptr(P, d, phase, P.me), epoch);
    const uint64_t t0 = globaltimer_ns();
    for (int s = 0; s < P.ep; ++s) {
        const uint32_t* f = flag_ptr(P, P.me, phase, s);
        while (ld_acquire_sys(f) != epoch) {
            if (globaltimer_ns() - t0 > P.timeout_ns) return false;
            __nanosleep(64);
        }
    }
    return true;
}

// Single block of kUniqueThreads.  For every destination rank d, the tokens
// of this rank with at least one pair routed to d (vid = virtual expert, rank
// vid / epr), numbered in token order: uidx[d][t] (-1 when none) and
// utok[d][u]; ucount[d] rows.  Per 1024-token chunk one block scan per group
// of four destinations, each destination a 16-bit field of a 64-bit sum (a
// chunk counts at most 1024 tokens, so the fields never carry).
constexpr int kUniqueThreads = 1024;

__global__ void __launch_bounds__(kUniqueThreads)
ep_unique_kernel(const int32_t* __restrict__ vid, int T, int K, int ep, int epr, int32_t* __restrict__ uidx,
                 int32_t* __restrict__ utok, int32_t* __restrict__ ucount) {
    __shared__ unsigned long long wsum[kUniqueThreads / 32];
    __shared__ int run[kMaxEpRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int d = tid; d < ep; d += kUniqueThreads) run[d] = 0;
    __syncthreads();
    const int groups = (ep + 3) / 4;
    for (int c0 = 0; c0 < T; c0 += kUniqueThreads) {
        const int t = c0 + tid;
        unsigned long long mask = 0;
        if (t < T)
            for (int s = 0; s < K; ++s) {
                const int v = vid[static_cast<size_t>(t) * K + s];
                if (v >= 0 && v < ep * epr) mask |= 1ull << (v / epr);
            }
        for (int g = 0; g < groups; ++g) {
            unsigned long long x = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int d = 4 * g + q;
                if (d < ep && ((mask >> d) & 1ull)) x |= 1ull << (16 * q);
            }
            unsigned long long inc = x;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            if (lane == 31) wsum[warp] = inc;
            __syncthreads();
            if (warp == 0) {
                unsigned long long w = wsum[lane];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned long long y = __shfl_up_sync(0xffffffffu, w, o);
                    if (lane >= o) w += y;
                }
                wsum[lane] = w;
            }
            __syncthreads();
            const unsigned long long excl = inc - x + (warp ? wsum[warp - 1] : 0ull);
            if (t < T) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int d = 4 * g + q;
                    if (d >= ep) break;
                    if ((mask >> d) & 1ull) {
                        const int u = run[d] + static_cast<int>((excl >> (16 * q)) & 0xFFFFull);
                        uidx[static_cast<size_t>(d) * T + t] = u;
                        utok[static_cast<size_t>(d) * T + u] = t;
                    } else {
                        uidx[static_cast<size_t>(d) * T + t] = -1;
                    }
                }
            }
            __syncthreads();   // every thread has read run[] and wsum[]
            if (tid < 4 && 4 * g + tid < ep)
                run[4 * g + tid] += static_cast<int>((wsum[kUniqueThreads / 32 - 1] >> (16 * tid)) & 0xFFFFull);
            __syncthreads();
        }
    }
    for (int d = tid; d < ep; d += kUniqueThreads) ucount[d] = run[d];
}

// Single block: counts into every table, barrier, then the exchange plan.
// A table row is [E per-expert pair counts][ep row counts per destination].
__global__ void __launch_bounds__(256)
ep_counts_kernel(const EpPeers P, const int32_t* __restrict__ ecounts, const int32_t* __restrict__ ucounts,
                 uint32_t* __restrict__ epoch_dev, int32_t* __restrict__ plan,
                 int32_t* __restrict__ rcounts, int* __restrict__ error_word) {
    const int tid = threadIdx.x;
    const int W = P.E + P.ep;   // table row stride
    for (int d = 0; d < P.ep; ++d) {
        int32_t* tab = reinterpret_cast<int32_t*>(P.base[d] + P.off_table) + static_cast<size_t>(P.me) * W;
        for (int e = tid; e < P.E; e += blockDim.x) tab[e] = ecounts[e];
        for (int e = tid; e < P.ep; e += blockDim.x) tab[P.E + e] = ucounts[e];
    }
    __threadfence_system();
    __syncthreads();
    __shared__ int ok;
    if (tid == 0) {
        // the forward's epoch lives on the device (a captured graph replays with the next one)
        const uint32_t epoch = *epoch_dev + 1u;
        *epoch_dev = epoch;
        ok = signal_and_wait(P, kFlagCounts, epoch) ? 1 : 0;
    }
    __syncthreads();
    if (!ok) {
        if (tid == 0) {
            if (error_word) atomicExch(error_word, 3);
            for (int i = 0; i < kPlanStride * P.ep + 3; ++i) plan[i] = 0;   // nothing moves
        }
        for (int i = tid; i < P.ep * P.epr; i += blockDim.x) rcounts[i] = 0;
        return;
    }
    // every source's counts and this rank's own into shared memory, then one
    // warp per destination rank sums its plan entries in parallel (the sums
    // are integers: the order does not matter)
    extern __shared__ int sh_counts[];
    const int EE = P.E, ep = P.ep, epr = P.epr, me = P.me;
    int* stab = sh_counts;              // [ep][W]
    int* mine_c = sh_counts + ep * W;   // [E]
    const int32_t* tab = reinterpret_cast<const int32_t*>(P.base[P.me] + P.off_table);   // [ep][W], all sources
    for (int i = tid; i < ep * W; i += blockDim.x) stab[i] = tab[i];
    for (int i = tid; i < EE; i += blockDim.x) mine_c[i] = ecounts[i];
    __syncthreads();
    for (int i = tid; i < ep * epr; i += blockDim.x) {
        const int s = i / epr, j = i % epr;
        rcounts[i] = stab[s * W + me * epr + j];
    }
    __shared__ int v_sn[kMaxEpRanks], v_rn[kMaxEpRanks], v_before[kMaxEpRanks], v_ys[kMaxEpRanks];
    __shared__ int v_ubefore[kMaxEpRanks];
    const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    for (int d = warp; d < ep; d += nwarps) {
        int sn = 0, rn = 0, before = 0, ys = 0, ubefore = 0;
        for (int j = lane; j < epr; j += 32) {
            sn += mine_c[d * epr + j];                   // my pairs for d
            rn += stab[d * W + me * epr + j];            // d's pairs for me
        }
        for (int i = lane; i < me * epr; i += 32) {
            before += stab[(i / epr) * W + d * epr + i % epr];   // earlier sources' pairs for d
            ys += stab[d * W + i];                                // d's pairs before mine
        }
        for (int s = lane; s < me; s += 32) ubefore += stab[s * W + EE + d];   // earlier sources' rows for d
        for (int o = 16; o > 0; o >>= 1) {
            sn += __shfl_xor_sync(0xffffffffu, sn, o);
            rn += __shfl_xor_sync(0xffffffffu, rn, o);
            before += __shfl_xor_sync(0xffffffffu, before, o);
            ys += __shfl_xor_sync(0xffffffffu, ys, o);
            ubefore += __shfl_xor_sync(0xffffffffu, ubefore, o);
        }
        if (lane == 0) {
            v_sn[d] = sn;
            v_rn[d] = rn;
            v_before[d] = before;
            v_ys[d] = ys;
            v_ubefore[d] = ubefore;
        }
    }
    __syncthreads();
    if (tid == 0) {
        int32_t* pl = plan;
        int so = 0, ro = 0, uo = 0;
        for (int d = 0; d < ep; ++d) {
            int32_t* q = pl + kPlanStride * d;
            const int un = stab[me * W + EE + d];   // my rows for d
            q[kPlanSoff] = so;
            q[kPlanSrows] = v_sn[d];
            q[kPlanRoffIn] = v_before[d];
            q[kPlanRecvOff] = ro;
            q[kPlanRrows] = v_rn[d];
            q[kPlanYsoff] = v_ys[d];
            q[kPlanUsoff] = uo;
            q[kPlanUsrows] = un;
            q[kPlanUoffIn] = v_ubefore[d];
            so += v_sn[d];
            ro += v_rn[d];
            uo += un;
        }
        pl[kPlanStride * ep] = so;       // stot
        pl[kPlanStride * ep + 1] = ro;   // rtot
        pl[kPlanStride * ep + 2] = uo;   // utot
    }
}

// Warp per sent row -- one per (destination, token with a pair there) --
// packs values + scales straight into the destination's recv; then a thread
// per sent pair writes the pair's row index into the destination's pmap.
__global__ void __launch_bounds__(256)
ep_dispatch_kernel(const EpPeers P, const uint8_t* __restrict__ xq, const float* __restrict__ xs, int xs_ld,
                   const int32_t* __restrict__ stok, const int32_t* __restrict__ uidx,
                   const int32_t* __restrict__ utok, int T, const int32_t* __restrict__ plan, int H, size_t row_bytes,
                   int recv_cap, const uint8_t* __restrict__ xq_lo) {
    __shared__ int s_soff[kMaxEpRanks], s_roff[kMaxEpRanks], s_usoff[kMaxEpRanks], s_uoff[kMaxEpRanks];
    for (int d = threadIdx.x; d < P.ep; d += blockDim.x) {
        s_soff[d] = plan[kPlanStride * d + kPlanSoff];
        s_roff[d] = plan[kPlanStride * d + kPlanRoffIn];
        s_usoff[d] = plan[kPlanStride * d + kPlanUsoff];
        s_uoff[d] = plan[kPlanStride * d + kPlanUoffIn];
    }
    __syncthreads();
    const int stot = plan[kPlanStride * P.ep];
    const int utot = plan[kPlanStride * P.ep + 2];
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16, nblk = H / 128;
    const int nscale_padded = (nblk * 4 + 15) / 16 * 4;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < utot; i += nwarps) {
        int d = P.ep - 1;
        while (d > 0 && s_usoff[d] > i) --d;
        const int u = i - s_usoff[d];
        const int dest = s_uoff[d] + u;
        if (u >= T || dest >= recv_cap) continue;   // cannot happen within max_tokens (checked by the plan)
        const int t = utok[static_cast<size_t>(d) * T + u];
        if (t < 0 || t >= T) continue;
        uint8_t* dst = P.base[d] + P.off_recv + static_cast<size_t>(dest) * row_bytes;
        const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
        for (int c = lane; c < vec; c += 32) reinterpret_cast<int4*>(dst)[c] = src[c];
        if (xq_lo) {
            const int4* slo = reinterpret_cast<const int4*>(xq_lo + static_cast<size_t>(t) * H);
            for (int c = lane; c < vec; c += 32) reinterpret_cast<int4*>(dst + H)[c] = slo[c];
        }
        float* ds = reinterpret_cast<float*>(dst + static_cast<size_t>(xq_lo ? 2 : 1) * H);
        for (int b = lane; b < nscale_padded; b += 32) ds[b] = (b < nblk) ? xs[static_cast<size_t>(b) * xs_ld + t] : 0.0f;
    }
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < stot; r += gridDim.x * blockDim.x) {
        int d = P.ep - 1;
        while (d > 0 && s_soff[d] > r) --d;
        const int pos = s_roff[d] + (r - s_soff[d]);
        if (pos >= recv_cap) continue;
        const int t = stok[r];
        const int u = (t >= 0 && t < T) ? uidx[static_cast<size_t>(d) * T + t] : -1;
        reinterpret_cast<int32_t*>(P.base[d] + P.off_pmap)[pos] = u >= 0 ? s_uoff[d] + u : recv_cap;
    }
    __threadfence_system();
}

// Warp per received row: its expert output goes back into the token owner's yrecv.
__global__ void __launch_bounds__(256)
ep_combine_send_kernel(const EpPeers P, const uint8_t* __restrict__ y, const int32_t* __restrict__ recv_dst,
                       const int32_t* __restrict__ plan, size_t row_bytes, int ycap, int y_rows) {
    __shared__ int s_roff[kMaxEpRanks], s_ys[kMaxEpRanks];
    for (int d = threadIdx.x; d < P.ep; d += blockDim.x) {
        s_roff[d] = plan[kPlanStride * d + kPlanRecvOff];
        s_ys[d] = plan[kPlanStride * d + kPlanYsoff];
    }
    __syncthreads();
    const int rtot = plan[kPlanStride * P.ep + 1];
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = static_cast<int>(row_bytes / 16);
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rtot; i += nwarps) {
        int s = P.ep - 1;
        while (s > 0 && s_roff[s] > i) --s;
        const int dest = s_ys[s] + (i - s_roff[s]);
        const int yr = recv_dst[i];
        if (dest >= ycap || yr < 0 || yr >= y_rows) continue;
        const int4* src = reinterpret_cast<const int4*>(y + static_cast<size_t>(yr) * row_bytes);
        int4* dst = reinterpret_cast<int4*>(P.base[s] + P.off_yrecv + static_cast<size_t>(dest) * row_bytes);
        for (int c = lane; c < vec; c += 32) dst[c] = src[c];
    }
    __threadfence_system();
}

// Thread per GEMM row: the address its down-projection output goes to when the
// GEMM returns rows itself -- a received row's place in its token owner's
// yrecv (the row ep_combine_send_kernel would copy there), nullptr for this
// rank's shared-expert and padding rows, which stay in the local y.
__global__ void __launch_bounds__(256)
ep_return_rows_kernel(const EpPeers P, const int32_t* __restrict__ row_src, const int32_t* __restrict__ total_rows,
                      const int32_t* __restrict__ plan, size_t row_bytes, int ycap, int row_capacity,
                      void** __restrict__ row_out) {
    __shared__ int s_roff[kMaxEpRanks], s_ys[kMaxEpRanks];
    for (int d = threadIdx.x; d < P.ep; d += blockDim.x) {
        s_roff[d] = plan[kPlanStride * d + kPlanRecvOff];
        s_ys[d] = plan[kPlanStride * d + kPlanYsoff];
    }
    __syncthreads();
    const int R = min(*total_rows, row_capacity);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
        const int sb = row_src[r];
        void* dst = nullptr;
        if (sb >= 0) {
            int s = P.ep - 1;
            while (s > 0 && s_roff[s] > sb) --s;
            const int dest = s_ys[s] + (sb - s_roff[s]);
            if (dest >= 0 && dest < ycap) dst = P.base[s] + P.off_yrecv + static_cast<size_t>(dest) * row_bytes;
        }
        row_out[r] = dst;
    }
}

__global__ void ep_signal_wait_kernel(const EpPeers P, int phase, const uint32_t* __restrict__ epoch_dev,
                                      int* __restrict__ error_word) {
    if (threadIdx.x == 0 && !signal_and_wait(P, phase, *epoch_dev) && error_word) atomicExch(error_word, 3);
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

moe_status_t moe_ep_remap_experts(const int32_t* topk_idx, int num_pairs, int E, const int32_t* slot_of_expert,
                                  int32_t* vidx, cwStream_t stream) {
    if (num_pairs < 0 || E <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (num_pairs == 0) return MOE_OK;
    if (!topk_idx || !slot_of_expert || !vidx) return MOE_ERR_INVALID_ARGUMENT;
    int blocks = (num_pairs + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    ep_remap_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(topk_idx, num_pairs, E, slot_of_expert, vidx);
    return launch_status();
}

moe_status_t moe_ep_token_rows(const int32_t* vidx, int T, int k, int ep_size, int experts_per_rank, int32_t* uidx,
                               int32_t* utok, int32_t* ucount, cwStream_t stream) {
    if (T < 0 || k <= 0 || ep_size <= 0 || ep_size > kMaxEpRanks || experts_per_rank <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (!ucount || (T > 0 && (!vidx || !uidx || !utok))) return MOE_ERR_INVALID_ARGUMENT;
    ep_unique_kernel<<<1, kUniqueThreads, 0, static_cast<cudaStream_t>(stream)>>>(vidx, T, k, ep_size,
                                                                                 experts_per_rank, uidx, utok, ucount);
    return launch_status();
}

moe_status_t moe_ep_pack_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                                 const int32_t* row_token, const int32_t* num_rows, int row_capacity, int H,
                                 void* packed, cwStream_t stream) {
    const size_t rb = moe_ep_row_bytes(H) + (xq_lo ? static_cast<size_t>(H) : 0);
    if (H <= 0 || H % 128 || !xq || !xs || !row_token || !num_rows || !packed || row_capacity < 0)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(xq) || !aligned16(packed) || (xq_lo && !aligned16(xq_lo))) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    ep_pack_rows_kernel<<<grid_for_rows(row_capacity), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(xq), xs, xs_ld, row_token, num_rows, row_capacity, H,
        static_cast<uint8_t*>(packed), rb, static_cast<const uint8_t*>(xq_lo));
    return launch_status();
}

moe_status_t moe_ep_pack_rows(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                              const int32_t* num_rows, int row_capacity, int H, void* packed, cwStream_t stream) {
    return moe_ep_pack_rows_x2(xq, nullptr, xs, xs_ld, row_token, num_rows, row_capacity, H, packed, stream);
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

moe_status_t moe_ep_gather_x2(const void* packed, const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                              const int32_t* row_src, const int32_t* total_rows, int row_capacity, int H, void* xp,
                              void* xp_lo, float* xps, int xps_ld, cwStream_t stream) {
    const size_t rb = moe_ep_row_bytes(H) + (xp_lo ? static_cast<size_t>(H) : 0);
    if (H <= 0 || H % 128 || !packed || !xq || !xs || !row_src || !total_rows || !xp || !xps || row_capacity < 0 ||
        xps_ld < row_capacity)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!xq_lo != !xp_lo) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(packed) || !aligned16(xq) || !aligned16(xp) || (xp_lo && (!aligned16(xp_lo) || !aligned16(xq_lo))))
        return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    ep_gather_kernel<<<grid_for_rows(row_capacity), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(packed), rb, static_cast<const uint8_t*>(xq), xs, xs_ld, row_src, total_rows,
        row_capacity, H, static_cast<uint8_t*>(xp), xps, xps_ld, static_cast<const uint8_t*>(xq_lo),
        static_cast<uint8_t*>(xp_lo));
    return launch_status();
}

moe_status_t moe_ep_gather(const void* packed, const void* xq, const float* xs, int xs_ld, const int32_t* row_src,
                           const int32_t* total_rows, int row_capacity, int H, void* xp, float* xps, int xps_ld,
                           cwStream_t stream) {
    return moe_ep_gather_x2(packed, xq, nullptr, xs, xs_ld, row_src, total_rows, row_capacity, H, xp, nullptr, xps,
                            xps_ld, stream);
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

namespace tbep {

namespace {

EpPeers to_dev(const Peers& P) {
    EpPeers d;
    std::memset(&d, 0, sizeof(d));
    for (int r = 0; r < P.ep && r < kMaxRanks; ++r) d.base[r] = static_cast<uint8_t*>(P.base[r]);
    d.ep = P.ep;
    d.me = P.me;
    d.E = P.E;
    d.epr = P.epr;
    d.off_flags = P.lay.off_flags;
    d.off_table = P.lay.off_table;
    d.off_recv = P.lay.off_recv;
    d.off_pmap = P.lay.off_pmap;
    d.off_yrecv = P.lay.off_yrecv;
    d.timeout_ns = P.timeout_ns;
    return d;
}

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

Layout layout(int ep, int E, int recv_cap, size_t row_bytes, size_t y_rows, int H) {
    Layout L;
    size_t o = 0;
    L.off_flags = o;
    o = up256(o + 3 * kMaxEpRanks * sizeof(uint32_t));
    L.off_table = o;
    o = up256(o + static_cast<size_t>(ep) * (E + ep) * sizeof(int32_t));
    L.off_recv = o;
    o = up256(o + static_cast<size_t>(recv_cap) * row_bytes);
    L.off_pmap = o;
    o = up256(o + static_cast<size_t>(recv_cap) * sizeof(int32_t));
    L.off_yrecv = o;
    o = up256(o + y_rows * static_cast<size_t>(H) * 2);
    L.bytes = o;
    return L;
}

moe_status_t unique_rows(const Peers& P, const int32_t* vid, int T, int K, int32_t* uidx, int32_t* utok,
                         int32_t* ucounts, cudaStream_t st) {
    return moe_ep_token_rows(vid, T, K, P.ep, P.epr, uidx, utok, ucounts, st);
}

moe_status_t counts(const Peers& P, const int32_t* ecounts, const int32_t* ucounts, uint32_t* epoch_dev,
                    int32_t* plan, int32_t* rcounts, int* error_word, cudaStream_t st) {
    // the counts of every source and this rank's own, staged in shared memory
    // (the opt-in is to the largest size once per device, so any layer fits)
    const size_t smem = (static_cast<size_t>(P.ep) * (P.E + P.ep) + P.E) * sizeof(int);
    if (smem > 227 * 1024) return MOE_ERR_UNSUPPORTED;
    static bool attr[kMaxDevices] = {};
    if (smem > 48 * 1024 && smem_optin_once(ep_counts_kernel, 227 * 1024, attr) != cudaSuccess) return MOE_ERR_CUDA;
    ep_counts_kernel<<<1, 256, smem, st>>>(to_dev(P), ecounts, ucounts, epoch_dev, plan, rcounts, error_word);
    return launch_status();
}

moe_status_t dispatch(const Peers& P, const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                      const int32_t* stok, const int32_t* uidx, const int32_t* utok, int T, const int32_t* plan, int H,
                      size_t row_bytes, int recv_cap, int max_rows, cudaStream_t st) {
    if (max_rows <= 0) return MOE_OK;
    ep_dispatch_kernel<<<grid_for_rows(max_rows), 256, 0, st>>>(to_dev(P), static_cast<const uint8_t*>(xq), xs,
                                                                 xs_ld, stok, uidx, utok, T, plan, H, row_bytes,
                                                                 recv_cap, static_cast<const uint8_t*>(xq_lo));
    return launch_status();
}

moe_status_t gather(const Peers& P, const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                    const int32_t* row_src, const int32_t* total_rows, int row_capacity, int H, size_t row_bytes,
                    int recv_cap, void* xp, void* xp_lo, float* xps, int xps_ld, cudaStream_t st) {
    if (row_capacity <= 0) return MOE_OK;
    const uint8_t* mine = static_cast<const uint8_t*>(P.base[P.me]);
    ep_gather_kernel<<<grid_for_rows(row_capacity), 256, 0, st>>>(
        mine + P.lay.off_recv, row_bytes, static_cast<const uint8_t*>(xq), xs, xs_ld, row_src, total_rows,
        row_capacity, H, static_cast<uint8_t*>(xp), xps, xps_ld, static_cast<const uint8_t*>(xq_lo),
        static_cast<uint8_t*>(xp_lo), reinterpret_cast<const int32_t*>(mine + P.lay.off_pmap), recv_cap);
    return launch_status();
}

moe_status_t signal_wait(const Peers& P, int phase, const uint32_t* epoch_dev, int* error_word, cudaStream_t st) {
    ep_signal_wait_kernel<<<1, 32, 0, st>>>(to_dev(P), phase, epoch_dev, error_word);
    return launch_status();
}

moe_status_t return_rows(const Peers& P, const int32_t* row_src, const int32_t* total_rows, const int32_t* plan,
                         int H, int y_cap, int row_capacity, void** row_out, cudaStream_t st) {
    if (row_capacity <= 0) return MOE_OK;
    int blocks = (row_capacity + 255) / 256;
    if (blocks > 148 * 4) blocks = 148 * 4;
    ep_return_rows_kernel<<<blocks, 256, 0, st>>>(to_dev(P), row_src, total_rows, plan, static_cast<size_t>(H) * 2,
                                                  y_cap, row_capacity, row_out);
    return launch_status();
}

moe_status_t combine_send(const Peers& P, const void* y_bf16, const int32_t* recv_dst, const int32_t* plan,
                          int H, int y_cap, int y_rows, int max_rows, cudaStream_t st) {
    if (max_rows <= 0) return MOE_OK;
    ep_combine_send_kernel<<<grid_for_rows(max_rows), 256, 0, st>>>(
        to_dev(P), static_cast<const uint8_t*>(y_bf16), recv_dst, plan, static_cast<size_t>(H) * 2, y_cap, y_rows);
    return launch_status();
}

}  // namespace tbep
