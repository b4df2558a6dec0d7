// moe_ep_peer.h -- internal interface between the layer (moe_layer.cu) and the
// peer-memory expert-parallel exchange kernels (moe_ep.cu).  Not part of the
// C-ABI.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "moe_layer.h"

namespace tbep {

constexpr int kMaxRanks = 64;

// Byte layout of one rank's symmetric exchange buffer (identical on every rank).
struct Layout {
    size_t off_flags, off_table, off_recv, off_pmap, off_yrecv, bytes;
};

Layout layout(int ep, int E, int recv_cap, size_t row_bytes, size_t y_rows, int H);

struct Peers {
    void* base[kMaxRanks];   // rank r's buffer as mapped in this process
    int ep, me, E, epr;
    Layout lay;
    unsigned long long timeout_ns;
};

// plan (device int32): 9 per rank + stot + rtot + utot
inline int plan_ints(int ep) { return 9 * ep + 3; }

// For every destination rank d, this rank's tokens with at least one pair
// routed there (vid: virtual expert per pair, -1 for none), in token order:
// uidx [ep][T] (-1 when none), utok [ep][T], ucounts [ep].
moe_status_t unique_rows(const Peers& P, const int32_t* vid, int T, int K, int32_t* uidx, int32_t* utok,
                         int32_t* ucounts, cudaStream_t st);
// epoch_dev: this rank's forward counter on the device (counts() increments it)
moe_status_t counts(const Peers& P, const int32_t* ecounts, const int32_t* ucounts, uint32_t* epoch_dev,
                    int32_t* plan, int32_t* rcounts, int* error_word, cudaStream_t st);
// one row per (destination, token with a pair there) into the destination's
// recv, and every sent pair's row index into its pmap
moe_status_t dispatch(const Peers& P, const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                      const int32_t* stok, const int32_t* uidx, const int32_t* utok, int T, const int32_t* plan, int H,
                      size_t row_bytes, int recv_cap, int max_rows, cudaStream_t st);
// moe_ep_gather_x2 over this rank's recv, each received pair read through pmap
moe_status_t gather(const Peers& P, const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                    const int32_t* row_src, const int32_t* total_rows, int row_capacity, int H, size_t row_bytes,
                    int recv_cap, void* xp, void* xp_lo, float* xps, int xps_ld, cudaStream_t st);
moe_status_t signal_wait(const Peers& P, int phase, const uint32_t* epoch_dev, int* error_word, cudaStream_t st);
// row_out[r] (r < *total_rows): where GEMM row r's down-projection output
// belongs -- a received row's slot in its owner's yrecv, nullptr for rows that
// stay local -- for cbwFp8BlockScaledGroupedGemmRowOut (replaces combine_send)
moe_status_t return_rows(const Peers& P, const int32_t* row_src, const int32_t* total_rows, const int32_t* plan,
                         int H, int y_cap, int row_capacity, void** row_out, cudaStream_t st);
moe_status_t combine_send(const Peers& P, const void* y_bf16, const int32_t* recv_dst, const int32_t* plan,
                          int H, int y_cap, int y_rows, int max_rows, cudaStream_t st);

enum Phase { kCounts = 0, kDispatch = 1, kCombine = 2 };

}  // namespace tbep
