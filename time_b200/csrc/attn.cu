// attn.cu -- paged-KV decode attention block for sm_100a (one new token per
// sequence), the tensor-parallel attention half of the GLM-4.x decoder layer:
//
//   partial RoPE + bf16 page write   attn_rope_kv_write
//   split-context flash decode       attn_decode_paged   (split kernel + merge)
//   TP sum of o_proj partials        attn_tp_reduce_residual
//
// Reference semantics: decode attention kernels.fut:245-279 (softmax over
// positions 0..len-1 of q.k * scale, times V), GQA head mapping
// kernels.cu:331 (kv head = q head / (nq / nkv)), KV page layout
// [page][slot][kv_head][d] kernels.cu:394-410, rotate-half RoPE
// kernels.cu:87-108 restricted to the first `rot` dims with
// inv_freq_i = theta^(-2i/rot) (the new-build partial-RoPE semantics).
//
// The decode kernel is HBM-bound (every K/V byte of every sequence is read
// once per step): one CTA per (context split, sequence x kv head), four warps
// each streaming their own 16-token pages through a cp.async ring into
// padded shared-memory rows, the 16 (padded) query heads of the GQA group x
// 16 tokens score tile and the P.V update on mma.sync bf16 tensor cores with
// an fp32 online softmax (log2 domain), then a shared-memory merge of the
// warps and one unnormalised partial per split.  A merge kernel combines the
// splits, normalises, writes bf16 and (optionally) the e4m3 1x128
// quantisation the o_proj GEMM reads.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cfloat>
#include <cmath>
#include <cstdint>

#include "attn_block.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int kD = 128;            // head_dim (the kernels are specialised)
constexpr int kPage = 16;          // tokens per KV page
constexpr int kRowPad = kD + 8;    // bf16 elements per shared row (272 B: conflict-free ldmatrix)
constexpr int kGPad = 16;          // query rows of one GQA group, padded to the MMA M
constexpr int kWarps = 4;
constexpr int kNst = 3;            // pages in flight per warp
constexpr float kLog2e = 1.4426950408889634f;

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

// ---------------------------------------------------------------- RoPE + page write

// Page-table row of row b: row_seq[b] when the rows are tokens of several
// sequences (prefill chunks, slot-indexed batches), else b; -1 when outside
// [0, num_seqs).
__device__ __forceinline__ int seq_of_row(const int32_t* row_seq, int b, int num_seqs) {
    const int s = row_seq ? row_seq[b] : b;
    return (s >= 0 && s < num_seqs) ? s : -1;
}

// One 64-thread block per (token, head): heads 0..nq-1 are queries, the next
// nkv keys (both rotated on their first `rot` dims, pairs i, i + rot/2), the
// last nkv values (copied); k and v go to the token's page slot.
__global__ void __launch_bounds__(64)
rope_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, int nq, int nkv, int rot,
                     const float* __restrict__ inv_freq, const int32_t* __restrict__ positions,
                     const int32_t* __restrict__ row_seq, int num_seqs,
                     const int32_t* __restrict__ page_table, int max_pages, int num_cache_pages,
                     __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                     __nv_bfloat16* __restrict__ v_cache, int32_t* __restrict__ seq_lens_out,
                     int* __restrict__ error_word) {
    const int b = blockIdx.x, h = blockIdx.y;
    const int pos = positions[b];
    const int pidx = pos / kPage;
    const int seq = seq_of_row(row_seq, b, num_seqs);
    if (h == 0 && threadIdx.x == 0 && seq_lens_out) seq_lens_out[b] = (pos >= 0 && seq >= 0) ? pos + 1 : 0;
    if (seq < 0) {
        if (h == 0 && threadIdx.x == 0 && error_word) atomicExch(error_word, 7);
        return;
    }
    if (pos < 0 || pidx >= max_pages) {
        if (h == 0 && threadIdx.x == 0 && error_word) atomicExch(error_word, 4);
        return;
    }
    const int phys = page_table[static_cast<size_t>(seq) * max_pages + pidx];
    if (phys < 0 || phys >= num_cache_pages) {
        if (h == 0 && threadIdx.x == 0 && error_word) atomicExch(error_word, 6);
        return;
    }
    const int slot = pos % kPage;
    const __nv_bfloat16* src = qkv + static_cast<size_t>(b) * (nq + 2 * nkv) * kD + static_cast<size_t>(h) * kD;
    __nv_bfloat16* dst;
    if (h < nq) dst = q_out + (static_cast<size_t>(b) * nq + h) * kD;
    else if (h < nq + nkv) dst = k_cache + ((static_cast<size_t>(phys) * kPage + slot) * nkv + (h - nq)) * kD;
    else dst = v_cache + ((static_cast<size_t>(phys) * kPage + slot) * nkv + (h - nq - nkv)) * kD;
    const int half = (h < nq + nkv) ? rot / 2 : 0;   // values are not rotated
    for (int i = threadIdx.x; i < kD; i += blockDim.x) {
        if (i < half) {
            const float ang = static_cast<float>(pos) * inv_freq[i];
            float sn, cs;
            sincosf(ang, &sn, &cs);
            const float x0 = __bfloat162float(src[i]), x1 = __bfloat162float(src[i + half]);
            dst[i] = __float2bfloat16_rn(x0 * cs - x1 * sn);
            dst[i + half] = __float2bfloat16_rn(x0 * sn + x1 * cs);
        } else if (i >= 2 * half) {
            dst[i] = src[i];
        }
    }
}

// ---------------------------------------------------------------- mma.sync helpers

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// D = A (16x16 bf16, row) * B (16x8 bf16, col) + D, fp32 accumulate
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------- split decode

struct DecodeParams {
    const __nv_bfloat16* q;        // [B][nq][128]
    const __nv_bfloat16* k_cache;  // [pages][16][nkv][128]
    const __nv_bfloat16* v_cache;
    const int32_t* page_table;     // [num_seqs][max_pages]
    const int32_t* row_seq;        // [B] page-table row of each row, or null (row b -> b)
    const int32_t* seq_lens;       // [B]
    float* part_o;                 // [B*nkv][max_splits][G][128]
    float* part_ml;                // [B*nkv][max_splits][G][2]  (max in log2 units, sum)
    int* error_word;
    int nq, nkv, G, max_pages, num_cache_pages, split_tokens, max_splits, num_seqs;
    int first_row;                 // rows below it belong to the prefill kernel
    float scale_log2;              // softmax scale * log2(e)
};

// Row b continues row a: the same sequence, one position later (seq_lens
// holds position + 1, 0 for a row the page write skipped).
__device__ __forceinline__ bool row_follows(const int32_t* row_seq, const int32_t* lens, int num_seqs, int a, int b) {
    const int sa = seq_of_row(row_seq, a, num_seqs), sb = seq_of_row(row_seq, b, num_seqs);
    return sa >= 0 && sa == sb && lens[a] > 0 && lens[b] == lens[a] + 1;
}

// Tokens attended for sequence b: its length, cut to what the page table and
// the split partials can hold (a longer one records error 5).
__device__ __forceinline__ int clamp_len(int len, int max_pages, int split_tokens, int max_splits) {
    const long long cap = min(static_cast<long long>(max_pages) * kPage, static_cast<long long>(max_splits) * split_tokens);
    return len < 0 ? 0 : (len > cap ? static_cast<int>(cap) : len);
}

constexpr int kWarpRing = kNst * 2 * kPage * kRowPad;   // bf16 elements of one warp's K/V ring
constexpr int kQElems = kGPad * kRowPad;
constexpr int kMaxSplitPages = 512;                     // split_tokens <= 8192
constexpr size_t kDecodeSmem = (static_cast<size_t>(kWarps) * kWarpRing + kQElems) * 2 + kMaxSplitPages * 4;
// the warp merge reuses the rings: per warp 16 x 128 fp32 O + 16 (m, l)
static_assert(kWarps * (kGPad * kD + 2 * kGPad) * 4 <= kWarps * kWarpRing * 2, "merge scratch fits the rings");

__global__ void __launch_bounds__(kWarps * 32, 2)
decode_split_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) __nv_bfloat16 sm[];
    const int split = blockIdx.x;
    const int bk = blockIdx.y;                 // b * nkv + kv head
    const int b = bk / p.nkv, kvh = bk % p.nkv;
    const int seq = seq_of_row(p.row_seq, b, p.num_seqs);
    if (seq < 0) return;                       // recorded (7) by the page write; the merge writes zeros
    if (b < p.first_row) return;               // a prefill row
    const int len_in = p.seq_lens[b];
    const int len = clamp_len(len_in, p.max_pages, p.split_tokens, p.max_splits);
    if (len != len_in && split == 0 && threadIdx.x == 0 && kvh == 0 && p.error_word) atomicExch(p.error_word, 5);
    const int t0 = split * p.split_tokens;
    if (t0 >= len) return;                     // this sequence has fewer splits
    const int t1 = min(t0 + p.split_tokens, len);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;

    __nv_bfloat16* q_s = sm + kWarps * kWarpRing;
    __nv_bfloat16* ring = sm + warp * kWarpRing;   // [kNst][K 16 rows | V 16 rows][kRowPad]
    int* pid_s = reinterpret_cast<int*>(q_s + kQElems);   // physical page of each page of the split
    const int page0 = t0 / kPage;
    const int npages = (t1 - 1) / kPage - page0 + 1;
    {
        const int32_t* ptb = p.page_table + static_cast<size_t>(seq) * p.max_pages + page0;
        for (int i = threadIdx.x; i < npages; i += blockDim.x) {
            const int phys = ptb[i];
            // a page id outside the cache reads nothing (zeros) and records error 6
            if ((phys < 0 || phys >= p.num_cache_pages) && p.error_word) atomicExch(p.error_word, 6);
            pid_s[i] = (phys < 0 || phys >= p.num_cache_pages) ? -1 : phys;
        }
    }

    // query rows of the group (rows >= G are zero)
    for (int c = threadIdx.x; c < kGPad * (kD / 8); c += blockDim.x) {
        const int r = c / (kD / 8), q8 = c % (kD / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < p.G)
            v = *reinterpret_cast<const uint4*>(p.q + (static_cast<size_t>(b) * p.nq + kvh * p.G + r) * kD + q8 * 8);
        *reinterpret_cast<uint4*>(q_s + r * kRowPad + q8 * 8) = v;
    }
    __syncthreads();
    uint32_t qa[kD / 16][4];
    {
        const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks)
            ldsm_x4(smem_u32(q_s + rr * kRowPad + ks * 16 + 8 * (mi >> 1)), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    }

    const int my_pages = npages > warp ? (npages - warp + kWarps - 1) / kWarps : 0;
    const size_t row_stride = static_cast<size_t>(p.nkv) * kD;   // elements between two slots of a page

    auto load_page = [&](int i, int stage) {
        int phys = pid_s[warp + i * kWarps];
        const uint32_t nbytes = phys >= 0 ? 16u : 0u;
        phys = phys >= 0 ? phys : 0;
        const __nv_bfloat16* kp = p.k_cache + static_cast<size_t>(phys) * kPage * row_stride + kvh * kD;
        const __nv_bfloat16* vp = p.v_cache + static_cast<size_t>(phys) * kPage * row_stride + kvh * kD;
        __nv_bfloat16* dst = ring + stage * 2 * kPage * kRowPad;
        // 2 x 16 rows x 16 chunks of 16 B
#pragma unroll
        for (int c = lane; c < 2 * kPage * (kD / 8); c += 32) {
            const int which = c / (kPage * (kD / 8));
            const int r = (c / (kD / 8)) % kPage, q8 = c % (kD / 8);
            const __nv_bfloat16* src = (which ? vp : kp) + r * row_stride + q8 * 8;
            cp_async16(dst + (which * kPage + r) * kRowPad + q8 * 8, src, nbytes);
        }
    };

    float o[kD / 8][4];
#pragma unroll
    for (int i = 0; i < kD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};

#pragma unroll
    for (int s = 0; s < kNst - 1; ++s) {
        if (s < my_pages) load_page(s, s);
        cp_async_commit();
    }
    for (int i = 0; i < my_pages; ++i) {
        cp_async_wait<kNst - 2>();
        __syncwarp();
        if (i + kNst - 1 < my_pages) load_page(i + kNst - 1, (i + kNst - 1) % kNst);
        cp_async_commit();
        const __nv_bfloat16* ks_ = ring + (i % kNst) * 2 * kPage * kRowPad;
        const __nv_bfloat16* vs_ = ks_ + kPage * kRowPad;
        // S = Q K^T: two 8-token tiles
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        {
            const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi >> 1), cofs = 8 * (mi & 1);
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(ks_ + rr * kRowPad + ks * 16 + cofs), b0, b1, b2, b3);
                mma_bf16(s0, qa[ks], b0, b1);
                mma_bf16(s1, qa[ks], b2, b3);
            }
        }
        // scale, mask the tokens past the split, online softmax (rows g and g+8)
        const int tok = (page0 + warp + i * kWarps) * kPage;
        const int c0 = 2 * tq;
        float sv[2][4];   // [row half][tile0 c0, c0+1, tile1 c0, c0+1]
        sv[0][0] = s0[0]; sv[0][1] = s0[1]; sv[0][2] = s1[0]; sv[0][3] = s1[1];
        sv[1][0] = s0[2]; sv[1][1] = s0[3]; sv[1][2] = s1[2]; sv[1][3] = s1[3];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int t = tok + c0 + (j & 1) + 8 * (j >> 1);
                sv[h][j] = (t >= t0 && t < t1) ? sv[h][j] * p.scale_log2 : -INFINITY;
            }
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(fmaxf(sv[h][0], sv[h][1]), fmaxf(sv[h][2], sv[h][3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m_r[h], mx);
            // mn is finite: every page holds at least one token of the split
            alpha[h] = exp2f(m_r[h] - mn);
            m_r[h] = mn;
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sv[h][j] = exp2f(sv[h][j] - mn);
                rs += sv[h][j];
            }
            l_r[h] = l_r[h] * alpha[h] + rs;
        }
        if (alpha[0] != 1.0f || alpha[1] != 1.0f) {   // the running max moved
#pragma unroll
            for (int nd = 0; nd < kD / 8; ++nd) {
                o[nd][0] *= alpha[0]; o[nd][1] *= alpha[0];
                o[nd][2] *= alpha[1]; o[nd][3] *= alpha[1];
            }
        }
        // O += P V
        uint32_t pa[4];
        pa[0] = pack_bf16(sv[0][0], sv[0][1]);
        pa[1] = pack_bf16(sv[1][0], sv[1][1]);
        pa[2] = pack_bf16(sv[0][2], sv[0][3]);
        pa[3] = pack_bf16(sv[1][2], sv[1][3]);
        {
            const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1), cofs = 8 * (mi >> 1);
#pragma unroll
            for (int nd = 0; nd < kD / 8; nd += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_u32(vs_ + rr * kRowPad + nd * 8 + cofs), b0, b1, b2, b3);
                mma_bf16(o[nd], pa, b0, b1);
                mma_bf16(o[nd + 1], pa, b2, b3);
            }
        }
    }
    cp_async_wait<0>();
    // full row sums
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
    }
    __syncthreads();   // every warp is done with its ring: reuse as merge scratch
    float* mo = reinterpret_cast<float*>(sm);                       // [warp][16][128]
    float* mml = mo + kWarps * kGPad * kD;                          // [warp][16][2]
    {
        float* ow = mo + warp * kGPad * kD;
#pragma unroll
        for (int nd = 0; nd < kD / 8; ++nd) {
            const int col = nd * 8 + 2 * tq;
            *reinterpret_cast<float2*>(ow + g * kD + col) = make_float2(o[nd][0], o[nd][1]);
            *reinterpret_cast<float2*>(ow + (g + 8) * kD + col) = make_float2(o[nd][2], o[nd][3]);
        }
        if (tq == 0) {
            mml[(warp * kGPad + g) * 2 + 0] = m_r[0];
            mml[(warp * kGPad + g) * 2 + 1] = l_r[0];
            mml[(warp * kGPad + g + 8) * 2 + 0] = m_r[1];
            mml[(warp * kGPad + g + 8) * 2 + 1] = l_r[1];
        }
    }
    __syncthreads();
    const size_t base = (static_cast<size_t>(bk) * p.max_splits + split) * p.G;
    for (int r = 0; r < p.G; ++r) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mml[(w * kGPad + r) * 2]);
        float L = 0.0f, acc = 0.0f;
        const int d = threadIdx.x;   // 128 threads, one per dim
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float mw = mml[(w * kGPad + r) * 2];
            const float f = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
            L += mml[(w * kGPad + r) * 2 + 1] * f;
            acc += mo[(w * kGPad + r) * kD + d] * f;
        }
        p.part_o[(base + r) * kD + d] = acc;
        if (d == 0) {
            p.part_ml[(base + r) * 2 + 0] = M;
            p.part_ml[(base + r) * 2 + 1] = L;
        }
    }
}

// One block (128 threads = head_dim) per (sequence, query head): merge the
// splits, normalise, write bf16 and optionally the e4m3 row + its scale.
__global__ void __launch_bounds__(kD)
decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                    const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ row_seq, int num_seqs, int nq,
                    int nkv, int G, int max_pages, int split_tokens, int max_splits,
                    __nv_bfloat16* __restrict__ out, uint8_t* __restrict__ out_q, float* __restrict__ out_s,
                    int out_ld, int first_row) {
    const int b = blockIdx.x / nq, h = blockIdx.x % nq;
    if (b < first_row) return;                 // a prefill row
    const int kvh = h / G, r = h % G;
    const int d = threadIdx.x;
    const int len = seq_of_row(row_seq, b, num_seqs) < 0 ? 0 : clamp_len(seq_lens[b], max_pages, split_tokens, max_splits);
    const int ns = len > 0 ? (len + split_tokens - 1) / split_tokens : 0;
    const size_t bk = static_cast<size_t>(b) * nkv + kvh;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, part_ml[((bk * max_splits + s) * G + r) * 2]);
    float L = 0.0f, acc = 0.0f;
    for (int s = 0; s < ns; ++s) {
        const size_t i = (bk * max_splits + s) * G + r;
        const float f = exp2f(part_ml[i * 2] - M);
        L += part_ml[i * 2 + 1] * f;
        acc += part_o[i * kD + d] * f;
    }
    const float v = ns > 0 ? acc / L : 0.0f;
    out[(static_cast<size_t>(b) * nq + h) * kD + d] = __float2bfloat16_rn(v);
    if (out_q) {
        __shared__ float red[kD / 32];
        float a = fabsf(v);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o2));
        if ((d & 31) == 0) red[d >> 5] = a;
        __syncthreads();
        float amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        uint8_t qv = 0;
        if (amax > 0.0f) {
            const float inv = 448.0f / amax;
            qv = static_cast<uint8_t>(cvt_e4m3x2(v * inv, 0.0f) & 0xFFu);
        }
        out_q[static_cast<size_t>(b) * nq * kD + h * kD + d] = qv;
        if (d == 0) out_s[static_cast<size_t>(h) * out_ld + b] = amax > 0.0f ? amax / 448.0f : 0.0f;
    }
}

// ---------------------------------------------------------------- prefill rows
//
// The first rows of a call (prompt positions of prefill chunks) are attended
// by one CTA per (16-row block, kv head): a block's runs of consecutive
// positions of one sequence are taken one after the other, each run's
// (position, query head) rows -- up to 16 x 16 -- being the M rows of 16-row
// mma.sync tiles, one warp each, while every 16-token K/V page of the
// sequence up to the run's last position is staged once in shared memory for
// all of them (the decode kernel streams the prefix again for every row).
// Each row keeps one fp32 online softmax over the pages in order 0, 1, ...
// with the causal limit of its own position, and a page past that limit
// leaves it unchanged, so a row's result does not depend on which rows share
// its block or its call: prompts give the same bits whichever way they are
// packed into forwards.  The remaining rows (decode steps) stay with the split
// decode kernel.
constexpr int kPfRows = 16;                  // positions per CTA block
constexpr int kPfWarps = 16;                 // one 16-row tile of (position, head) rows each
constexpr int kPfNst = 4;                    // K/V pages in flight
constexpr size_t kPfSmem = (static_cast<size_t>(kPfRows) * kGPad * kRowPad + kPfNst * 2 * kPage * kRowPad) * 2;
static_assert(kPfWarps * 32 == 2 * kPage * (kD / 8), "one 16-byte chunk of a page per thread");

struct PrefillParams {
    const __nv_bfloat16* q;        // [B][nq][128]
    const __nv_bfloat16* k_cache;  // [pages][16][nkv][128]
    const __nv_bfloat16* v_cache;
    const int32_t* page_table;     // [num_seqs][max_pages]
    const int32_t* row_seq;        // [B]
    const int32_t* seq_lens;       // [B]: position + 1
    __nv_bfloat16* out;            // [B][nq][128]
    uint8_t* out_q;                // [B][nq * 128] e4m3 or null
    float* out_s;                  // [nq][out_ld]
    int* error_word;
    int B;                         // prefill rows: [0, B) of the call
    int nq, nkv, G, max_pages, num_cache_pages, num_seqs, out_ld;
    float scale_log2;
};

__global__ void __launch_bounds__(kPfWarps * 32, 1)
prefill_rows_kernel(const PrefillParams p) {
    extern __shared__ __align__(128) __nv_bfloat16 sm[];
    __nv_bfloat16* q_s = sm;                                   // [256][kRowPad]
    __nv_bfloat16* ring = sm + kPfRows * kGPad * kRowPad;      // [kPfNst][K 16 | V 16][kRowPad]
    const int blk0 = blockIdx.x * kPfRows, kvh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int rend = min(blk0 + kPfRows, p.B);
    const int cap = p.max_pages * kPage;
    const size_t row_stride = static_cast<size_t>(p.nkv) * kD;
    int r = blk0;
    while (r < rend) {
        if (seq_of_row(p.row_seq, r, p.num_seqs) < 0 || p.seq_lens[r] <= 0) {
            // a row the page write skipped (error 7 recorded there): zeros, as the decode merge writes
            for (int c = threadIdx.x; c < p.G * kD; c += blockDim.x) {
                const int head = kvh * p.G + c / kD, d = c % kD;
                p.out[(static_cast<size_t>(r) * p.nq + head) * kD + d] = __float2bfloat16_rn(0.0f);
                if (p.out_q) {
                    p.out_q[static_cast<size_t>(r) * p.nq * kD + head * kD + d] = 0;
                    if (d == 0) p.out_s[static_cast<size_t>(head) * p.out_ld + r] = 0.0f;
                }
            }
            ++r;
            continue;
        }
        int n = 1;
        while (r + n < rend && row_follows(p.row_seq, p.seq_lens, p.num_seqs, r + n - 1, r + n)) ++n;
        const int seq = seq_of_row(p.row_seq, r, p.num_seqs);
        const int last_in = p.seq_lens[r + n - 1];
        if (last_in > cap && threadIdx.x == 0 && kvh == 0 && p.error_word) atomicExch(p.error_word, 5);
        const int npages = (min(last_in, cap) + kPage - 1) / kPage;
        const int rows = n * p.G;                              // (position, head) rows, position-major
        const int ntiles = (rows + 15) / 16;
        __syncthreads();                                       // the previous run's shared memory is free
        for (int c = threadIdx.x; c < kPfRows * kGPad * (kD / 8); c += blockDim.x) {
            const int i = c / (kD / 8), q8 = c % (kD / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (i < rows)
                v = *reinterpret_cast<const uint4*>(
                    p.q + (static_cast<size_t>(r + i / p.G) * p.nq + kvh * p.G + i % p.G) * kD + q8 * 8);
            *reinterpret_cast<uint4*>(q_s + i * kRowPad + q8 * 8) = v;
        }
        // tokens each of this thread's two rows attends (padding rows: token 0 only, never stored)
        int len_r[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = warp * 16 + g + 8 * h;
            len_r[h] = i < rows ? min(p.seq_lens[r + i / p.G], cap) : 1;
        }
        auto load_page = [&](int pg, int stage) {
            int phys = p.page_table[static_cast<size_t>(seq) * p.max_pages + pg];
            const bool ok = phys >= 0 && phys < p.num_cache_pages;
            if (!ok && threadIdx.x == 0 && p.error_word) atomicExch(p.error_word, 6);
            phys = ok ? phys : 0;
            const int t = threadIdx.x, which = t >> 8, rr = (t >> 4) & 15, q8 = t & 15;
            const __nv_bfloat16* src =
                (which ? p.v_cache : p.k_cache) + (static_cast<size_t>(phys) * kPage + rr) * row_stride + kvh * kD + q8 * 8;
            cp_async16(ring + (static_cast<size_t>(stage) * 2 * kPage + which * kPage + rr) * kRowPad + q8 * 8, src,
                       ok ? 16u : 0u);
        };
#pragma unroll
        for (int st = 0; st < kPfNst - 1; ++st) {
            if (st < npages) load_page(st, st);
            cp_async_commit();
        }
        __syncthreads();                                       // q_s written
        uint32_t qa[kD / 16][4];
        {
            const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1);
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks)
                ldsm_x4(smem_u32(q_s + (warp * 16 + rr) * kRowPad + ks * 16 + 8 * (mi >> 1)), qa[ks][0], qa[ks][1],
                        qa[ks][2], qa[ks][3]);
        }
        float o[kD / 8][4];
#pragma unroll
        for (int i = 0; i < kD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
        float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
        const bool active = warp < ntiles;
        for (int i = 0; i < npages; ++i) {
            cp_async_wait<kPfNst - 2>();
            __syncthreads();                                   // page i landed; page i - 1's stage is free
            if (i + kPfNst - 1 < npages) load_page(i + kPfNst - 1, (i + kPfNst - 1) % kPfNst);
            cp_async_commit();
            if (!active) continue;
            const __nv_bfloat16* ks_ = ring + (i % kPfNst) * 2 * kPage * kRowPad;
            const __nv_bfloat16* vs_ = ks_ + kPage * kRowPad;
            float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
            {
                const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi >> 1), cofs = 8 * (mi & 1);
#pragma unroll
                for (int ks = 0; ks < kD / 16; ++ks) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(smem_u32(ks_ + rr * kRowPad + ks * 16 + cofs), b0, b1, b2, b3);
                    mma_bf16(s0, qa[ks], b0, b1);
                    mma_bf16(s1, qa[ks], b2, b3);
                }
            }
            const int tok = i * kPage;
            const int c0 = 2 * tq;
            float sv[2][4];
            sv[0][0] = s0[0]; sv[0][1] = s0[1]; sv[0][2] = s1[0]; sv[0][3] = s1[1];
            sv[1][0] = s0[2]; sv[1][1] = s0[3]; sv[1][2] = s1[2]; sv[1][3] = s1[3];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int t = tok + c0 + (j & 1) + 8 * (j >> 1);
                    sv[h][j] = t < len_r[h] ? sv[h][j] * p.scale_log2 : -INFINITY;
                }
            float alpha[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float mx = fmaxf(fmaxf(sv[h][0], sv[h][1]), fmaxf(sv[h][2], sv[h][3]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                // finite: page 0 holds token 0, which every row attends
                const float mn = fmaxf(m_r[h], mx);
                alpha[h] = exp2f(m_r[h] - mn);
                m_r[h] = mn;
                float rs = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sv[h][j] = exp2f(sv[h][j] - mn);
                    rs += sv[h][j];
                }
                l_r[h] = l_r[h] * alpha[h] + rs;
            }
            if (alpha[0] != 1.0f || alpha[1] != 1.0f) {
#pragma unroll
                for (int nd = 0; nd < kD / 8; ++nd) {
                    o[nd][0] *= alpha[0]; o[nd][1] *= alpha[0];
                    o[nd][2] *= alpha[1]; o[nd][3] *= alpha[1];
                }
            }
            uint32_t pa[4];
            pa[0] = pack_bf16(sv[0][0], sv[0][1]);
            pa[1] = pack_bf16(sv[1][0], sv[1][1]);
            pa[2] = pack_bf16(sv[0][2], sv[0][3]);
            pa[3] = pack_bf16(sv[1][2], sv[1][3]);
            {
                const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1), cofs = 8 * (mi >> 1);
#pragma unroll
                for (int nd = 0; nd < kD / 8; nd += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(smem_u32(vs_ + rr * kRowPad + nd * 8 + cofs), b0, b1, b2, b3);
                    mma_bf16(o[nd], pa, b0, b1);
                    mma_bf16(o[nd + 1], pa, b2, b3);
                }
            }
        }
        cp_async_wait<0>();
        if (active) {
            // normalise; bf16 rows and the e4m3 1x128 quantisation of each (position, head) row
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float l = l_r[h];
                l += __shfl_xor_sync(0xffffffffu, l, 1);
                l += __shfl_xor_sync(0xffffffffu, l, 2);
                float amax = 0.0f;
#pragma unroll
                for (int nd = 0; nd < kD / 8; ++nd) {
                    o[nd][2 * h] = o[nd][2 * h] / l;
                    o[nd][2 * h + 1] = o[nd][2 * h + 1] / l;
                    amax = fmaxf(amax, fmaxf(fabsf(o[nd][2 * h]), fabsf(o[nd][2 * h + 1])));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                const int i = warp * 16 + g + 8 * h;
                if (i >= rows) continue;
                const size_t row = static_cast<size_t>(r + i / p.G);
                const int head = kvh * p.G + i % p.G;
                __nv_bfloat16* orow = p.out + (row * p.nq + head) * kD;
                const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
#pragma unroll
                for (int nd = 0; nd < kD / 8; ++nd) {
                    const int col = nd * 8 + 2 * tq;
                    *reinterpret_cast<uint32_t*>(orow + col) = pack_bf16(o[nd][2 * h], o[nd][2 * h + 1]);
                    if (p.out_q) {
                        const uint16_t qv = amax > 0.0f ? cvt_e4m3x2(o[nd][2 * h] * inv, o[nd][2 * h + 1] * inv) : 0;
                        *reinterpret_cast<uint16_t*>(p.out_q + row * p.nq * kD + head * kD + col) = qv;
                    }
                }
                if (p.out_q && tq == 0) p.out_s[static_cast<size_t>(head) * p.out_ld + row] = amax > 0.0f ? amax / 448.0f : 0.0f;
            }
        }
        r += n;
    }
}

// ---------------------------------------------------------------- TP sum

// out[t][i] = bf16( residual[t][i] + sum_r partial_r[t][i] ), ranks summed in
// order 0..tp-1 in fp32 (the same bits on every rank).
__global__ void __launch_bounds__(256)
tp_reduce_kernel(const __nv_bfloat16* const* __restrict__ parts, int tp, const __nv_bfloat16* __restrict__ residual,
                 size_t n, __nv_bfloat16* __restrict__ out) {
    const size_t i8 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i8 >= n) return;
    float acc[8];
    {
        const uint4 rv = *reinterpret_cast<const uint4*>(residual + i8);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(rb[j]);
    }
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < tp; ++r) {
        const uint4 pv = *reinterpret_cast<const uint4*>(parts[r] + i8);
        const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&pv);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += __bfloat162float(pb[j]);
    }
    uint4 ov;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = __float2bfloat16_rn(acc[j] + s[j]);
    *reinterpret_cast<uint4*>(out + i8) = ov;
}

inline bool a16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

}  // namespace

extern "C" {

moe_status_t attn_rope_kv_write_rows(const void* qkv_bf16, int B, int nq, int nkv, int head_dim, int rot,
                                     const float* inv_freq, const int32_t* positions, const int32_t* row_seq,
                                     int num_seqs, const int32_t* page_table, int max_pages, int page_size,
                                     int num_cache_pages, void* q_out_bf16, void* k_cache, void* v_cache,
                                     int32_t* seq_lens_out, int* error_word, cwStream_t stream) {
    if (B < 0 || nq <= 0 || nkv <= 0 || nq % nkv || head_dim != kD || page_size != kPage) return MOE_ERR_INVALID_ARGUMENT;
    if (num_cache_pages <= 0 || num_seqs <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (rot < 0 || rot > kD || rot % 2 || max_pages <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (B == 0) return MOE_OK;
    if (!qkv_bf16 || (rot > 0 && !inv_freq) || !positions || !page_table || !q_out_bf16 || !k_cache || !v_cache)
        return MOE_ERR_INVALID_ARGUMENT;
    if (nq + 2 * nkv > 65535) return MOE_ERR_UNSUPPORTED;
    rope_kv_write_kernel<<<dim3(B, nq + 2 * nkv), 64, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(qkv_bf16), nq, nkv, rot, inv_freq, positions, row_seq, num_seqs, page_table,
        max_pages, num_cache_pages, static_cast<__nv_bfloat16*>(q_out_bf16), static_cast<__nv_bfloat16*>(k_cache),
        static_cast<__nv_bfloat16*>(v_cache), seq_lens_out, error_word);
    return launch_status();
}

moe_status_t attn_rope_kv_write(const void* qkv_bf16, int B, int nq, int nkv, int head_dim, int rot,
                                const float* inv_freq, const int32_t* positions, const int32_t* page_table,
                                int max_pages, int page_size, int num_cache_pages, void* q_out_bf16, void* k_cache,
                                void* v_cache, int32_t* seq_lens_out, int* error_word, cwStream_t stream) {
    return attn_rope_kv_write_rows(qkv_bf16, B, nq, nkv, head_dim, rot, inv_freq, positions, nullptr, B > 0 ? B : 1,
                                   page_table, max_pages, page_size, num_cache_pages, q_out_bf16, k_cache, v_cache,
                                   seq_lens_out, error_word, stream);
}

size_t attn_decode_workspace_bytes(int B, int nq, int max_splits) {
    if (B <= 0 || nq <= 0 || max_splits <= 0) return 0;
    return static_cast<size_t>(B) * nq * max_splits * (kD + 2) * sizeof(float);
}

}  // extern "C"

namespace {

// Split decode over the rows of a call; rows below first_row are left to the
// prefill kernel.
moe_status_t decode_rows(const void* q_bf16, const void* k_cache, const void* v_cache, int num_cache_pages,
                         const int32_t* page_table, int max_pages, const int32_t* row_seq, int num_seqs,
                         const int32_t* seq_lens, int B, int nq, int nkv, int head_dim, int page_size, float scale,
                         int split_tokens, int max_splits, void* workspace, size_t workspace_bytes, void* out_bf16,
                         void* out_q, float* out_s, int out_ld, int* error_word, cudaStream_t st, int first_row) {
    if (num_seqs <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (B < 0 || nq <= 0 || nkv <= 0 || nq % nkv || nq / nkv > kGPad || head_dim != kD || page_size != kPage)
        return MOE_ERR_INVALID_ARGUMENT;
    if (split_tokens <= 0 || split_tokens % kPage || split_tokens > kMaxSplitPages * kPage || max_splits <= 0 ||
        max_splits > 65535 || max_pages <= 0 ||
        num_cache_pages <= 0)
        return MOE_ERR_INVALID_ARGUMENT;
    if (static_cast<long long>(B) * nkv > 65535) return MOE_ERR_UNSUPPORTED;
    if (B == 0) return MOE_OK;
    if (!q_bf16 || !k_cache || !v_cache || !page_table || !seq_lens || !workspace || !out_bf16)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!a16(q_bf16) || !a16(k_cache) || !a16(v_cache) || !a16(workspace)) return MOE_ERR_INVALID_ARGUMENT;
    if (out_q && (!out_s || out_ld < B)) return MOE_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < attn_decode_workspace_bytes(B, nq, max_splits)) return MOE_ERR_WORKSPACE;
    static bool attr[kMaxDevices] = {};
    if (smem_optin_once(decode_split_kernel, static_cast<int>(kDecodeSmem), attr) != cudaSuccess) return MOE_ERR_CUDA;
    DecodeParams p;
    p.q = static_cast<const __nv_bfloat16*>(q_bf16);
    p.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
    p.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
    p.page_table = page_table;
    p.row_seq = row_seq;
    p.num_seqs = num_seqs;
    p.seq_lens = seq_lens;
    p.part_o = static_cast<float*>(workspace);
    p.part_ml = p.part_o + static_cast<size_t>(B) * nq * max_splits * kD;
    p.nq = nq;
    p.nkv = nkv;
    p.G = nq / nkv;
    p.max_pages = max_pages;
    p.num_cache_pages = num_cache_pages;
    p.error_word = error_word;
    p.split_tokens = split_tokens;
    p.max_splits = max_splits;
    p.scale_log2 = scale * kLog2e;
    p.first_row = first_row;
    if (first_row >= B) return MOE_OK;
    decode_split_kernel<<<dim3(max_splits, B * nkv), kWarps * 32, kDecodeSmem, st>>>(p);
    moe_status_t s = launch_status();
    if (s != MOE_OK) return s;
    decode_merge_kernel<<<B * nq, kD, 0, st>>>(p.part_o, p.part_ml, seq_lens, row_seq, num_seqs, nq, nkv, p.G,
                                              max_pages, split_tokens, max_splits,
                                              static_cast<__nv_bfloat16*>(out_bf16), static_cast<uint8_t*>(out_q),
                                              out_s, out_ld, first_row);
    return launch_status();
}

}  // namespace

extern "C" {

moe_status_t attn_decode_paged_rows(const void* q_bf16, const void* k_cache, const void* v_cache,
                                    int num_cache_pages, const int32_t* page_table, int max_pages,
                                    const int32_t* row_seq, int num_seqs, const int32_t* seq_lens, int B, int nq,
                                    int nkv, int head_dim, int page_size, float scale, int split_tokens,
                                    int max_splits, void* workspace, size_t workspace_bytes, void* out_bf16,
                                    void* out_q, float* out_s, int out_ld, int* error_word, cwStream_t stream) {
    return decode_rows(q_bf16, k_cache, v_cache, num_cache_pages, page_table, max_pages, row_seq, num_seqs, seq_lens,
                       B, nq, nkv, head_dim, page_size, scale, split_tokens, max_splits, workspace, workspace_bytes,
                       out_bf16, out_q, out_s, out_ld, error_word, static_cast<cudaStream_t>(stream), 0);
}

moe_status_t attn_paged_rows(const void* q_bf16, const void* k_cache, const void* v_cache, int num_cache_pages,
                             const int32_t* page_table, int max_pages, const int32_t* row_seq, int num_seqs,
                             const int32_t* seq_lens, int B, int num_prefill_rows, int nq, int nkv, int head_dim,
                             int page_size, float scale, int split_tokens, int max_splits, void* workspace,
                             size_t workspace_bytes, void* out_bf16, void* out_q, float* out_s, int out_ld,
                             int* error_word, cwStream_t stream) {
    if (num_prefill_rows < 0 || num_prefill_rows > B) return MOE_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    moe_status_t s = decode_rows(q_bf16, k_cache, v_cache, num_cache_pages, page_table, max_pages, row_seq, num_seqs,
                                 seq_lens, B, nq, nkv, head_dim, page_size, scale, split_tokens, max_splits, workspace,
                                 workspace_bytes, out_bf16, out_q, out_s, out_ld, error_word, st, num_prefill_rows);
    if (s != MOE_OK || num_prefill_rows == 0) return s;
    static bool attr[kMaxDevices] = {};
    if (smem_optin_once(prefill_rows_kernel, static_cast<int>(kPfSmem), attr) != cudaSuccess) return MOE_ERR_CUDA;
    PrefillParams p;
    p.q = static_cast<const __nv_bfloat16*>(q_bf16);
    p.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
    p.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
    p.page_table = page_table;
    p.row_seq = row_seq;
    p.seq_lens = seq_lens;
    p.out = static_cast<__nv_bfloat16*>(out_bf16);
    p.out_q = static_cast<uint8_t*>(out_q);
    p.out_s = out_s;
    p.error_word = error_word;
    p.B = num_prefill_rows;
    p.nq = nq;
    p.nkv = nkv;
    p.G = nq / nkv;
    p.max_pages = max_pages;
    p.num_cache_pages = num_cache_pages;
    p.num_seqs = num_seqs;
    p.out_ld = out_ld;
    p.scale_log2 = scale * kLog2e;
    prefill_rows_kernel<<<dim3((num_prefill_rows + kPfRows - 1) / kPfRows, nkv), kPfWarps * 32, kPfSmem, st>>>(p);
    return launch_status();
}

moe_status_t attn_decode_paged(const void* q_bf16, const void* k_cache, const void* v_cache, int num_cache_pages,
                               const int32_t* page_table, int max_pages, const int32_t* seq_lens, int B, int nq,
                               int nkv, int head_dim, int page_size, float scale, int split_tokens, int max_splits,
                               void* workspace, size_t workspace_bytes, void* out_bf16, void* out_q, float* out_s,
                               int out_ld, int* error_word, cwStream_t stream) {
    return attn_decode_paged_rows(q_bf16, k_cache, v_cache, num_cache_pages, page_table, max_pages, nullptr,
                                  B > 0 ? B : 1, seq_lens, B, nq, nkv, head_dim, page_size, scale, split_tokens,
                                  max_splits, workspace, workspace_bytes, out_bf16, out_q, out_s, out_ld, error_word,
                                  stream);
}

moe_status_t attn_tp_reduce_residual(const void* const* partials_dev, int tp, const void* residual_bf16, int T, int H,
                                     void* out_bf16, cwStream_t stream) {
    if (tp <= 0 || T < 0 || H <= 0 || H % 8) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!partials_dev || !residual_bf16 || !out_bf16 || !a16(residual_bf16) || !a16(out_bf16))
        return MOE_ERR_INVALID_ARGUMENT;
    const size_t n = static_cast<size_t>(T) * H;
    const size_t threads = n / 8;
    const int blocks = static_cast<int>((threads + 255) / 256);
    tp_reduce_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const __nv_bfloat16* const*>(partials_dev), tp,
        static_cast<const __nv_bfloat16*>(residual_bf16), n, static_cast<__nv_bfloat16*>(out_bf16));
    return launch_status();
}

}  // extern "C"
