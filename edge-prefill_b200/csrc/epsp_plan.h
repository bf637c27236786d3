// epsp_plan.h -- block geometry of page gating, shared by host code and all
// kernels so that every part of the path agrees on it bit for bit.
//
// Restates the reference graph branch (patches/llama-prefill-attn-top-k.patch):
//   W = local_pages * P, or the block length when local_pages == 0   (:983-985)
//   start_row = max(0, N - n_tok - W), lsp = start_row / P            (:982-986)
//   gating engages only when n_pages > 0 && lsp > 0                  (:932)
//   n_local = P + N - lsp * P                                         (:987-988)
//   k_sel = min(sel, lsp) [reference], then the graph-width guard     (:990-993)
// generalised with the extended knobs (page size, per-KV-head lists with
// k_eff = min(k, lsp - 1), sub-blocks, an optional width guard), plus the
// pooled (compressed) rows of the qg_pool_pages budget (reserved at :578,
// row semantics of :1595-1715): the n_pool candidates ranked right after the
// selected pages each add one mean row, n_pool = min(pool_pages, candidates
// left after the selection).
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define EPSP_HD __host__ __device__ __forceinline__
#else
#define EPSP_HD inline
#endif

namespace epsp {

struct BlockPlan {
    int32_t b0, b1;   // query rows [b0, b1); visible KV rows [0, b1)
    int32_t lsp;      // local_start_page
    int32_t gated;    // page selection engaged
    int32_t k_sel;    // pages to select (0 when not gated)
    int32_t n_local;  // sink page + local window rows (gated)
    int32_t n_pool;   // pooled (page-mean) rows (gated, pool_pages > 0)
};

struct GateParams {
    int32_t page_size;
    int32_t local_pages;
    int32_t shared;           // 1: reference mode (one list, MAX over KV heads)
    int32_t max_gather_rows;  // 0: unlimited
    int32_t pool_pages = 0;   // pooled rows per gating block (0: off)
};

EPSP_HD BlockPlan plan_block(const GateParams& g, int32_t b0, int32_t b1, int32_t k_budget) {
    BlockPlan out;
    const int64_t P = g.page_size;
    const int64_t n_blk = (int64_t)b1 - b0;
    const int64_t N = b1;
    const int64_t W = g.local_pages > 0 ? (int64_t)g.local_pages * P : n_blk;
    int64_t start_row = N - n_blk - W;
    if (start_row < 0) start_row = 0;
    const int64_t lsp = start_row / P;
    const int64_t n_pages = N / P;
    out.b0 = b0;
    out.b1 = b1;
    out.lsp = (int32_t)lsp;
    out.gated = (k_budget >= 0 && n_pages > 0 && lsp > 0) ? 1 : 0;
    out.n_pool = 0;
    if (!out.gated) {
        out.k_sel = 0;
        out.n_local = (int32_t)N;
        return out;
    }
    const int64_t n_local = P + N - lsp * P;
    int64_t k = k_budget;
    if (g.shared) {
        if (k > lsp) k = lsp;
    } else {
        if (k > lsp - 1) k = lsp - 1;
    }
    if (g.max_gather_rows > 0) {
        const int64_t room = (int64_t)g.max_gather_rows - n_local;
        const int64_t cap = room < 0 ? 0 : room / P;
        if (k > cap) k = cap;
    }
    if (k < 0) k = 0;
    out.k_sel = (int32_t)k;
    out.n_local = (int32_t)n_local;
    if (g.pool_pages > 0) {
        const int64_t n_cand = lsp - 1;
        const int64_t left = n_cand - (k < n_cand ? k : n_cand);
        out.n_pool = (int32_t)(left < g.pool_pages ? left : g.pool_pages);
    }
    return out;
}

// Paged KV cache: logical row r of the sequence lives at physical row
// table[r / block_rows] * block_rows + r % block_rows of a pool of pool_rows
// rows ([pool_rows][Hkv][d]); block_rows is a multiple of the page size, so a
// page (and every kernel segment inside it) is contiguous.  block_rows == 0:
// the cache is contiguous (physical row = logical row).
struct KvPaging {
    const int32_t* table = nullptr;  // device, [n_entries]
    int32_t block_rows = 0;
    int32_t n_entries = 0;
    int32_t pool_rows = 0;
};

// Physical row of logical row r (block-aligned runs stay contiguous).  A
// table entry outside the pool sets `bad` and maps to row 0.
#if defined(__CUDACC__)
__device__ __forceinline__ int32_t phys_row(const KvPaging& pg, int32_t r, bool& bad) {
    if (pg.block_rows <= 0) return r;
    const int32_t i = r / pg.block_rows;
    if (i < 0 || i >= pg.n_entries) {
        bad = true;
        return 0;
    }
    const int64_t blk = __ldg(pg.table + i);
    const int64_t row = blk * pg.block_rows + r % pg.block_rows;
    if (blk < 0 || row >= pg.pool_rows) {
        bad = true;
        return 0;
    }
    return (int32_t)row;
}
#endif

// Gating block i of a ubatch covering rows [u0, u0 + n_tok): blocks of
// q_subblock rows (the last one shorter), or the whole ubatch when 0.
EPSP_HD int32_t block_len(int32_t n_tok, int32_t q_subblock) {
    return q_subblock > 0 && q_subblock < n_tok ? q_subblock : n_tok;
}
EPSP_HD int32_t n_blocks_of(int32_t n_tok, int32_t q_subblock) {
    const int32_t L = block_len(n_tok, q_subblock);
    return (n_tok + L - 1) / L;
}

}  // namespace epsp
