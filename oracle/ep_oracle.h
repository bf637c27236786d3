/*
 * ep_oracle.h -- CPU oracle for the page-gated sparse prefill attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * leg may load it.  The product (edge-prefill_b200/libepsp.so) never links,
 * loads or calls it.
 *
 * It restates, in plain C with fp64 arithmetic, what the reference's
 * llama.cpp patch computes for the AR006 "in-graph query-aware page gating"
 * branch (patches/llama-prefill-attn-top-k.patch):
 *   - the block geometry (local window, local_start_page, k_sel, the 4096-row
 *     graph-width guard):          patch :976-993, :754-792, :925-933
 *   - page scoring q . sum(K_page):  patch :1035-1055
 *   - the -inf bias on sink/local pages and top-k:  patch :763-766, :1057-1058
 *   - the local union gather + attention:  patch :1002-1016, :1060-1092
 *   - the ubatch partition (ChunkScheduler::plan): src/chunk_scheduler.cpp:9-45
 *   - FFN skip (skipped => FFN contributes zero, residual kept):
 *       patches/llama-prefill-ffn-skip.patch:146-149, generalised to rows
 *       (src/sparse_prefill.cpp:214-232 drops non-selected rows).
 *
 * Arithmetic contract shared with the CUDA kernels (ggml's own float order is
 * not available here, so parity with ggml is unpinned; parity with this
 * restatement is bit-exact for page indices):
 *   - page sums: fp64; the rows of each 16-row group are added in ascending
 *     order starting from 0.0, then the page's groups are added in ascending
 *     order starting from group 0's sum (the CUDA kernel sums the groups in
 *     parallel and combines them in this fixed order);
 *   - page score: channels in groups of 16; each group an fp64 fma chain in
 *     ascending channel order from 0.0 (acc = fma(q_c, S_c, acc)), the group
 *     partials added in ascending group order (the CUDA kernel scores a page
 *     with one thread per group and combines them in that order);
 *   - shared (reference) mode: score = max over KV heads (exact);
 *   - top-k order: score descending, ties -> lower page index; the returned
 *     list is sorted by page index ascending;
 *   - reference-mode off-by-one: when k_sel exceeds the lsp-1 selectable pages
 *     (patch :990-992 vs the bias at :765) the extra picks are -inf pages; the
 *     oracle takes the lowest -inf page ids, i.e. page 0 (the sink) first,
 *     which duplicates the sink rows in the gather exactly as a top-k that
 *     returns a -inf page does;
 *   - attention: fp64 scores and softmax over the kept multiset, causal.
 */
#ifndef EP_ORACLE_H
#define EP_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { EPO_F32 = 0, EPO_F16 = 1, EPO_BF16 = 2 };
enum { EPO_GROUP_ROWS = 16, EPO_GROUP_CH = 16 };

typedef struct epo_params {
    int32_t n_head;          /* query heads Hq */
    int32_t n_head_kv;       /* KV heads Hkv (Hq % Hkv == 0) */
    int32_t head_dim;        /* d */
    int32_t page_size;       /* P rows per page (reference: 32) */
    int32_t sel_pages;       /* default top-k budget (reference qg_sel_pages) */
    int32_t local_pages;     /* window W = local_pages*P rows; 0 => W = block length */
    int32_t shared;          /* 1: reference mode (MAX over KV heads, one list) */
    int32_t q_subblock;      /* 0: one gating block per ubatch; else block rows */
    int32_t max_gather_rows; /* 0: unlimited; reference: 4096 (patch :993) */
    double kq_scale;         /* softmax scale; 0 => 1/sqrt(d) */
    int32_t pool_pages;      /* pooled (compressed) rows per block: 0 off (see epo_pool_block) */
    int32_t route_mode;      /* per-KV-head routing by score spread: 0 off, 1, 2 (epo_route_block) */
    double route_threshold;  /* spread below it: a streaming head */
} epo_params;

typedef struct epo_block_plan {
    int32_t b0, b1;          /* query rows [b0,b1); KV rows visible: [0,b1) */
    int32_t lsp;             /* local_start_page */
    int32_t gated;           /* 1 when page selection engages */
    int32_t k_sel;           /* pages selected (0 when !gated) */
    int32_t n_local;         /* rows in sink page + local window (gated) */
} epo_block_plan;

/* Block geometry for query rows [b0,b1) with top-k budget k_budget
 * (k_budget < 0: dense head, never gated). */
void epo_plan_block(const epo_params* p, int32_t b0, int32_t b1, int32_t k_budget,
                    epo_block_plan* out);

/* ChunkScheduler::plan restated (src/chunk_scheduler.cpp:9-45).  Writes up to
 * cap [begin,end) pairs into ranges (2*cap ints).  Returns the number of
 * ranges, or -2 (InvalidArgument) for n_tokens == 0 / n_ubatch == 0 / null. */
int32_t epo_chunk_plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                       uint32_t* ranges, int32_t cap);

/* Number of gating blocks of a prefill of n_tokens (chunk plan x sub-blocks). */
int32_t epo_count_blocks(const epo_params* p, uint32_t n_tokens, uint32_t chunk_size,
                         uint32_t n_ubatch);

/* Fills blocks[2*i], blocks[2*i+1] = b0, b1 of every gating block. */
int32_t epo_list_blocks(const epo_params* p, uint32_t n_tokens, uint32_t chunk_size,
                        uint32_t n_ubatch, int32_t* blocks, int32_t cap);

/* fp64 page sums of full pages: out[h][page][c] for pages [0, n_rows/P). */
void epo_page_sums(const void* k, int32_t dtype, int32_t n_rows, int32_t n_head_kv,
                   int32_t head_dim, int32_t page_size, double* out);

/* Selection for one block.  q_last: the block's last query row [Hq][d].
 * psum: [Hkv][n_pages_stride][d].  head >= 0: per-KV-head selection for that
 * head; head < 0: shared mode.  Writes plan->k_sel pages sorted ascending
 * into out_pages; also writes the fp64 scores of pages 0..lsp-1 into
 * scores_out when non-null (score of page p at scores_out[p]).  Returns k_sel. */
int32_t epo_select_block(const epo_params* p, const epo_block_plan* plan,
                         const void* q_last, int32_t dtype, const double* psum,
                         int32_t n_pages_stride, int32_t head, int32_t* out_pages,
                         double* scores_out);

/* Pooled ("compressed") pages of one block -- the qg_pool_pages budget the
 * reference reserves (patch :578) with the AR004 pooled-row semantics (patch
 * :1595-1715: a page that is not gathered contributes one row, the mean of its
 * K rows and of its V rows, causally gated by the page's last position).
 * Here the pooled pages are the next p->pool_pages candidates after the
 * block's top-k in the same rank order (score descending, ties -> lower page),
 * i.e. ranks [min(k_sel, lsp-1), min(k_sel, lsp-1) + pool_pages) of pages
 * 1..lsp-1; written ascending into out_pages.  Returns their number.  Every
 * such page ends before the block's first row, so its row is visible to every
 * query of the block. */
int32_t epo_pool_block(const epo_params* p, const epo_block_plan* plan,
                       const void* q_last, int32_t dtype, const double* psum,
                       int32_t n_pages_stride, int32_t head, int32_t* out_pages);

/* Per-KV-head routing of one block by the live page-score spread, the
 * head-routing design of AR006 (specs/archive/AR006-in-graph-query-aware-
 * sparse-prefill/design.md:139-146): with u_h(p) = score_h(p) / page_size (the
 * page-mean score) over the candidates p = 1..lsp-1,
 *   spread_h = (max_p u_h - mean_p u_h) / (|mean_p u_h| + EPO_ROUTE_EPS),
 * the mean's sum taken in ascending page order in fp64 from 0.0, then divided
 * by the candidate count.  A head with spread_h < p->route_threshold is a
 * streaming head: it selects no page (sink + local window only).  Mode 1
 * leaves the other (retrieval) heads' budgets as they are; mode 2 hands the
 * pages the streaming heads gave up to the retrieval heads of the block in
 * equal shares (the remainder one page each to the lowest-index retrieval
 * heads), each capped at the block's candidate count.  k_in[h]: the budgets
 * after the block plan (epo_block_plan.k_sel per head); k_out[h]: the
 * effective budgets; spread_out (nullable) the spreads.  Heads with no
 * candidate keep k_in. */
#define EPO_ROUTE_EPS 1e-6
void epo_route_block(const epo_params* p, const epo_block_plan* plan, const void* q_last, int32_t dtype,
                     const double* psum, int32_t n_pages_stride, const int32_t* k_in, int32_t* k_out,
                     double* spread_out);

/* A pooled row's element: the fp64 page sum / page_size, rounded to f32, then
 * to the cache type (f16/bf16 round to nearest even; f32 unchanged) and read
 * back as a number -- ggml's f32 average pool followed by the cast back to the
 * cache type (patch :1667-1676). */
double epo_pool_elem(double page_sum, int32_t page_size, int32_t dtype);

/* The whole gated prefill of ONE layer, restating the chunk loop
 * (src/sparse_prefill.cpp:352-487) with the graph branch per ubatch.
 *   q [n_tokens][Hq][d], k, v [n_tokens][Hkv][d] in dtype;
 *   k_budget: per-KV-head top-k for this layer ([Hkv], -1 dense) or NULL
 *             to use p->sel_pages for every head;
 *   out: [n_tokens][Hq][d] fp64, or NULL to skip attention;
 *   rows / n_rows: subset of query rows to compute (NULL: all rows);
 *   sel_out: [n_blocks][Hkv][sel_cap] selected pages (sorted ascending; in
 *            shared mode every head row holds the shared list), sel_count:
 *            [n_blocks][Hkv]; both nullable.
 * Returns the number of blocks, or a negative error. */
int32_t epo_prefill_layer(const epo_params* p, const int32_t* k_budget,
                          const void* q, const void* k, const void* v, int32_t dtype,
                          uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                          double* out, const int32_t* rows, int32_t n_rows,
                          int32_t* sel_out, int32_t* sel_count, int32_t sel_cap,
                          int32_t n_threads);

/* epo_prefill_layer plus the pooled pages of every block and KV head
 * (pool_out [n_blocks][Hkv][pool_cap], pool_count [n_blocks][Hkv]; both
 * nullable); with p->pool_pages > 0 the attention also sees one pooled row
 * per pooled page (epo_pool_block, epo_pool_elem). */
int32_t epo_prefill_layer_ex(const epo_params* p, const int32_t* k_budget,
                             const void* q, const void* k, const void* v, int32_t dtype,
                             uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                             double* out, const int32_t* rows, int32_t n_rows,
                             int32_t* sel_out, int32_t* sel_count, int32_t sel_cap,
                             int32_t* pool_out, int32_t* pool_count, int32_t pool_cap,
                             int32_t n_threads);

/* FFN-skip compaction: rows with keep[r] != 0 are copied, in row order, into
 * x_kept; row_ids[i] = source row of kept row i.  layer_skipped != 0 means the
 * layer's FFN is skipped entirely (reference per-layer mask): nothing is kept.
 * Returns n_keep. */
int32_t epo_ffn_compact(const void* x, int32_t elem_bytes, const uint8_t* keep,
                        int32_t n_rows, int32_t hidden, int32_t layer_skipped,
                        void* x_kept, int32_t* row_ids);

/* Scatter-add: residual[row_ids[i]] = round(float(residual) + float(ffn_out[i]))
 * in fp32 with round-to-nearest-even into dtype; rows not listed untouched. */
void epo_ffn_scatter(const void* ffn_out, void* residual, int32_t dtype,
                     const int32_t* row_ids, int32_t n_keep, int32_t hidden);

/* Conversions used by the contract (exposed for tests). */
float epo_f16_to_f32(uint16_t h);
float epo_bf16_to_f32(uint16_t h);
uint16_t epo_f32_to_f16(float f);
uint16_t epo_f32_to_bf16(float f);

#ifdef __cplusplus
}
#endif
#endif
