/*
 * epsp.h -- C ABI of the B200 page-gated sparse prefill attention library
 * (libepsp.so).
 *
 * The library is a drop-in for EdgePrefill's AR006 "in-graph query-aware page
 * gating" path: the graph branch the reference adds to llama.cpp's
 * llm_graph_context::build_attn (patches/llama-prefill-attn-top-k.patch:963-1095)
 * and the extern "C" controls that arm it (patch :93-111 declarations, :403-437
 * implementation; patches/llama-prefill-ffn-skip.patch:9-21,65-92).  The
 * arithmetic runs in hand-written sm_100a kernels:
 *   K1 page sums of K (fp64), K2 page scoring + top-k page select,
 *   K3 sparse flash attention on tcgen05/TMEM with TMA page loads,
 *   K4 FFN-skip row compaction / scatter.
 *
 * Conventions (kept from the reference):
 *   - every entry point returns an int32 status with the numbering of
 *     edge_prefill::ErrorCode (include/edge_prefill/status.h:7-23):
 *     0 Ok, 2 InvalidArgument, 6 Prefill, 9 Unsupported, 10 OutOfMemory,
 *     12 Internal, 13 Unavailable; no C++ exception crosses this ABI;
 *   - getters return 0 on a null context (patch :439-444);
 *   - scalar setters copy, array setters copy the caller's array, so the
 *     caller keeps ownership (patch :189);
 *   - a context is single-threaded: setters run between compute calls on the
 *     caller's thread;
 *   - compute calls are stream-ordered on the caller's cudaStream_t (passed as
 *     void*), take caller-owned DEVICE pointers and never synchronise the host.
 *
 * Tensor layouts (row-major, ggml's ne[] order reversed, i.e. llama.cpp's own):
 *   q, out:   [n_tok][n_head][head_dim]        (the ubatch's query rows)
 *   k, v:     [kv_len][n_head_kv][head_dim]    (KV cache rows 0..kv_len-1 of the
 *                                               layer; v is NOT transposed)
 *   the ubatch's own rows are kv rows [kv_len - n_tok, kv_len).
 */
#ifndef EPSP_H
#define EPSP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: edge_prefill::ErrorCode (include/edge_prefill/status.h:7-23). */
#define EP_SP_OK 0
#define EP_SP_INVALID_ARGUMENT 2
#define EP_SP_PREFILL 6
#define EP_SP_UNSUPPORTED 9
#define EP_SP_OUT_OF_MEMORY 10
#define EP_SP_INTERNAL 12
#define EP_SP_UNAVAILABLE 13

/* Element types of Q/K/V/out and FFN rows. */
#define EP_SP_F32 0
#define EP_SP_F16 1
#define EP_SP_BF16 2

typedef struct ep_sp_ctx ep_sp_ctx;

/* Context configuration.  A context serves one model (n_layer layers) on one
 * device and owns the slice of KV heads [kv_head_offset, kv_head_offset +
 * n_head_kv) of a model with n_head_kv_total KV heads (head-parallel
 * sharding); the tensors passed to it hold only that slice. */
typedef struct ep_sp_config {
    int32_t n_layer;
    int32_t n_head;          /* query heads of this slice (n_head % n_head_kv == 0) */
    int32_t n_head_kv;       /* KV heads of this slice */
    int32_t head_dim;        /* 64 or 128 */
    int32_t dtype;           /* EP_SP_BF16 / EP_SP_F16 / EP_SP_F32 for q, k, v */
    int32_t out_dtype;       /* element type of the attention output */
    int32_t max_ctx;         /* maximum kv_len */
    int32_t page_size;       /* rows per page: 32 (the reference's), 64 or 128 */
    int32_t device;          /* CUDA device ordinal */
    int32_t kv_head_offset;  /* global index of this slice's first KV head */
    int32_t n_head_kv_total; /* KV heads of the whole model; 0 => n_head_kv */
    float kq_scale;          /* softmax scale; 0 => 1/sqrt(head_dim) */
} ep_sp_config;

/* Creates a context.  Validates the configuration (rc 2) and checks the device
 * (rc 13 when no CUDA device with that ordinal exists, rc 9 when it is not an
 * sm_100 part).  Device memory is reserved on the first compute call or by
 * ep_sp_reserve.  Replaces the reference's context setup for this path
 * (src/backend.cpp:154-194). */
int32_t ep_sp_create(const ep_sp_config* cfg, ep_sp_ctx** out);
int32_t ep_sp_reserve(ep_sp_ctx* ctx); /* rc 10 on allocation failure */
void ep_sp_destroy(ep_sp_ctx* ctx);

/* Arms / disarms page gating.  Identical validation and codes to
 * llama_set_prefill_qg_bound (patch :403-437): rc 2 for a null ctx, enabled not
 * 0/1, sel_pages outside [0,128], local_pages outside [0,1024] or pool_pages <
 * 0.  Arming clears every other sparse mode the context holds (none besides
 * this one here); disarming zeroes the budgets.  The local window is
 * local_pages * page_size rows (0 => the gating block's own length).
 * pool_pages (reserved but unused in the reference, patch :578) arms the
 * pooled "compressed" rows with the AR004 row semantics (patch :1595-1715):
 * per gating block (and KV head in per-KV-head mode) the pool_pages candidate
 * pages ranked right after the selected ones (same score order; fewer when
 * fewer candidates remain) each add ONE row to the kept set whose K and V are
 * the page's mean K and V rows (fp64 sums / page_size, rounded to f32 and then
 * to the cache type), visible to every query of the block (the page ends
 * before the block: the reference's max-position gate).  0 = off. */
int32_t ep_sp_set_qg_bound(ep_sp_ctx* ctx, int32_t enabled, int32_t sel_pages,
                           int32_t local_pages, int32_t pool_pages);
/* 1 when armed, 0 otherwise or for a null ctx (patch :439-444). */
int32_t ep_sp_get_qg_bound(const ep_sp_ctx* ctx);

/* Extended semantics beyond the reference's hard-coded ones (no reference
 * counterpart; defaults reproduce the reference):
 *   per_kv_head      0: one page list shared by all KV heads, scored by the MAX
 *                    over heads and with the reference's k_sel formula (patch
 *                    :990-992, :1053-1055); 1: one list per KV head,
 *                    k_eff = min(k, lsp-1).
 *   q_subblock       0: one gating block per ubatch (patch :1040-1041, query =
 *                    the ubatch's last row); > 0: blocks of that many rows,
 *                    each gated with its own last row.
 *   max_gather_rows  graph-width guard of patch :993 (reference: 4096);
 *                    0 = unlimited.
 * Returns rc 2 for a negative value or per_kv_head not 0/1.  Setting
 * per_kv_head = 0 clears the k-matrix. */
int32_t ep_sp_set_ext(ep_sp_ctx* ctx, int32_t per_kv_head, int32_t q_subblock,
                      int32_t max_gather_rows);

/* Per-(layer, KV head) top-k budgets for per-KV-head gating, n ==
 * n_layer * n_head_kv_total (row-major [layer][head]); -1 marks a dense head,
 * >= 1 a page budget.  n == 0 clears the matrix (every head uses sel_pages).
 * Same element rules as llama_set_prefill_attn_head_top_k (patch :237-262):
 * rc 2 for NULL with n > 0, a wrong length, an element 0 or < -1; also rc 2
 * when the context is in shared (per_kv_head = 0) mode.  Copied. */
int32_t ep_sp_set_k_matrix(ep_sp_ctx* ctx, const int32_t* k, size_t n);
int32_t ep_sp_get_k_matrix_size(const ep_sp_ctx* ctx);

/* Prefill mode and per-layer FFN skip (patches/llama-prefill-ffn-skip.patch
 * :9-21, :65-92).  Gating only engages in prefill mode.  The FFN mask keeps
 * bits < n_layer; n_layer >= 64 forces 0 (ffn patch :77-82). */
void ep_sp_set_prefill_mode(ep_sp_ctx* ctx, int32_t prefill);
int32_t ep_sp_get_prefill_mode(const ep_sp_ctx* ctx);
void ep_sp_set_ffn_skip(ep_sp_ctx* ctx, uint64_t layer_mask);
uint64_t ep_sp_get_ffn_skip(const ep_sp_ctx* ctx);

/* Forgets the pooled page sums (a new sequence starts at row 0).  A call with
 * kv_len == n_tok also restarts the sequence. */
int32_t ep_sp_reset(ep_sp_ctx* ctx);

/* Number of gating blocks a ubatch of n_tok rows is split into. */
int32_t ep_sp_query_blocks(const ep_sp_ctx* ctx, int32_t n_tok, int32_t* n_blocks);

/* One layer of one ubatch: the graph branch of patch :971-1095 followed by the
 * attention of :1092, replaced by K1 (pool the ubatch's completed pages), K2
 * (score + select per gating block), K3 (sparse attention over sink page +
 * selected pages + local window, causal).  With gating disarmed or not in
 * prefill mode the same kernel runs dense causal attention over [0, kv_len).
 *   q, out     [n_tok][n_head][head_dim]; k, v [kv_len][n_head_kv][head_dim];
 *   sel_pages  optional device output [n_blocks][n_head_kv][sel_cap]: the
 *              selected page ids of each gating block and KV head, ascending;
 *   sel_counts optional device output [n_blocks][n_head_kv];
 * rc 2 for bad sizes (n_tok < 1, kv_len < n_tok, kv_len > max_ctx, layer out
 * of range, sel_cap smaller than a block's k_sel), 12 on a CUDA launch error,
 * 6 when a device-side bounded wait expired (ep_sp_last_error says where). */
int32_t ep_sp_attend_layer(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k,
                           const void* v, int32_t kv_len, int32_t n_tok, void* out,
                           int32_t* sel_pages, int32_t* sel_counts, int32_t sel_cap,
                           void* stream);

/* The two halves of ep_sp_attend_layer, for callers that overlap the output
 * of one part of a call with the attention of the next part (for example a
 * head-parallel all-gather per group of gating blocks; no reference
 * counterpart):
 *   ep_sp_select_layer  K1 + K2 of the call (and the f16 shadows of an f32
 *                       context); the selection stays in the context (or in
 *                       sel_pages / sel_counts when given);
 *   ep_sp_attend_rows   K3 for the query rows [row_begin, row_end) of the same
 *                       call, which must cover whole gating blocks; out is the
 *                       call's whole [n_tok][n_head][head_dim] output.
 * ep_sp_attend_rows returns rc 2 unless the last ep_sp_select_layer of the
 * context was for the same (layer, kv_len, n_tok) and settings; q, k and v of
 * that call must stay valid until its rows are attended. */
int32_t ep_sp_select_layer(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v,
                           int32_t kv_len, int32_t n_tok, int32_t* sel_pages, int32_t* sel_counts, int32_t sel_cap,
                           void* stream);
int32_t ep_sp_attend_rows(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin,
                          int32_t row_end, void* out, void* stream);

/* Parts of one call's attention, for splitting a layer's work across GPUs
 * (no reference counterpart).  K3 runs a grid of CTAs that is head-major:
 * for KV head h (of this context) and gating block b, ctas_per_head =
 * n_blocks * ctas_per_block consecutive ids, id = h * ctas_per_head +
 * b * ctas_per_block + j, each CTA ep_sp_get_attn_tiles() query tiles of
 * 128 / G tokens.
 *   ep_sp_select_heads     K1 + K2 for the KV heads [head_begin, head_end)
 *                          only (per-KV-head selection; rc 9 with the shared
 *                          reference selection unless the range is every head);
 *   ep_sp_attend_ctas      K3 for the CTA ids [cta_begin, cta_end) of the
 *                          call (their KV heads must be inside the last
 *                          selection's head range), out as in attend_rows;
 *   ep_sp_attention_grid   ctas_per_head of a call of n_tok rows;
 *   ep_sp_balance_ctas     cuts[0..n_parts] (cuts[0] = 0, cuts[n_parts] =
 *                          n_head_kv * ctas_per_head) splitting the call's
 *                          grid into n_parts contiguous ranges of equal
 *                          estimated cost (the KV tiles each CTA walks under
 *                          the armed budgets, plus a fixed share per CTA that
 *                          includes the exchange epilogue to n_parts ranks,
 *                          smaller once a multicast address is attached with
 *                          ep_sp_xchg_attach_buffers: compute the cuts after
 *                          attaching).  Equal budgets give the plain
 *                          head-parallel split;
 *                          uneven per-head budgets move the cuts into the
 *                          neighbouring heads' blocks.  Deterministic: every
 *                          rank computes the same cuts. */
/* KV-cache append with fused page sums (no reference counterpart; it stands
 * in for llama.cpp's cpy_k / cpy_v of a ubatch's new rows followed by K1):
 * writes n_new rows of K and V ([n_new][n_head_kv][head_dim], context dtype)
 * into the caches at rows [kv_pos, kv_pos + n_new) and, in the same pass over
 * the new K rows, the page sums of every page those rows complete, with K1's
 * arithmetic (the sums are bit-identical).  After an append the context
 * trusts its page-sum watermarks for that layer, so ep_sp_select_layer /
 * ep_sp_attend_layer pool only pages no append has summed, until
 * ep_sp_reset.  rc 2 on bad arguments. */
int32_t ep_sp_append_kv(ep_sp_ctx* ctx, int32_t layer, const void* k_new, const void* v_new, int32_t n_new,
                        void* k_cache, void* v_cache, int32_t kv_pos, void* stream);

/* K3 variant: query tiles per CTA, 2 (default: one 384-thread CTA per SM
 * whose two tiles ping-pong on the tensor core) or 1 (two 256-thread CTAs per
 * SM, so one CTA computes while the other drains its output -- e.g. the
 * exchange's stores to the other GPUs).  The arithmetic, and therefore every
 * output bit, is the same; only the CTA grid of ep_sp_attention_grid /
 * ep_sp_balance_ctas / ep_sp_attend_ctas changes (a prepared selection is
 * dropped).  No reference counterpart.  rc 2 for other values. */
int32_t ep_sp_set_attn_tiles(ep_sp_ctx* ctx, int32_t tiles_per_cta);
int32_t ep_sp_get_attn_tiles(const ep_sp_ctx* ctx);

/* Paged KV cache: the KV-layout adapter for hosts whose cache is a pool of
 * fixed-size blocks addressed through a per-sequence block table (paged
 * attention caches; the reference attends llama.cpp's contiguous cells,
 * patch :999-1016).  After this call, the k / v (and k_cache / v_cache)
 * pointers of every compute call are POOLS of pool_rows rows
 * ([pool_rows][n_head_kv][head_dim]), and logical row r of the sequence lives
 * at pool row block_table[r / block_rows] * block_rows + r % block_rows.
 * block_table is a DEVICE array of n_entries int32 block ids that the caller
 * owns and may rewrite between calls (stream-ordered); it must cover kv_len
 * rows (rc 2 from the compute calls otherwise).  block_rows must be a multiple
 * of the page size (so every page is contiguous in the pool), pool_rows a
 * multiple of block_rows.  A table entry outside the pool is caught on the
 * device (no access is made through it; ep_sp_sync_status reports rc 6).
 * Rows a block holds past kv_len may contain anything (stale rows, NaN): the
 * attention masks their scores and zeroes their V rows on chip before they
 * reach the tensor cores.  block_rows = 0 returns to the contiguous layout.
 * The f16 tensor-core mode of f32 contexts needs the contiguous layout (rc 9).
 * rc 2 on bad arguments.  No reference counterpart. */
int32_t ep_sp_set_paged_kv(ep_sp_ctx* ctx, int32_t block_rows, const int32_t* block_table, int32_t n_entries,
                           int32_t pool_rows);

/* Per-KV-head routing by the live page-score spread: the head routing of
 * AR006 (specs/archive/AR006-in-graph-query-aware-sparse-prefill/design.md
 * :139-146, designed there but not built).  For each gating block and KV head,
 * over the candidate pages p = 1..lsp-1 with the page-mean score
 * u(p) = q . sum(K_p) / page_size,
 *   spread = (max_p u - mean_p u) / (|mean_p u| + 1e-6)
 * (the mean's sum taken in ascending page order in fp64).  A head with
 * spread < threshold is a streaming head: it selects no page and attends the
 * sink page and the local window only (plus its pooled rows when armed).
 *   mode 0  off (default);
 *   mode 1  retrieval heads keep their budgets;
 *   mode 2  the pages the streaming heads give up are re-split over the
 *           block's retrieval heads in equal shares (the remainder one page
 *           each to the lowest-index ones), each capped at the candidates --
 *           adaptive budgets, the block's total page count unchanged.
 * Routing needs per-KV-head selection (rc 9 from the compute calls in the
 * shared mode) and, in mode 2, every KV head of the context in one call
 * (<= 32 heads; rc 9 from ep_sp_select_heads on a part).  The routed counts
 * are what sel_counts reports and what the attention uses.  rc 2 for another
 * mode or a non-finite threshold.  No counterpart in the reference's code. */
int32_t ep_sp_set_head_routing(ep_sp_ctx* ctx, int32_t mode, double threshold);
int32_t ep_sp_get_head_routing(const ep_sp_ctx* ctx, int32_t* mode, double* threshold);

/* Pooled pages of the last ep_sp_select_layer / ep_sp_attend_layer call (no
 * reference counterpart; the reference exposes no page lists): device outputs
 * pages [n_blocks][n_head_kv][cap] (ascending) and counts [n_blocks][n_head_kv]
 * (all 0 when no pooled rows were armed).  rc 2 without a prior selection or
 * when cap is smaller than a block's pooled pages. */
int32_t ep_sp_get_pooled_pages(ep_sp_ctx* ctx, int32_t* pages, int32_t* counts, int32_t cap, void* stream);

/* Attention arithmetic of an f32 context (dtype EP_SP_F32).  The reference
 * attends an f32 KV cache in f32 (patch :1081-1093: the gathered rows keep the
 * cache type and build_attn_mha runs in f32).
 *   0 (default)  f32: every operand, score, exponential and accumulator in
 *                fp32, on the CUDA cores (same kept sets and CTA grid as the
 *                16-bit kernel; no exchange mode).
 *   1            f16 tensor cores: Q/K/V are converted to f16 shadows (a
 *                device copy of the layer's K/V, allocated on first use) and
 *                attended by the tcgen05 kernel.  A finite input outside the
 *                f16 range (|x| >= 65520 rounds to inf) is not attended
 *                faithfully: the conversion records it and the next
 *                ep_sp_sync_status returns rc 9 (Unsupported).
 * Page scoring and selection always read the f32 inputs in fp64.  rc 2 for
 * other values.  No reference counterpart (the reference has one CPU/ggml
 * path per type). */
int32_t ep_sp_set_f32_attention(ep_sp_ctx* ctx, int32_t mode);
int32_t ep_sp_get_f32_attention(const ep_sp_ctx* ctx);
int32_t ep_sp_select_heads(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v,
                           int32_t kv_len, int32_t n_tok, int32_t head_begin, int32_t head_end, void* stream);
int32_t ep_sp_attend_ctas(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                          int32_t cta_end, void* out, void* stream);
int32_t ep_sp_attention_grid(const ep_sp_ctx* ctx, int32_t n_tok, int32_t* ctas_per_head);
int32_t ep_sp_balance_ctas(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t n_parts,
                           int32_t* cuts);
/* Algorithmic work of the CTA ids [cta_begin, cta_end) of a call under the
 * armed settings: out[0] K3 flops (4 * head_dim per visible (row, key) pair),
 * out[1] bytes of Q read and output written, out[2] visible (row, key) pairs. */
int32_t ep_sp_cta_work(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                       int32_t cta_end, double* out);

/* Head-parallel output exchange over NVLink peer memory (no reference
 * counterpart: the reference runs on one device).  A group of n_ranks
 * contexts, one per GPU, with the same n_head_kv_total, n_head / n_head_kv
 * ratio, head_dim and 16-bit out_dtype, gives each rank one exchange buffer:
 *   [4096-byte header: one uint64 completion counter per slot]
 *   [n_slots slots of rows x (n_head_kv_total * n_head / n_head_kv) x head_dim
 *    out_dtype elements, each 4096-byte aligned]
 * ep_sp_attend_rows_xchg / ep_sp_attend_ctas_xchg run K3 like
 * ep_sp_attend_rows / ep_sp_attend_ctas, but every output tile goes from the
 * kernel's epilogue straight into slot `slot` of EVERY rank's buffer
 * (coalesced stores over NVLink, at the tile's own head columns of the
 * full-width rows),
 * so the attention and its all-gather are one kernel; once it has completed,
 * a one-warp kernel on the same stream adds the call's number of (token,
 * query head) rows to the slot's counter on every rank.
 * ep_sp_xchg_wait enqueues a bounded wait (rc 6 from ep_sp_sync_status on
 * timeout) until `rows` more full-width rows have landed in this rank's slot
 * since the previous wait on it, i.e. until the exchange calls of all ranks
 * between the two waits covered rows x all heads.  Any split works (KV-head
 * slices, ep_sp_balance_ctas ranges of whole-model contexts, ...) as long as
 * the ranks' calls together cover every (row, head) exactly once.
 *
 * Setup, on every rank: ep_sp_xchg_alloc (which also returns the buffer's
 * 64-byte CUDA IPC handle when ipc_handle is not NULL), an all-gather of the
 * handles over the process group, ep_sp_xchg_open of each peer's handle,
 * ep_sp_xchg_attach with every rank's base as mapped in this process
 * (bases[rank] = the own buffer; contexts of one process may pass each
 * other's buffers directly), then a barrier of the group before the first
 * exchange call.  A slot's data may be read after ep_sp_xchg_wait until any
 * rank's next exchange call into that slot, so rotate two or more slots and
 * enqueue a slot's readers on the stream before this rank's next exchange
 * call.  rc 2 on bad arguments or a missing setup step, 9 for a non-16-bit
 * out_dtype. */
#define EP_SP_XCHG_MAX_RANKS 8
#define EP_SP_XCHG_HANDLE_BYTES 64
int32_t ep_sp_xchg_alloc(ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, void** base, void* ipc_handle);
int32_t ep_sp_xchg_open(ep_sp_ctx* ctx, const void* ipc_handle, void** base);
int32_t ep_sp_xchg_attach(ep_sp_ctx* ctx, int32_t n_ranks, int32_t rank, void* const* bases);
/* Caller-allocated exchange buffers instead of ep_sp_xchg_alloc / open /
 * attach: bases[r] is rank r's buffer as mapped in this process (the layout
 * above, ep_sp_xchg_bytes bytes, 4096-byte aligned; bases[rank] is this
 * rank's own and its counters are zeroed here), and mc_base, when not NULL, is
 * an NVLink multicast mapping that binds every rank's buffer at the same
 * offset (a symmetric-memory allocation's multicast address).  With mc_base
 * the exchange epilogue stores each 16-byte chunk of an output tile ONCE
 * through the multicast address and the switch replicates it to every rank,
 * instead of once per rank; the completion counters stay per rank.  The
 * caller keeps ownership (the context frees nothing) and must keep every
 * rank's buffer and mapping alive until all ranks' exchange calls are done.
 * rc 2 on bad arguments or an already attached buffer, 9 for a non-16-bit
 * out_dtype. */
int32_t ep_sp_xchg_attach_buffers(ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, int32_t n_ranks, int32_t rank,
                                  void* const* bases, void* mc_base);
/* Bytes of one rank's exchange buffer for rows x n_slots. */
int32_t ep_sp_xchg_bytes(const ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, size_t* bytes);
/* Device address of slot `slot` of this rank's buffer (full-width rows). */
int32_t ep_sp_xchg_slot(const ep_sp_ctx* ctx, int32_t slot, void** data);
int32_t ep_sp_attend_rows_xchg(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin,
                               int32_t row_end, int32_t slot, void* stream);
int32_t ep_sp_attend_ctas_xchg(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                               int32_t cta_end, int32_t slot, void* stream);
int32_t ep_sp_xchg_wait(ep_sp_ctx* ctx, int32_t slot, int32_t rows, void* stream);

/* Options of the native chunk loop, the bound-gating subset of
 * SparsePrefiller::Options (include/edge_prefill/sparse_prefill.h:15-56). */
typedef struct ep_sp_prefill_options {
    uint32_t chunk_size;      /* 0 = align to n_ubatch */
    int32_t enable_chunking;  /* 0: auto n_ubatch chunks (gating is chunk-scoped) */
    int32_t enable_qg_bound;
    uint32_t qg_sel_pages;
    uint32_t qg_local_rows;   /* passed unchanged as local_pages, as the reference does */
    uint32_t qg_pool_pages;
} ep_sp_prefill_options;

typedef struct ep_sp_prefill_stats {
    uint32_t chunks;
    int32_t query_gating;   /* bound gating engaged */
    int32_t attn_fallback;  /* arming rejected: ran dense */
    uint32_t qg_groups;
    uint32_t chunk_attn_rows; /* audit: local + sink + sel_pages * page_size (sparse_prefill.cpp:469-474) */
} ep_sp_prefill_stats;

/* Native prefill loop of SparsePrefiller::prefill / attn_prefill restricted to
 * the attention path (src/sparse_prefill.cpp:133-148, 252-262, 352-487): arms
 * bound gating (a rejected arming degrades to dense attention with
 * attn_fallback = 1, never an error), enters prefill mode, plans chunks with
 * ChunkScheduler::plan semantics (chunk clamped to n_ubatch), runs every layer
 * of every chunk, then always disarms and leaves prefill mode.
 *   q[l], out[l]: [n_tokens][n_head][head_dim]; k[l], v[l]: [n_tokens][n_head_kv][head_dim]
 *   (host arrays of n_layers device pointers).
 * The sequence restarts at row 0. */
int32_t ep_sp_prefill(ep_sp_ctx* ctx, const ep_sp_prefill_options* opts, int32_t n_layers,
                      const void* const* q, const void* const* k, const void* const* v,
                      void* const* out, int32_t n_tokens, int32_t n_ubatch,
                      ep_sp_prefill_stats* stats, void* stream);

/* K4a: FFN-skip row compaction.  Rows r with keep_mask[r] != 0 are copied, in
 * row order, into x_kept[0..n_keep); row_ids[i] = source row; *n_keep (device
 * int32) receives the count.  In prefill mode a layer whose bit is set in the
 * FFN skip mask keeps no row (its FFN contributes zero: ffn patch :146-149).
 * x, x_kept: [n_rows][hidden] of the context dtype. */
int32_t ep_sp_ffn_compact(ep_sp_ctx* ctx, int32_t layer, const void* x,
                          const uint8_t* keep_mask, int32_t n_rows, int32_t hidden,
                          void* x_kept, int32_t* row_ids, int32_t* n_keep, void* stream);

/* K4b: scatter-add of the FFN output of the kept rows back into the residual:
 * residual[row_ids[i]] += ffn_out[i] (fp32 add, rounded to the dtype) for
 * i < *n_keep; every other row is left untouched, which is the reference's
 * skipped-FFN semantics per row.  n_rows bounds *n_keep. */
int32_t ep_sp_ffn_scatter(ep_sp_ctx* ctx, int32_t layer, const void* ffn_out, void* residual,
                          const int32_t* row_ids, const int32_t* n_keep, int32_t n_rows,
                          int32_t hidden, void* stream);

/* Synchronises the stream and reads the context's device error word: rc 6
 * (Prefill) when a kernel's bounded wait expired or a selection was out of
 * range or a paged-KV block table entry lay outside the pool since the last
 * check, rc 9 (Unsupported) when an f32 input left the
 * f16 range of the tensor-core mode (the word is then cleared), 12 on a CUDA
 * error.
 * It also reads and clears the error word of ep_sp_select_pages_noalloc on
 * the context's device.  The compute calls themselves never synchronise. */
int32_t ep_sp_sync_status(ep_sp_ctx* ctx, void* stream);

/* Kernel timing for benchmarks (no reference counterpart).  While enabled,
 * every kernel the context launches is bracketed by CUDA events on its launch
 * stream.  ep_sp_profile_read synchronises, then reports per kernel family
 * (0 K1 page sums, 1 K2 select, 2 K3 attention, 3 K4 compaction, 4 K4
 * scatter, 5 exchange signal + wait) the summed device milliseconds and the launch
 * count since the last enable. */
#define EP_SP_NUM_KERNELS 6
int32_t ep_sp_profile_enable(ep_sp_ctx* ctx, int32_t on);
int32_t ep_sp_profile_read(ep_sp_ctx* ctx, double* ms, int64_t* launches);

/* Algorithmic work of one ep_sp_attend_layer(layer, kv_len, n_tok) call with
 * the context's current settings, from the same block plan the kernels use:
 *   out[0] K1 bytes (new pages read + fp64 sums written)
 *   out[1] K2 bytes (page sums read + query + list written)   out[2] K2 flops
 *   out[3] K3 flops (4*d per unmasked (query row, q head, key))
 *   out[4] K3 bytes (Q + out + unique kept K/V rows per block and KV head)
 *   out[5] K3 kept keys summed over (query row, q head)
 * Assumes the pages before kv_len - n_tok were pooled by earlier calls. */
int32_t ep_sp_layer_work(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, double* out);

/* Page selection without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they need a selection -- an operator callback inside a graph executor such
 * as ggml's, which receives only its input and output tensors after the
 * executor has planned and reserved every buffer (a cudaMalloc there would
 * synchronise the device and break that plan), or a host with a fixed device
 * memory budget.
 *
 * Computes exactly what ep_sp_attend_layer writes to sel_pages / sel_counts
 * for the same (layer, q, k, kv_len, n_tok) and context settings -- K1 page
 * sums of the scored pages, then K2 score + top-k -- but keeps its scratch
 * (page sums, budgets, error word) in one file-scope device array of
 * EP_SP_NOALLOC_SCRATCH_BYTES bytes that every GPU loading the library holds
 * until the process exits.  Makes no cudaMalloc / cudaFree call, never
 * reserves the context's own device memory and runs no attention.
 *   q [n_tok][n_head][head_dim], k [kv_len][n_head_kv][head_dim] (device);
 *   sel_pages [n_blocks][n_head_kv][sel_cap], sel_counts [n_blocks][n_head_kv].
 * The context's device must be current.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) and caches it; make that
 * first call before any stream capture.  Every call shares the array, so calls
 * whose work overlaps on the GPU (other streams, other threads) race; each
 * call rewrites everything it reads.  The budgets reach the device as kernel
 * parameters, so no host buffer outlives the call.  A device-side error (a
 * selection out of range) lands in the array's error word, which the next
 * ep_sp_sync_status of any context on that device reports (rc 6) and clears.
 * rc 2 for more than 256 KV heads, for the usual argument errors, or when
 * the call's page sums and scores do not fit the scratch, i.e. unless
 *   2048 + (Hkv * head_dim + n_blocks * Hkv) * 8 * max_lsp
 *     <= EP_SP_NOALLOC_SCRATCH_BYTES,
 * with n_blocks the call's gating blocks and max_lsp the largest local start
 * page of a selecting block (every page before it is scored). */
#define EP_SP_NOALLOC_SCRATCH_BYTES (4u << 20)
int32_t ep_sp_select_pages_noalloc(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k,
                                   int32_t kv_len, int32_t n_tok, int32_t* sel_pages, int32_t* sel_counts,
                                   int32_t sel_cap, void* stream);

/* Last error message of the context ("" when none; never NULL). */
const char* ep_sp_last_error(const ep_sp_ctx* ctx);
/* edge_prefill::error_code_name (src/status.cpp:5-22). */
const char* ep_sp_error_name(int32_t code);

/* Host-side planning, no device needed ----------------------------------- */

/* ChunkScheduler::plan (src/chunk_scheduler.cpp:9-45): up to cap [begin,end)
 * pairs in ranges[2*i], ranges[2*i+1]; *n_out = number of ranges. */
int32_t ep_sp_chunk_plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                         uint32_t* ranges, int32_t cap, int32_t* n_out);
/* FfnSkipController::auto_mask / parse (src/ffn_skip.cpp:41-117).  warning
 * receives "mask-bit-out-of-range" or "" (cap bytes, NUL-terminated). */
int32_t ep_sp_ffn_auto_mask(int32_t n_layer, double ratio, uint64_t* out);
int32_t ep_sp_ffn_parse(const char* spec, int32_t n_layer, uint64_t* out, char* warning,
                        int32_t cap);
/* The four bound-gating keys of the reference's config file parser
 * (src/config.cpp:527-538): qg_bound (bool), qg_sel_pages <= 128,
 * qg_local_rows <= 32768, qg_pool_pages <= 4096.  Other keys are skipped.
 * rc 11 (Io) when the file cannot be opened, rc 2 on a bad value or a line
 * without '='.  Defaults: off, 8, 0, 0. */
int32_t ep_sp_parse_config(const char* path, ep_sp_prefill_options* out);

#ifdef __cplusplus
}
#endif
#endif /* EPSP_H */
