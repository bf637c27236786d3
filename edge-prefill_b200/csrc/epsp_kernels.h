// epsp_kernels.h -- host-side launch interface of the sm_100a kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "epsp_plan.h"

namespace epsp {

// Rows summed sequentially per group in the page-sum contract; the groups of
// a page are then added in ascending order (both in fp64).
constexpr int kPageSumGroupRows = 16;

// Device error word values written by the kernels (first failure wins).
enum DeviceError : int32_t {
    kDevOk = 0,
    kDevWaitProducer = 0x101,
    kDevWaitMma = 0x102,
    kDevWaitSoftmax = 0x103,
    kDevWaitEpilogue = 0x104,
    kDevWaitExchange = 0x105,  // peers' output tiles did not all arrive in time
    kDevWaitPool = 0x106,      // a K1 page span did not arrive in time
    kDevWaitPoolProducer = 0x107,  // K1's producer waited too long for a free stage
    kDevBadSelection = 0x201,
    kDevF16Range = 0x301,      // an f32 input is outside the f16 range of the tensor-core mode
    kDevBadBlockTable = 0x401, // a paged-KV block table entry lies outside the pool
};

// The device error word is err[0] of a 4-word record: the kernel whose
// atomicCAS on err[0] wins also writes err[1] = where (role * 16 + barrier),
// err[2] = its block index, err[3] = its KV tile, for ep_sp_sync_status.
#if defined(__CUDACC__)
__device__ __forceinline__ void report_error(int32_t* err, int32_t code, int32_t where, int32_t tile) {
    if (atomicCAS(err, 0, code) == 0) {
        err[1] = where;
        err[2] = (int32_t)blockIdx.x;
        err[3] = tile;
    }
}
#endif

// Ranks of one head-parallel output exchange (destinations of a K3 call).
constexpr int kMaxDest = 8;

struct PoolArgs {
    const void* k;         // [kv_len][Hkv][d]
    int32_t dtype;         // 0 f32, 1 f16, 2 bf16
    int32_t n_head_kv;
    int32_t head_dim;
    int32_t page_size;
    int32_t page_begin;    // pool pages [page_begin, page_end)
    int32_t page_end;
    int32_t max_pages;     // row stride of psum
    double* psum;          // [Hkv][max_pages][d]
    int32_t head_begin = 0, head_count = 0;  // KV heads pooled (count 0: all)
    int32_t* err = nullptr;      // device error word (bounded waits of the TMA variant)
    uint64_t timeout_ns = 0;     // 0: use the direct variant
    // Append mode (k_new != nullptr): rows >= new_begin are read from k_new
    // ([rows - new_begin][Hkv][d]) and also written to the cache k_store at
    // their row; older rows of a page come from the cache `k`.
    const void* k_new = nullptr;
    void* k_store = nullptr;
    int32_t new_begin = 0;
    KvPaging paging;  // k / k_store are pools when paging.block_rows > 0
};
cudaError_t launch_pool_pages(const PoolArgs& a, cudaStream_t s);

struct SelectArgs {
    const void* q;          // ubatch queries [n_tok][Hq][d]
    int32_t dtype;
    int32_t n_head, n_head_kv, head_dim;
    int32_t u0, n_tok;      // ubatch rows [u0, u0 + n_tok)
    int32_t q_subblock;
    GateParams gate;
    const int32_t* k_budget;  // [Hkv] top-k budget per KV head for this layer (-1 dense)
    const double* psum;       // [Hkv][max_pages][d]
    int32_t max_pages;
    int32_t* sel;             // [n_blocks][Hkv][sel_cap]
    int32_t* cnt;             // [n_blocks][Hkv]
    int32_t sel_cap;
    int32_t* err;
    double* scores;           // workspace [n_blocks][Hkv][max_pages] (select_scores_elems)
    int32_t max_cand;         // largest lsp - 1 over the blocks that select (sizes the sort)
    int32_t score_chunks;     // set by the launcher
    int32_t head_begin = 0, head_count = 0;  // per-KV-head mode: heads selected (count 0: all)
    // pooled pages (gate.pool_pages > 0): the n_pool candidates ranked right
    // after the selection, ascending, [n_blocks][Hkv][pool_cap] + counts
    int32_t* pool = nullptr;
    int32_t* pool_cnt = nullptr;
    int32_t pool_cap = 0;
    // Per-KV-head routing by the live page-score spread (route_mode 1 / 2,
    // per-KV-head selection only): K2r writes each (block, head)'s effective
    // budget into route_k [n_blocks][Hkv] between K2a and K2b.
    int32_t route_mode = 0;
    double route_threshold = 0.0;
    int32_t* route_k = nullptr;
};
// Spread guard of the routing (the denominator's epsilon).
constexpr double kRouteEps = 1e-6;
// K2a (scores, wide grid), K2r (routing, when armed), then K2b (bitonic top-k
// per block and KV head).
cudaError_t launch_select_pages(const SelectArgs& a, cudaStream_t s);
size_t select_scores_elems(int n_blocks, int n_head_kv, int max_pages);

// K2c: the pooled rows of one call: for gating block b, KV head h and pooled
// page j < pool_cnt[b][h], row b * pool_stride + j of pk / pv ([rows][Hkv][d]
// in out_dtype) = the page's K / V sums / page_size (fp64 -> f32 -> out_dtype);
// rows j in [pool_cnt, pool_stride) are zero.
struct PoolRowArgs {
    const double* ksum;   // [Hkv][max_pages][d]
    const double* vsum;
    int32_t max_pages;
    const int32_t* pool;  // [n_blocks][Hkv][pool_cap]
    const int32_t* pool_cnt;
    int32_t pool_cap;
    int32_t n_blocks, n_head_kv, head_dim, page_size;
    int32_t pool_stride;  // rows per gating block in pk / pv
    int32_t out_dtype;    // 0 f32, 1 f16, 2 bf16
    void* pk;
    void* pv;
    int32_t head_begin = 0, head_count = 0;
};
cudaError_t launch_build_pooled_rows(const PoolRowArgs& a, cudaStream_t s);

struct AttnArgs {
    const void* q;           // [n_tok][Hq][d]
    const void* k;           // [kv_len][Hkv][d]
    const void* v;
    void* out;               // [n_tok][Hq][d] in out_dtype
    int32_t dtype, out_dtype;
    int32_t n_head, n_head_kv, head_dim;
    int32_t u0, n_tok, kv_len;
    int32_t q_subblock;
    GateParams gate;
    const int32_t* k_budget;  // [Hkv]
    const int32_t* sel;       // [n_blocks][Hkv][sel_cap]
    int32_t sel_cap;
    float kq_scale;
    int32_t* err;
    uint64_t timeout_ns;
    int32_t blk_begin, blk_count;  // gating blocks [blk_begin, blk_begin + blk_count) of the call
    // Output placement: query head hq of call row i lands at
    // out + ((i * out_heads) + out_head0 + hq) * head_dim elements.
    int32_t out_heads = 0;  // heads per output row (0: n_head)
    int32_t out_head0 = 0;
    // CTAs of the call: the grid is [Hkv][blk_count][ctas_per_block] head-major;
    // a launch runs ids [cta_begin, cta_begin + cta_count) (count 0: to the end).
    int32_t cta_begin = 0, cta_count = 0;
    // Query tiles per CTA: 2 (one CTA per SM, the tiles ping-pong on the tensor
    // core) or 1 (two CTAs per SM).
    int32_t tiles_per_cta = 2;
    // Exchange mode (n_dest > 0, 16-bit output): every tile goes to all
    // destination buffers (same layout as out); `out` is unused.  The
    // completion is signalled by launch_exchange_signal after the kernel.
    int32_t n_dest = 0;
    void* dest[kMaxDest] = {};
    // Multicast address of the slot (an NVLink multicast object over every
    // destination): each chunk is stored once with multimem.st instead of
    // once per destination.
    void* mc_dest = nullptr;
    // Pooled rows (gate.pool_pages > 0): the plan's n_pool rows of block b
    // start at row b * pool_stride of pk / pv ([rows][Hkv][d], dtype).
    const void* pk = nullptr;
    const void* pv = nullptr;
    int32_t pool_stride = 0;
    int32_t pool_rows_total = 0;  // rows of pk / pv
    // Per-(block, head) counts written by K2 ([n_blocks][Hkv]); when set they
    // replace the plan's k_sel / n_pool (head routing changes them).
    const int32_t* cnt = nullptr;
    const int32_t* pool_cnt = nullptr;
    KvPaging paging;  // k / v are pools when paging.block_rows > 0
};
// Returns cudaErrorNotSupported for shapes the tcgen05 kernel does not cover.
cudaError_t launch_sparse_attention(const AttnArgs& a, cudaStream_t s);
// The same attention for f32 Q/K/V in fp32 on the CUDA cores (same CTA grid
// and arguments; no exchange mode).
cudaError_t launch_sparse_attention_f32(const AttnArgs& a, cudaStream_t s);
// CTAs per gating block and KV head (groups of tiles_per_cta query tiles of
// 128 / G tokens).
int attention_ctas_per_block(int n_head, int n_head_kv, int n_tok, int q_subblock, int tiles_per_cta);

// After an exchange-mode K3 on the same stream (whose completion orders all of
// its stores first): adds `value` to each of the n counters with system-scope
// release.
cudaError_t launch_exchange_signal(unsigned long long* const* sig, int n, unsigned long long value, cudaStream_t s);

// Bounded wait (one thread) until *sig >= target with system-scope acquire;
// on timeout the error word gets kDevWaitExchange.
cudaError_t launch_exchange_wait(const unsigned long long* sig, unsigned long long target, int32_t* err,
                                 uint64_t timeout_ns, cudaStream_t s);
// Shared-memory bytes the attention kernel needs for a head_dim (for checks).
int attention_smem_bytes(int head_dim);

struct FfnCompactArgs {
    const void* x;         // [n_rows][hidden]
    int32_t elem_bytes;
    const uint8_t* keep;   // [n_rows]
    int32_t n_rows, hidden;
    void* x_kept;          // [n_rows][hidden]
    int32_t* row_ids;      // [n_rows]
    int32_t* n_keep;       // device scalar
    int32_t skip_layer;    // 1: keep nothing
};
cudaError_t launch_ffn_compact(const FfnCompactArgs& a, cudaStream_t s);

struct FfnScatterArgs {
    const void* ffn_out;   // [n_keep][hidden]
    void* residual;        // [n_rows][hidden]
    int32_t dtype;
    const int32_t* row_ids;
    const int32_t* n_keep;
    int32_t n_rows, hidden;
};
cudaError_t launch_ffn_scatter(const FfnScatterArgs& a, cudaStream_t s);

// Device-to-device copy of `bytes` (16-byte vectors on the SMs when both
// addresses and the size allow it, else cudaMemcpyAsync).
cudaError_t launch_copy_rows(const void* src, void* dst, size_t bytes, cudaStream_t s);

// Copy of n_rows contiguous rows into the logical rows [row_begin, ...) of a
// paged pool (16-byte vectors on the SMs).
cudaError_t launch_copy_rows_paged(const void* src, void* dst_pool, int32_t row_begin, int32_t n_rows, size_t row_bytes,
                                   const KvPaging& pg, int32_t* err, cudaStream_t s);

// Reads and clears the device error word of the no-allocation selection path
// on the current device (0 when that device never ran it).
cudaError_t noalloc_take_error_word(int32_t* word);

// f32 -> f16 conversion of rows (f32 contexts in the tensor-core mode keep an
// f16 shadow); a finite value that leaves the f16 range records kDevF16Range.
cudaError_t launch_convert_f32_to_f16(const float* src, void* dst, int64_t n, int32_t* err, cudaStream_t s);

}  // namespace epsp
