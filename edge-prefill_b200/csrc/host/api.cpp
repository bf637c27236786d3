// api.cpp -- the extern "C" entry points of include/epsp.h: context
// lifecycle, arming (patch :403-437), and the per-layer launch sequence
// K1 -> K2 -> K3 on the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../epsp_kernels.h"
#include "../epsp_plan.h"
#include "epsp_host.h"

using namespace edge_prefill_b200;

namespace {

constexpr int32_t kOk = 0;
constexpr int32_t kInvalid = static_cast<int32_t>(ErrorCode::InvalidArgument);
constexpr int32_t kPrefill = static_cast<int32_t>(ErrorCode::Prefill);
constexpr int32_t kUnsupported = static_cast<int32_t>(ErrorCode::Unsupported);
constexpr int32_t kOom = static_cast<int32_t>(ErrorCode::OutOfMemory);
constexpr int32_t kInternal = static_cast<int32_t>(ErrorCode::Internal);
constexpr int32_t kUnavailable = static_cast<int32_t>(ErrorCode::Unavailable);

int32_t fail(ep_sp_ctx* ctx, int32_t rc, const std::string& msg) {
    if (ctx) ctx->last_error = msg;
    return rc;
}

int32_t cuda_fail(ep_sp_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, e == cudaErrorMemoryAllocation ? kOom : kInternal,
                std::string(what) + ": " + cudaGetErrorString(e));
}

size_t esize(int32_t dtype) { return dtype == EP_SP_F32 ? 4 : 2; }

epsp::GateParams gate_of(const ep_sp_ctx* c) {
    epsp::GateParams g;
    g.page_size = c->cfg.page_size;
    g.local_pages = c->local_pages;
    g.shared = c->per_kv_head ? 0 : 1;
    g.max_gather_rows = c->max_gather_rows;
    g.pool_pages = c->pool_pages;
    return g;
}

bool gating_active(const ep_sp_ctx* c) { return c->prefill_mode && c->qg_bound; }

// Budget of KV head h (local index) in layer l while gating is armed.
int32_t budget_of(const ep_sp_ctx* c, int32_t l, int32_t h) {
    if (!c->k_matrix.empty()) return c->k_matrix[(size_t)l * c->n_head_kv_total + c->cfg.kv_head_offset + h];
    return c->sel_pages;
}

int32_t ensure_device(ep_sp_ctx* c) {
    if (c->reserved) return kOk;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || c->cfg.device >= n) {
        cudaGetLastError();
        return fail(c, kUnavailable, "no CUDA device " + std::to_string(c->cfg.device));
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, c->cfg.device) != cudaSuccess) return fail(c, kUnavailable, "device query failed");
    if (prop.major != 10) return fail(c, kUnsupported, std::string("not an sm_100 device: ") + prop.name);
    cudaError_t e = cudaSetDevice(c->cfg.device);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
    const int32_t Hkv = c->cfg.n_head_kv, d = c->cfg.head_dim, nl = c->cfg.n_layer;
    c->max_pages = std::max(1, c->cfg.max_ctx / c->cfg.page_size);
    const size_t psum_bytes = (size_t)nl * Hkv * d * c->max_pages * sizeof(double);
    if ((e = cudaMalloc(&c->psum, psum_bytes)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc page sums");
    if ((e = cudaMalloc(&c->d_budget, sizeof(int32_t) * nl * Hkv)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc");
    if ((e = cudaMalloc(&c->d_dense, sizeof(int32_t) * Hkv)) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc");
    if ((e = cudaMalloc(&c->d_err, 4 * sizeof(int32_t))) != cudaSuccess) return cuda_fail(c, e, "cudaMalloc");
    std::vector<int32_t> dense(Hkv, -1);
    cudaMemcpy(c->d_dense, dense.data(), sizeof(int32_t) * Hkv, cudaMemcpyHostToDevice);
    cudaMemset(c->d_err, 0, 4 * sizeof(int32_t));
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(c, e, "device init");
    c->pooled.assign((size_t)nl * Hkv, 0);
    c->v_pooled.assign((size_t)nl * Hkv, 0);
    c->appended.assign(nl, 0);
    c->shadowed.assign(nl, 0);
    c->reserved = true;
    return kOk;
}

// Grows a stream-ordered workspace of T.
template <class T>
int32_t grow(ep_sp_ctx* c, T** p, size_t* have, size_t need, cudaStream_t s) {
    if (*have >= need) return kOk;
    if (*p) cudaFreeAsync(*p, s);
    *p = nullptr;
    *have = 0;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(p), need * sizeof(T), s);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaMallocAsync workspace");
    *have = need;
    return kOk;
}

void* take_event(ep_sp_ctx* c) {
    if (!c->event_pool.empty()) {
        void* e = c->event_pool.back();
        c->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

// Runs one kernel launch, bracketed by events on its stream when profiling.
template <class F>
cudaError_t timed(ep_sp_ctx* c, int kind, cudaStream_t s, F&& launch) {
    ++c->launches[kind];
    if (!c->profiling) return launch();
    void* a = take_event(c);
    void* b = take_event(c);
    if (a) cudaEventRecord(static_cast<cudaEvent_t>(a), s);
    const cudaError_t e = launch();
    if (b) cudaEventRecord(static_cast<cudaEvent_t>(b), s);
    if (a && b) c->events.push_back({kind, a, b});
    return e;
}

// K3 arguments of rows [row_begin, row_end) of the last selection.
int32_t attn_args_rows(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin, int32_t row_end,
                  epsp::AttnArgs& aa) {
    const ep_sp_config& cf = ctx->cfg;
    if (!ctx->sel_valid || ctx->sel_layer != layer || ctx->sel_kv_len != kv_len || ctx->sel_n_tok != n_tok ||
        ctx->sel_epoch != ctx->epoch)
        return fail(ctx, kInvalid, "no ep_sp_select_layer for this (layer, kv_len, n_tok) and settings");
    const int32_t L = epsp::block_len(n_tok, ctx->q_subblock);
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    if (row_begin < 0 || row_end > n_tok || row_begin >= row_end || row_begin % L || (row_end % L && row_end != n_tok))
        return fail(ctx, kInvalid, "row range must cover whole gating blocks of the call");
    aa.q = ctx->att_q;
    aa.k = ctx->att_k;
    aa.v = ctx->att_v;
    aa.out = nullptr;
    aa.dtype = ctx->att_dtype;
    aa.out_dtype = cf.out_dtype;
    aa.n_head = cf.n_head;
    aa.n_head_kv = cf.n_head_kv;
    aa.head_dim = cf.head_dim;
    aa.u0 = kv_len - n_tok;
    aa.n_tok = n_tok;
    aa.kv_len = kv_len;
    aa.q_subblock = ctx->q_subblock;
    aa.gate = gate_of(ctx);
    aa.k_budget = ctx->sel_budget;
    aa.sel = ctx->sel_ptr;
    aa.sel_cap = ctx->sel_cap_used;
    aa.kq_scale = cf.kq_scale;
    aa.err = ctx->d_err;
    aa.timeout_ns = ctx->timeout_ns;
    aa.blk_begin = row_begin / L;
    aa.blk_count = std::min(nb, (row_end + L - 1) / L) - aa.blk_begin;
    aa.cta_begin = 0;
    aa.cta_count = 0;
    aa.tiles_per_cta = ctx->attn_tiles;
    aa.cnt = ctx->sel_cnt_attn;
    aa.pool_cnt = ctx->sel_pool_cnt_attn;
    aa.paging = ctx->att_dtype == cf.dtype ? ctx->paging : epsp::KvPaging{};  // f16 shadows are contiguous
    if (ctx->sel_pool_cap > 0) {
        aa.pk = ctx->att_pk;
        aa.pv = ctx->att_pv;
        aa.pool_stride = ctx->sel_pool_stride;
        aa.pool_rows_total = ctx->sel_n_blocks * ctx->sel_pool_stride;
    } else {
        aa.gate.pool_pages = 0;
    }
    return kOk;
}

// K3 arguments of the CTA ids [cta_begin, cta_end) of the whole call's
// head-major grid; the last selection must cover their KV heads.
int32_t cta_args(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin, int32_t cta_end,
                 epsp::AttnArgs& aa) {
    const int32_t rc = attn_args_rows(ctx, layer, kv_len, n_tok, 0, n_tok, aa);
    if (rc) return rc;
    const int64_t per_head = (int64_t)aa.blk_count * epsp::attention_ctas_per_block(ctx->cfg.n_head, ctx->cfg.n_head_kv,
                                                                                     n_tok, ctx->q_subblock, ctx->attn_tiles);
    if (cta_begin < 0 || cta_end <= cta_begin || cta_end > per_head * ctx->cfg.n_head_kv)
        return fail(ctx, kInvalid, "CTA range out of the call's grid");
    if (cta_begin / per_head < ctx->sel_head_begin || (cta_end - 1) / per_head >= ctx->sel_head_end)
        return fail(ctx, kInvalid, "the last selection does not cover the KV heads of the CTA range");
    aa.cta_begin = cta_begin;
    aa.cta_count = cta_end - cta_begin;
    return kOk;
}

// Rows of the call: every KV head, so the selection must cover all of them.
int32_t attn_args(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin, int32_t row_end,
                  epsp::AttnArgs& aa) {
    const int32_t rc = attn_args_rows(ctx, layer, kv_len, n_tok, row_begin, row_end, aa);
    if (rc) return rc;
    if (ctx->sel_head_begin != 0 || ctx->sel_head_end != ctx->cfg.n_head_kv)
        return fail(ctx, kInvalid, "the last selection covers only some KV heads (use the CTA-range calls)");
    return kOk;
}

int32_t launch_attn(ep_sp_ctx* ctx, const epsp::AttnArgs& aa, cudaStream_t s) {
    const bool f32 = aa.dtype == EP_SP_F32;
    if (f32 && aa.n_dest > 0)
        return fail(ctx, kUnsupported, "the exchange needs the 16-bit tensor-core attention (ep_sp_set_f32_attention 1)");
    cudaError_t e = timed(ctx, 2, s, [&] {
        return f32 ? epsp::launch_sparse_attention_f32(aa, s) : epsp::launch_sparse_attention(aa, s);
    });
    if (e == cudaErrorNotSupported) return fail(ctx, kUnsupported, "attention shape not supported");
    if (e != cudaSuccess) return cuda_fail(ctx, e, "K3 attention");
    return kOk;
}

constexpr size_t kXchgHeader = 4096;  // per-slot uint64 counters, then the slots
constexpr int32_t kXchgMaxSlots = 64;

}  // namespace

extern "C" {

int32_t ep_sp_create(const ep_sp_config* cfg, ep_sp_ctx** out) {
    if (!cfg || !out) return kInvalid;
    *out = nullptr;
    const ep_sp_config& c = *cfg;
    if (c.n_layer < 1 || c.n_head_kv < 1 || c.n_head < 1 || c.n_head % c.n_head_kv) return kInvalid;
    if (c.n_head / c.n_head_kv > 128) return kInvalid;
    if (c.head_dim != 64 && c.head_dim != 128) return kInvalid;
    if (c.dtype < EP_SP_F32 || c.dtype > EP_SP_BF16 || c.out_dtype < EP_SP_F32 || c.out_dtype > EP_SP_BF16) return kInvalid;
    if (c.page_size != 32 && c.page_size != 64 && c.page_size != 128) return kInvalid;
    if (c.max_ctx < 1 || c.device < 0 || c.kv_head_offset < 0) return kInvalid;
    const int32_t total = c.n_head_kv_total > 0 ? c.n_head_kv_total : c.n_head_kv;
    if (c.kv_head_offset + c.n_head_kv > total) return kInvalid;
    if (!(c.kq_scale >= 0.f) || !std::isfinite(c.kq_scale)) return kInvalid;
    ep_sp_ctx* ctx = new (std::nothrow) ep_sp_ctx();
    if (!ctx) return kOom;
    ctx->cfg = c;
    ctx->n_head_kv_total = total;
    if (ctx->cfg.kq_scale == 0.f) ctx->cfg.kq_scale = 1.0f / std::sqrt(static_cast<float>(c.head_dim));
    *out = ctx;
    return kOk;
}

int32_t ep_sp_reserve(ep_sp_ctx* ctx) {
    if (!ctx) return kInvalid;
    return ensure_device(ctx);
}

void ep_sp_destroy(ep_sp_ctx* ctx) {
    if (!ctx) return;
    if (ctx->reserved) {
        cudaSetDevice(ctx->cfg.device);
        cudaDeviceSynchronize();
        cudaFree(ctx->psum);
        cudaFree(ctx->d_budget);
        cudaFree(ctx->d_dense);
        cudaFree(ctx->d_err);
        cudaFree(ctx->d_sel);
        cudaFree(ctx->d_cnt);
        cudaFree(ctx->d_scores);
        cudaFree(ctx->vsum);
        cudaFree(ctx->d_pool);
        cudaFree(ctx->d_pool_cnt);
        cudaFree(ctx->d_pkv);
        cudaFree(ctx->d_route);
        cudaFree(ctx->sh_q);
        cudaFree(ctx->sh_k);
        cudaFree(ctx->sh_v);
        for (auto& ev : ctx->events) {
            cudaEventDestroy(static_cast<cudaEvent_t>(ev.start));
            cudaEventDestroy(static_cast<cudaEvent_t>(ev.stop));
        }
        for (void* ev : ctx->event_pool) cudaEventDestroy(static_cast<cudaEvent_t>(ev));
        for (void* p : ctx->xchg_opened) cudaIpcCloseMemHandle(p);
        if (!ctx->xchg_external) cudaFree(ctx->xchg_base);
    }
    delete ctx;
}

// patch :403-437
int32_t ep_sp_set_qg_bound(ep_sp_ctx* ctx, int32_t enabled, int32_t sel_pages, int32_t local_pages,
                           int32_t pool_pages) {
    if (!ctx) return kInvalid;
    if (enabled != 0 && enabled != 1) return kInvalid;
    if (sel_pages < 0 || sel_pages > 128 || local_pages < 0 || local_pages > 1024 || pool_pages < 0) return kInvalid;
    // Arming clears every other sparse mode; this library holds no other one.
    ctx->qg_bound = enabled;
    ctx->sel_pages = enabled ? sel_pages : 0;
    ctx->local_pages = enabled ? local_pages : 0;
    ctx->pool_pages = enabled ? pool_pages : 0;
    ++ctx->epoch;
    return kOk;
}

int32_t ep_sp_get_qg_bound(const ep_sp_ctx* ctx) { return ctx ? ctx->qg_bound : 0; }

int32_t ep_sp_set_ext(ep_sp_ctx* ctx, int32_t per_kv_head, int32_t q_subblock, int32_t max_gather_rows) {
    if (!ctx) return kInvalid;
    if ((per_kv_head != 0 && per_kv_head != 1) || q_subblock < 0 || max_gather_rows < 0) return kInvalid;
    ctx->per_kv_head = per_kv_head;
    ctx->q_subblock = q_subblock;
    ctx->max_gather_rows = max_gather_rows;
    if (!per_kv_head) ctx->k_matrix.clear();
    ++ctx->epoch;
    return kOk;
}

int32_t ep_sp_set_k_matrix(ep_sp_ctx* ctx, const int32_t* k, size_t n) {
    if (!ctx) return kInvalid;
    if (n == 0) {
        ctx->k_matrix.clear();
        ++ctx->epoch;
        return kOk;
    }
    if (!k) return kInvalid;
    if (!ctx->per_kv_head) return kInvalid;
    if (n != (size_t)ctx->cfg.n_layer * ctx->n_head_kv_total) return kInvalid;
    for (size_t i = 0; i < n; ++i)
        if (k[i] == 0 || k[i] < -1) return kInvalid;
    ctx->k_matrix.assign(k, k + n);
    ++ctx->epoch;
    return kOk;
}

int32_t ep_sp_get_k_matrix_size(const ep_sp_ctx* ctx) { return ctx ? static_cast<int32_t>(ctx->k_matrix.size()) : 0; }

void ep_sp_set_prefill_mode(ep_sp_ctx* ctx, int32_t prefill) {
    if (ctx) ctx->prefill_mode = prefill ? 1 : 0;
}
int32_t ep_sp_get_prefill_mode(const ep_sp_ctx* ctx) { return ctx ? ctx->prefill_mode : 0; }

// ffn patch :73-84
void ep_sp_set_ffn_skip(ep_sp_ctx* ctx, uint64_t mask) {
    if (!ctx) return;
    const int32_t nl = ctx->cfg.n_layer;
    if (nl > 0 && nl < 64) {
        mask &= (uint64_t(1) << nl) - 1;
    } else if (nl >= 64) {
        mask = 0;
    }
    ctx->ffn_skip = mask;
}
uint64_t ep_sp_get_ffn_skip(const ep_sp_ctx* ctx) { return ctx ? ctx->ffn_skip : 0; }

int32_t ep_sp_reset(ep_sp_ctx* ctx) {
    if (!ctx) return kInvalid;
    std::fill(ctx->pooled.begin(), ctx->pooled.end(), 0);
    std::fill(ctx->v_pooled.begin(), ctx->v_pooled.end(), 0);
    std::fill(ctx->appended.begin(), ctx->appended.end(), 0);
    std::fill(ctx->shadowed.begin(), ctx->shadowed.end(), 0);
    return kOk;
}

int32_t ep_sp_query_blocks(const ep_sp_ctx* ctx, int32_t n_tok, int32_t* n_blocks) {
    if (!ctx || !n_blocks || n_tok < 1) return kInvalid;
    *n_blocks = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    return kOk;
}

const char* ep_sp_last_error(const ep_sp_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

int32_t ep_sp_sync_status(ep_sp_ctx* ctx, void* stream) {
    if (!ctx) return kInvalid;
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || ctx->cfg.device >= dev_count) {
        cudaGetLastError();
        return ctx->reserved ? fail(ctx, kUnavailable, "no CUDA device") : kOk;
    }
    cudaSetDevice(ctx->cfg.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "stream");
    // the no-allocation selection keeps its error word in its own scratch
    int32_t na = 0;
    e = epsp::noalloc_take_error_word(&na);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "no-allocation error word");
    if (na != 0) {
        char buf[96];
        std::snprintf(buf, sizeof buf, "no-allocation selection: device error word 0x%x (bad selection)", na);
        return fail(ctx, kPrefill, buf);
    }
    if (!ctx->reserved) return kOk;
    int32_t rec[4] = {0, 0, 0, 0};  // code, where, block, tile
    e = cudaMemcpy(rec, ctx->d_err, sizeof rec, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "error word");
    const int32_t err = rec[0];
    if (err != 0) {
        cudaMemset(ctx->d_err, 0, sizeof rec);
        if (err == epsp::kDevF16Range)
            return fail(ctx, kUnsupported,
                        "an f32 input lies outside the f16 range of the tensor-core mode (ep_sp_set_f32_attention 0 "
                        "attends it in f32)");
        char buf[160];
        std::snprintf(buf, sizeof buf,
                      "device error word 0x%x (bounded wait expired, bad selection or block table); where 0x%x, "
                      "block %d, tile %d",
                      err, rec[1], rec[2], rec[3]);
        return fail(ctx, kPrefill, buf);
    }
    return kOk;
}

int32_t select_impl(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v, int32_t kv_len,
                    int32_t n_tok, int32_t hb, int32_t he, int32_t* sel_pages, int32_t* sel_counts, int32_t sel_cap,
                    void* stream) {
    const ep_sp_config& cf = ctx->cfg;
    ctx->sel_valid = false;
    if (hb < 0 || he > cf.n_head_kv || hb >= he) return fail(ctx, kInvalid, "KV head range out of range");
    if (gating_active(ctx) && !ctx->per_kv_head && (hb != 0 || he != cf.n_head_kv))
        return fail(ctx, kUnsupported, "the shared (reference) selection spans every KV head");
    if (layer < 0 || layer >= cf.n_layer) return fail(ctx, kInvalid, "layer out of range");
    if (!q || !k || !v) return fail(ctx, kInvalid, "null tensor");
    if (n_tok < 1 || kv_len < n_tok || kv_len > cf.max_ctx) return fail(ctx, kInvalid, "bad kv_len / n_tok");
    if (ctx->paging.block_rows > 0 && (int64_t)ctx->paging.n_entries * ctx->paging.block_rows < kv_len)
        return fail(ctx, kInvalid, "the block table does not cover kv_len rows");
    if (ctx->paging.block_rows > 0 && cf.dtype == EP_SP_F32 && ctx->f32_mode == 1)
        return fail(ctx, kUnsupported, "the f16 tensor-core mode of f32 contexts needs a contiguous cache");
    if ((sel_pages != nullptr) != (sel_counts != nullptr) || (sel_pages && sel_cap < 1))
        return fail(ctx, kInvalid, "selection outputs need pages, counts and sel_cap >= 1");
    if (gating_active(ctx) && !ctx->per_kv_head && cf.n_head_kv < ctx->n_head_kv_total)
        return fail(ctx, kUnsupported, "shared (reference) selection needs every KV head in one context");
    const bool routing = gating_active(ctx) && ctx->route_mode != 0;
    if (routing && !ctx->per_kv_head)
        return fail(ctx, kUnsupported, "head routing needs per-KV-head selection (ep_sp_set_ext per_kv_head 1)");
    if (routing && ctx->route_mode == 2 && (hb != 0 || he != cf.n_head_kv || he - hb > 32))
        return fail(ctx, kUnsupported, "head routing mode 2 re-splits a block's pages over all its KV heads (<= 32)");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t P = cf.page_size, Hkv = cf.n_head_kv, d = cf.head_dim;
    const int32_t u0 = kv_len - n_tok;
    const bool active = gating_active(ctx);
    const epsp::GateParams gate = gate_of(ctx);
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    const int32_t L = epsp::block_len(n_tok, ctx->q_subblock);

    // Budgets of this layer's heads; largest k_sel any block can reach and the
    // largest candidate count of a selecting block.
    int32_t max_ksel = 0, max_cand = 0, max_pool = 0;
    if (active) {
        if (ctx->budget_epoch != ctx->epoch) {
            ctx->h_budget.resize((size_t)cf.n_layer * Hkv);
            for (int32_t l = 0; l < cf.n_layer; ++l)
                for (int32_t h = 0; h < Hkv; ++h) ctx->h_budget[(size_t)l * Hkv + h] = budget_of(ctx, l, h);
            cudaError_t e = cudaMemcpyAsync(ctx->d_budget, ctx->h_budget.data(), sizeof(int32_t) * ctx->h_budget.size(),
                                            cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "budget upload");
            ctx->budget_epoch = ctx->epoch;
        }
        for (int32_t b = 0; b < nb; ++b) {
            const int32_t b0 = u0 + b * L, b1 = std::min(u0 + n_tok, b0 + L);
            int32_t block_pages = 0, block_cand = 0;
            for (int32_t h = gate.shared ? 0 : hb; h < (gate.shared ? 1 : he); ++h) {
                const epsp::BlockPlan pl = epsp::plan_block(gate, b0, b1, ctx->h_budget[(size_t)layer * Hkv + h]);
                if (pl.gated) max_ksel = std::max(max_ksel, pl.k_sel);
                if (pl.gated) max_pool = std::max(max_pool, pl.n_pool);
                if (pl.gated && (pl.k_sel > 0 || pl.n_pool > 0)) max_cand = std::max(max_cand, pl.lsp - 1);
                if (pl.gated) {
                    block_pages += pl.k_sel;
                    block_cand = pl.lsp - 1;
                    // routing: a streaming head pools from the top of the ranking
                    if (routing) max_pool = std::max(max_pool, std::min(gate.pool_pages, pl.lsp - 1));
                }
            }
            // routing mode 2 may hand a head up to the block's pages, capped at its candidates
            if (routing && ctx->route_mode == 2) max_ksel = std::max(max_ksel, std::min(block_pages, block_cand));
        }
    }
    if (sel_pages && max_ksel > sel_cap) return fail(ctx, kInvalid, "sel_cap smaller than a block's k_sel");
    const int32_t* d_budget_layer = active ? ctx->d_budget + (size_t)layer * Hkv : ctx->d_dense;

    // f32 contexts attend in f32 (mode 0), or on f16 shadows of the new K/V
    // rows and of this call's Q for the tensor-core kernel (mode 1).
    ctx->att_q = q;
    ctx->att_k = k;
    ctx->att_v = v;
    ctx->att_dtype = cf.dtype;
    if (cf.dtype == EP_SP_F32 && ctx->f32_mode == 1) {
        const size_t row = (size_t)Hkv * d;
        const size_t lay = (size_t)cf.max_ctx * row * 2;
        if (!ctx->sh_k) {
            const size_t kv = (size_t)cf.n_layer * lay;
            cudaError_t e = cudaMalloc(&ctx->sh_k, kv);
            if (e == cudaSuccess) e = cudaMalloc(&ctx->sh_v, kv);
            if (e != cudaSuccess) {
                cudaFree(ctx->sh_k);
                ctx->sh_k = ctx->sh_v = nullptr;
                return cuda_fail(ctx, e, "cudaMalloc f16 shadow");
            }
            std::fill(ctx->shadowed.begin(), ctx->shadowed.end(), 0);
        }
        char* shk = static_cast<char*>(ctx->sh_k) + (size_t)layer * lay;
        char* shv = static_cast<char*>(ctx->sh_v) + (size_t)layer * lay;
        if (u0 == 0) ctx->shadowed[layer] = 0;
        const int32_t conv_from = std::min(ctx->shadowed[layer], u0);
        cudaError_t e = epsp::launch_convert_f32_to_f16(static_cast<const float*>(k) + (size_t)conv_from * row,
                                                        shk + (size_t)conv_from * row * 2,
                                                        (int64_t)(kv_len - conv_from) * row, ctx->d_err, s);
        if (e == cudaSuccess)
            e = epsp::launch_convert_f32_to_f16(static_cast<const float*>(v) + (size_t)conv_from * row,
                                                shv + (size_t)conv_from * row * 2, (int64_t)(kv_len - conv_from) * row,
                                                ctx->d_err, s);
        const size_t qbytes = (size_t)n_tok * cf.n_head * d * 2;
        if (e == cudaSuccess && ctx->sh_q_bytes < qbytes) {
            if (ctx->sh_q) cudaFreeAsync(ctx->sh_q, s);
            ctx->sh_q = nullptr;
            ctx->sh_q_bytes = 0;
            e = cudaMallocAsync(&ctx->sh_q, qbytes, s);
            if (e == cudaSuccess) ctx->sh_q_bytes = qbytes;
        }
        if (e == cudaSuccess)
            e = epsp::launch_convert_f32_to_f16(static_cast<const float*>(q), ctx->sh_q, (int64_t)n_tok * cf.n_head * d,
                                                ctx->d_err, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "f16 shadow");
        ctx->shadowed[layer] = kv_len;
        ctx->att_q = ctx->sh_q;
        ctx->att_k = shk;
        ctx->att_v = shv;
        ctx->att_dtype = EP_SP_F16;
    }

    // K1: pool the pages completed so far that are not pooled yet (per KV
    // head watermarks; heads of the range that are ahead are re-pooled to the
    // same values).
    // A layer whose cache is written through ep_sp_append_kv keeps exact
    // watermarks; otherwise the pages from the call's first row on are pooled
    // again, since the caller may have rewritten them.
    int32_t* pooled = ctx->pooled.data() + (size_t)layer * Hkv;
    const bool trusted = ctx->appended[layer] != 0;
    int32_t pg_begin = trusted ? kv_len / P : u0 / P;
    for (int32_t h = hb; h < he; ++h) {
        if (u0 == 0 && !trusted) pooled[h] = 0;
        pg_begin = std::min(pg_begin, pooled[h]);
    }
    const int32_t pg_end = kv_len / P;
    if (active) {
        epsp::PoolArgs pa;
        pa.k = k;
        pa.dtype = cf.dtype;
        pa.n_head_kv = Hkv;
        pa.head_dim = d;
        pa.page_size = P;
        pa.page_begin = pg_begin;
        pa.page_end = pg_end;
        pa.max_pages = ctx->max_pages;
        pa.psum = ctx->psum + (size_t)layer * Hkv * d * ctx->max_pages;
        pa.head_begin = hb;
        pa.head_count = he - hb;
        pa.err = ctx->d_err;
        pa.timeout_ns = ctx->timeout_ns;
        pa.paging = ctx->paging;
        if (pg_end > pg_begin) {
            cudaError_t e = timed(ctx, 0, s, [&] { return epsp::launch_pool_pages(pa, s); });
            if (e != cudaSuccess) return cuda_fail(ctx, e, "K1 page sums");
        }
        for (int32_t h = hb; h < he; ++h) pooled[h] = pg_end;
    } else {
        for (int32_t h = hb; h < he; ++h) pooled[h] = pg_begin;  // pooled from here on once gating is armed
    }
    // V page sums for the pooled rows, with watermarks of their own (an
    // appended cache writes V without summing it)
    int32_t* v_pooled = ctx->v_pooled.data() + (size_t)layer * Hkv;
    int32_t vg_begin = u0 / P;
    for (int32_t h = hb; h < he; ++h) {
        if (u0 == 0) v_pooled[h] = 0;
        vg_begin = std::min(vg_begin, v_pooled[h]);
    }
    if (active && max_pool > 0) {
        if (!ctx->vsum) {
            const size_t bytes = (size_t)cf.n_layer * Hkv * d * ctx->max_pages * sizeof(double);
            cudaError_t e = cudaMalloc(&ctx->vsum, bytes);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc V page sums");
            std::fill(ctx->v_pooled.begin(), ctx->v_pooled.end(), 0);
            vg_begin = 0;
        }
        epsp::PoolArgs pv;
        pv.k = v;
        pv.dtype = cf.dtype;
        pv.n_head_kv = Hkv;
        pv.head_dim = d;
        pv.page_size = P;
        pv.page_begin = vg_begin;
        pv.page_end = pg_end;
        pv.max_pages = ctx->max_pages;
        pv.psum = ctx->vsum + (size_t)layer * Hkv * d * ctx->max_pages;
        pv.head_begin = hb;
        pv.head_count = he - hb;
        pv.err = ctx->d_err;
        pv.timeout_ns = ctx->timeout_ns;
        pv.paging = ctx->paging;
        if (pg_end > vg_begin) {
            cudaError_t e = timed(ctx, 0, s, [&] { return epsp::launch_pool_pages(pv, s); });
            if (e != cudaSuccess) return cuda_fail(ctx, e, "K1 V page sums");
        }
        for (int32_t h = hb; h < he; ++h) v_pooled[h] = pg_end;
    } else if (!active) {
        for (int32_t h = hb; h < he; ++h) v_pooled[h] = std::min(v_pooled[h], vg_begin);
    }

    // K2: score + select per gating block.
    int32_t* sel = sel_pages;
    int32_t* cnt = sel_counts;
    int32_t cap = sel_cap;
    ctx->sel_pool_cap = 0;
    ctx->sel_cnt_attn = nullptr;
    ctx->sel_pool_cnt_attn = nullptr;
    if (active && (max_ksel > 0 || max_pool > 0)) {
        if (!sel) {
            cap = std::max(1, max_ksel);
            if ((rc = grow(ctx, &ctx->d_sel, &ctx->d_sel_elems, (size_t)nb * Hkv * cap, s))) return rc;
            if ((rc = grow(ctx, &ctx->d_cnt, &ctx->d_cnt_elems, (size_t)nb * Hkv, s))) return rc;
            sel = ctx->d_sel;
            cnt = ctx->d_cnt;
        }
        if ((rc = grow(ctx, &ctx->d_scores, &ctx->d_scores_elems,
                       epsp::select_scores_elems(nb, Hkv, ctx->max_pages), s)))
            return rc;
        epsp::SelectArgs sa;
        sa.scores = ctx->d_scores;
        sa.max_cand = max_cand;
        sa.score_chunks = 0;
        sa.q = q;
        sa.dtype = cf.dtype;
        sa.n_head = cf.n_head;
        sa.n_head_kv = Hkv;
        sa.head_dim = d;
        sa.u0 = u0;
        sa.n_tok = n_tok;
        sa.q_subblock = ctx->q_subblock;
        sa.gate = gate;
        sa.k_budget = d_budget_layer;
        sa.psum = ctx->psum + (size_t)layer * Hkv * d * ctx->max_pages;
        sa.max_pages = ctx->max_pages;
        sa.sel = sel;
        sa.cnt = cnt;
        sa.sel_cap = cap;
        sa.err = ctx->d_err;
        sa.head_begin = gate.shared ? 0 : hb;
        sa.head_count = gate.shared ? 0 : he - hb;
        const int32_t pool_stride = (max_pool + 127) / 128 * 128;  // whole segments of every page size
        if (routing) {
            if ((rc = grow(ctx, &ctx->d_route, &ctx->d_route_elems, (size_t)nb * Hkv, s))) return rc;
            sa.route_mode = ctx->route_mode;
            sa.route_threshold = ctx->route_threshold;
            sa.route_k = ctx->d_route;
        }
        if (max_pool > 0) {
            if ((rc = grow(ctx, &ctx->d_pool, &ctx->d_pool_elems, (size_t)nb * Hkv * max_pool, s))) return rc;
            if ((rc = grow(ctx, &ctx->d_pool_cnt, &ctx->d_pool_cnt_elems, (size_t)nb * Hkv, s))) return rc;
            sa.pool = ctx->d_pool;
            sa.pool_cnt = ctx->d_pool_cnt;
            sa.pool_cap = max_pool;
        }
        cudaError_t e = timed(ctx, 1, s, [&] { return epsp::launch_select_pages(sa, s); });
        if (e != cudaSuccess) return cuda_fail(ctx, e, "K2 select");
        if (max_pool > 0) {
            // K2c: the pooled rows in the attention's operand type
            const size_t rows = (size_t)nb * pool_stride;
            const size_t half = rows * Hkv * d * esize(ctx->att_dtype);
            if ((rc = grow(ctx, &ctx->d_pkv, &ctx->d_pkv_bytes, 2 * half, s))) return rc;
            epsp::PoolRowArgs pr;
            pr.ksum = sa.psum;
            pr.vsum = ctx->vsum + (size_t)layer * Hkv * d * ctx->max_pages;
            pr.max_pages = ctx->max_pages;
            pr.pool = ctx->d_pool;
            pr.pool_cnt = ctx->d_pool_cnt;
            pr.pool_cap = max_pool;
            pr.n_blocks = nb;
            pr.n_head_kv = Hkv;
            pr.head_dim = d;
            pr.page_size = P;
            pr.pool_stride = pool_stride;
            pr.out_dtype = ctx->att_dtype;
            pr.pk = ctx->d_pkv;
            pr.pv = ctx->d_pkv + half;
            pr.head_begin = hb;
            pr.head_count = he - hb;
            e = timed(ctx, 1, s, [&] { return epsp::launch_build_pooled_rows(pr, s); });
            if (e != cudaSuccess) return cuda_fail(ctx, e, "K2c pooled rows");
            ctx->sel_pool_cap = max_pool;
            ctx->sel_pool_stride = pool_stride;
            ctx->att_pk = pr.pk;
            ctx->att_pv = pr.pv;
        }
        if (routing) {  // K3 reads the routed counts instead of the plan's
            ctx->sel_cnt_attn = cnt;
            ctx->sel_pool_cnt_attn = max_pool > 0 ? ctx->d_pool_cnt : nullptr;
        }
    } else if (sel_counts) {
        cudaError_t e = cudaMemsetAsync(sel_counts, 0, sizeof(int32_t) * nb * Hkv, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "memset counts");
    }
    ctx->sel_ptr = sel ? sel : ctx->d_dense;
    ctx->sel_cap_used = cap > 0 ? cap : 1;
    ctx->sel_n_blocks = nb;
    ctx->sel_budget = d_budget_layer;
    ctx->sel_layer = layer;
    ctx->sel_kv_len = kv_len;
    ctx->sel_n_tok = n_tok;
    ctx->sel_epoch = ctx->epoch;
    ctx->sel_head_begin = hb;
    ctx->sel_head_end = he;
    ctx->sel_valid = true;
    return kOk;
}

int32_t ep_sp_select_layer(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v,
                           int32_t kv_len, int32_t n_tok, int32_t* sel_pages, int32_t* sel_counts, int32_t sel_cap,
                           void* stream) {
    if (!ctx) return kInvalid;
    return select_impl(ctx, layer, q, k, v, kv_len, n_tok, 0, ctx->cfg.n_head_kv, sel_pages, sel_counts, sel_cap,
                       stream);
}

int32_t ep_sp_select_heads(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v,
                           int32_t kv_len, int32_t n_tok, int32_t head_begin, int32_t head_end, void* stream) {
    if (!ctx) return kInvalid;
    return select_impl(ctx, layer, q, k, v, kv_len, n_tok, head_begin, head_end, nullptr, nullptr, 0, stream);
}

int32_t ep_sp_attend_rows(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin,
                          int32_t row_end, void* out, void* stream) {
    if (!ctx) return kInvalid;
    if (!out) return fail(ctx, kInvalid, "null output");
    epsp::AttnArgs aa;
    const int32_t rc = attn_args(ctx, layer, kv_len, n_tok, row_begin, row_end, aa);
    if (rc) return rc;
    aa.out = out;
    return launch_attn(ctx, aa, static_cast<cudaStream_t>(stream));
}

int32_t ep_sp_attend_layer(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k, const void* v,
                           int32_t kv_len, int32_t n_tok, void* out, int32_t* sel_pages, int32_t* sel_counts,
                           int32_t sel_cap, void* stream) {
    if (!ctx) return kInvalid;
    if (!out) return fail(ctx, kInvalid, "null tensor");
    const int32_t rc = ep_sp_select_layer(ctx, layer, q, k, v, kv_len, n_tok, sel_pages, sel_counts, sel_cap, stream);
    if (rc) return rc;
    return ep_sp_attend_rows(ctx, layer, kv_len, n_tok, 0, n_tok, out, stream);
}

int32_t ep_sp_ffn_compact(ep_sp_ctx* ctx, int32_t layer, const void* x, const uint8_t* keep_mask, int32_t n_rows,
                          int32_t hidden, void* x_kept, int32_t* row_ids, int32_t* n_keep, void* stream) {
    if (!ctx) return kInvalid;
    if (layer < 0 || layer >= ctx->cfg.n_layer) return fail(ctx, kInvalid, "layer out of range");
    if (!x || !keep_mask || !x_kept || !row_ids || !n_keep || n_rows < 1 || hidden < 1)
        return fail(ctx, kInvalid, "bad FFN compaction arguments");
    if ((hidden * esize(ctx->cfg.dtype)) % 16) return fail(ctx, kInvalid, "hidden * element size must be a multiple of 16");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    epsp::FfnCompactArgs a;
    a.x = x;
    a.elem_bytes = static_cast<int32_t>(esize(ctx->cfg.dtype));
    a.keep = keep_mask;
    a.n_rows = n_rows;
    a.hidden = hidden;
    a.x_kept = x_kept;
    a.row_ids = row_ids;
    a.n_keep = n_keep;
    a.skip_layer = (ctx->prefill_mode && layer < 64 && ((ctx->ffn_skip >> layer) & 1u)) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = timed(ctx, 3, s, [&] { return epsp::launch_ffn_compact(a, s); });
    if (e != cudaSuccess) return cuda_fail(ctx, e, "K4 compaction");
    return kOk;
}

int32_t ep_sp_ffn_scatter(ep_sp_ctx* ctx, int32_t layer, const void* ffn_out, void* residual, const int32_t* row_ids,
                          const int32_t* n_keep, int32_t n_rows, int32_t hidden, void* stream) {
    if (!ctx) return kInvalid;
    if (layer < 0 || layer >= ctx->cfg.n_layer) return fail(ctx, kInvalid, "layer out of range");
    if (!ffn_out || !residual || !row_ids || !n_keep || n_rows < 1 || hidden < 1)
        return fail(ctx, kInvalid, "bad FFN scatter arguments");
    if ((hidden * esize(ctx->cfg.dtype)) % 16) return fail(ctx, kInvalid, "hidden * element size must be a multiple of 16");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    epsp::FfnScatterArgs a;
    a.ffn_out = ffn_out;
    a.residual = residual;
    a.dtype = ctx->cfg.dtype;
    a.row_ids = row_ids;
    a.n_keep = n_keep;
    a.n_rows = n_rows;
    a.hidden = hidden;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = timed(ctx, 4, s, [&] { return epsp::launch_ffn_scatter(a, s); });
    if (e != cudaSuccess) return cuda_fail(ctx, e, "K4 scatter");
    return kOk;
}

int32_t ep_sp_profile_enable(ep_sp_ctx* ctx, int32_t on) {
    if (!ctx) return kInvalid;
    for (auto& ev : ctx->events) {
        ctx->event_pool.push_back(ev.start);
        ctx->event_pool.push_back(ev.stop);
    }
    ctx->events.clear();
    for (int i = 0; i < EP_SP_NUM_KERNELS; ++i) ctx->launches[i] = 0;
    ctx->profiling = on != 0;
    return kOk;
}

int32_t ep_sp_profile_read(ep_sp_ctx* ctx, double* ms, int64_t* launches) {
    if (!ctx || !ms || !launches) return kInvalid;
    for (int i = 0; i < EP_SP_NUM_KERNELS; ++i) {
        ms[i] = 0.0;
        launches[i] = ctx->launches[i];
    }
    for (auto& ev : ctx->events) {
        cudaError_t e = cudaEventSynchronize(static_cast<cudaEvent_t>(ev.stop));
        if (e != cudaSuccess) return cuda_fail(ctx, e, "profile event");
        float t = 0.f;
        e = cudaEventElapsedTime(&t, static_cast<cudaEvent_t>(ev.start), static_cast<cudaEvent_t>(ev.stop));
        if (e != cudaSuccess) return cuda_fail(ctx, e, "profile elapsed");
        ms[ev.kind] += t;
    }
    return kOk;
}

int32_t ep_sp_layer_work(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, double* out) {
    if (!ctx || !out || layer < 0 || layer >= ctx->cfg.n_layer || n_tok < 1 || kv_len < n_tok) return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    const double b_in = (double)esize(cf.dtype), b_out = (double)esize(cf.out_dtype);
    const int32_t P = cf.page_size, Hkv = cf.n_head_kv, d = cf.head_dim, G = cf.n_head / Hkv;
    const int32_t u0 = kv_len - n_tok;
    const bool active = gating_active(ctx);
    const epsp::GateParams gate = gate_of(ctx);
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    const int32_t L = epsp::block_len(n_tok, ctx->q_subblock);
    for (int i = 0; i < 6; ++i) out[i] = 0.0;
    const int32_t new_pages = kv_len / P - u0 / P;
    if (active) out[0] = (double)new_pages * P * Hkv * d * b_in + (double)new_pages * Hkv * d * 8.0;
    if (active && gate.pool_pages > 0) out[0] *= 2.0;  // V pages are pooled too
    for (int32_t b = 0; b < nb; ++b) {
        const int32_t b0 = u0 + b * L, b1 = std::min(u0 + n_tok, b0 + L);
        const double n_blk = b1 - b0;
        for (int32_t h = 0; h < Hkv; ++h) {
            const int32_t kb = active ? budget_of(ctx, layer, gate.shared ? 0 : h) : -1;
            const epsp::BlockPlan pl = epsp::plan_block(gate, b0, b1, kb);
            double fixed, uniq;  // keys visible to every row of the block; unique rows loaded
            if (pl.gated) {
                fixed = (double)P + (double)pl.k_sel * P + (double)(b0 - pl.lsp * P) + pl.n_pool;
                uniq = (double)P + (double)pl.k_sel * P + (double)(b1 - pl.lsp * P) + pl.n_pool;
                if (pl.k_sel > 0) {
                    const double scored = (double)(pl.lsp - 1) * (gate.shared ? (h == 0 ? Hkv : 0) : 1);
                    out[1] += scored * d * 8.0 + (gate.shared && h ? 0.0 : d * b_in + pl.k_sel * 4.0);
                    out[2] += 2.0 * scored * d;
                }
            } else {
                fixed = (double)b0;
                uniq = (double)b1;
            }
            // rows i in [b0,b1) see fixed + (i - b0 + 1) keys
            const double keys = n_blk * fixed + n_blk * (n_blk + 1) / 2.0;
            out[3] += 4.0 * d * G * keys;
            out[5] += G * keys;
            out[4] += uniq * 2.0 * d * b_in;
        }
    }
    out[4] += (double)n_tok * cf.n_head * d * (b_in + b_out);
    return kOk;
}

int32_t ep_sp_attend_ctas(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                          int32_t cta_end, void* out, void* stream) {
    if (!ctx) return kInvalid;
    if (!out) return fail(ctx, kInvalid, "null output");
    epsp::AttnArgs aa;
    const int32_t rc = cta_args(ctx, layer, kv_len, n_tok, cta_begin, cta_end, aa);
    if (rc) return rc;
    aa.out = out;
    return launch_attn(ctx, aa, static_cast<cudaStream_t>(stream));
}

int32_t ep_sp_append_kv(ep_sp_ctx* ctx, int32_t layer, const void* k_new, const void* v_new, int32_t n_new,
                        void* k_cache, void* v_cache, int32_t kv_pos, void* stream) {
    if (!ctx) return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    if (layer < 0 || layer >= cf.n_layer) return fail(ctx, kInvalid, "layer out of range");
    if (!k_new || !v_new || !k_cache || !v_cache) return fail(ctx, kInvalid, "null tensor");
    if (n_new < 1 || kv_pos < 0 || (int64_t)kv_pos + n_new > cf.max_ctx)
        return fail(ctx, kInvalid, "rows [kv_pos, kv_pos + n_new) must lie in [0, max_ctx)");
    const bool paged = ctx->paging.block_rows > 0;
    if (paged && (int64_t)ctx->paging.n_entries * ctx->paging.block_rows < (int64_t)kv_pos + n_new)
        return fail(ctx, kInvalid, "the block table does not cover rows [kv_pos, kv_pos + n_new)");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t P = cf.page_size, Hkv = cf.n_head_kv, d = cf.head_dim;
    const size_t row_bytes = (size_t)Hkv * d * esize(cf.dtype);
    const int32_t pg_first = kv_pos / P, pg_end = (kv_pos + n_new) / P;  // pages completed by these rows
    const int32_t fused_end = std::max(kv_pos, pg_end * P);               // K rows written by the fused K1
    // V rows and the K rows of an incomplete last page: plain copies on the SMs
    // (a copy engine here would queue behind the caller's host transfers)
    cudaError_t e;
    if (!paged) {
        e = epsp::launch_copy_rows(v_new, static_cast<char*>(v_cache) + (size_t)kv_pos * row_bytes,
                                   (size_t)n_new * row_bytes, s);
        if (e == cudaSuccess && kv_pos + n_new > fused_end)
            e = epsp::launch_copy_rows(static_cast<const char*>(k_new) + (size_t)(fused_end - kv_pos) * row_bytes,
                                       static_cast<char*>(k_cache) + (size_t)fused_end * row_bytes,
                                       (size_t)(kv_pos + n_new - fused_end) * row_bytes, s);
    } else {
        e = epsp::launch_copy_rows_paged(v_new, v_cache, kv_pos, n_new, row_bytes, ctx->paging, ctx->d_err, s);
        if (e == cudaSuccess && kv_pos + n_new > fused_end)
            e = epsp::launch_copy_rows_paged(static_cast<const char*>(k_new) + (size_t)(fused_end - kv_pos) * row_bytes,
                                             k_cache, fused_end, kv_pos + n_new - fused_end, row_bytes, ctx->paging,
                                             ctx->d_err, s);
    }
    if (e != cudaSuccess) return cuda_fail(ctx, e, "KV append copy");
    if (pg_end > pg_first) {
        epsp::PoolArgs pa;
        pa.k = k_cache;
        pa.dtype = cf.dtype;
        pa.n_head_kv = Hkv;
        pa.head_dim = d;
        pa.page_size = P;
        pa.page_begin = pg_first;
        pa.page_end = pg_end;
        pa.max_pages = ctx->max_pages;
        pa.psum = ctx->psum + (size_t)layer * Hkv * d * ctx->max_pages;
        pa.k_new = k_new;
        pa.k_store = k_cache;
        pa.new_begin = kv_pos;
        pa.paging = ctx->paging;
        pa.err = ctx->d_err;
        e = timed(ctx, 0, s, [&] { return epsp::launch_pool_pages(pa, s); });
        if (e != cudaSuccess) return cuda_fail(ctx, e, "K1 append page sums");
    }
    int32_t* pooled = ctx->pooled.data() + (size_t)layer * Hkv;
    for (int32_t h = 0; h < Hkv; ++h) {
        if (kv_pos == 0)
            pooled[h] = pg_end;
        else if (pooled[h] >= pg_first)
            pooled[h] = std::max(pooled[h], pg_end);
        // else: pages before pg_first are missing; the next selection pools from pooled[h]
    }
    ctx->appended[layer] = 1;
    return kOk;
}

int32_t ep_sp_set_attn_tiles(ep_sp_ctx* ctx, int32_t tiles_per_cta) {
    if (!ctx) return kInvalid;
    if (tiles_per_cta != 1 && tiles_per_cta != 2) return fail(ctx, kInvalid, "tiles per CTA must be 1 or 2");
    ctx->attn_tiles = tiles_per_cta;
    ctx->sel_valid = false;  // the CTA grid of a prepared call changes
    return kOk;
}

int32_t ep_sp_get_attn_tiles(const ep_sp_ctx* ctx) { return ctx ? ctx->attn_tiles : 0; }

int32_t ep_sp_set_paged_kv(ep_sp_ctx* ctx, int32_t block_rows, const int32_t* block_table, int32_t n_entries,
                           int32_t pool_rows) {
    if (!ctx) return kInvalid;
    if (block_rows == 0) {
        ctx->paging = epsp::KvPaging{};
    } else {
        if (block_rows < 0 || block_rows % ctx->cfg.page_size)
            return fail(ctx, kInvalid, "block_rows must be a multiple of the page size");
        if (!block_table || n_entries < 1 || pool_rows < block_rows || pool_rows % block_rows)
            return fail(ctx, kInvalid, "a block table of n_entries >= 1 and a pool of whole blocks are needed");
        ctx->paging.table = block_table;
        ctx->paging.block_rows = block_rows;
        ctx->paging.n_entries = n_entries;
        ctx->paging.pool_rows = pool_rows;
    }
    ctx->sel_valid = false;  // the operands of a prepared call change
    return kOk;
}

int32_t ep_sp_set_head_routing(ep_sp_ctx* ctx, int32_t mode, double threshold) {
    if (!ctx) return kInvalid;
    if (mode < 0 || mode > 2 || !std::isfinite(threshold))
        return fail(ctx, kInvalid, "head routing mode must be 0, 1 or 2 with a finite threshold");
    ctx->route_mode = mode;
    ctx->route_threshold = threshold;
    ++ctx->epoch;
    return kOk;
}

int32_t ep_sp_get_head_routing(const ep_sp_ctx* ctx, int32_t* mode, double* threshold) {
    if (!ctx || !mode || !threshold) return kInvalid;
    *mode = ctx->route_mode;
    *threshold = ctx->route_threshold;
    return kOk;
}

int32_t ep_sp_get_pooled_pages(ep_sp_ctx* ctx, int32_t* pages, int32_t* counts, int32_t cap, void* stream) {
    if (!ctx) return kInvalid;
    if (!pages || !counts || cap < 1) return fail(ctx, kInvalid, "pooled pages need pages, counts and cap >= 1");
    if (!ctx->sel_valid) return fail(ctx, kInvalid, "no selection to read the pooled pages of");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t nb = ctx->sel_n_blocks, Hkv = ctx->cfg.n_head_kv;
    cudaError_t e;
    if (ctx->sel_pool_cap == 0) {
        e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * nb * Hkv, s);
    } else {
        if (cap < ctx->sel_pool_cap) return fail(ctx, kInvalid, "cap smaller than a block's pooled pages");
        e = cudaMemcpy2DAsync(pages, sizeof(int32_t) * cap, ctx->d_pool, sizeof(int32_t) * ctx->sel_pool_cap,
                              sizeof(int32_t) * ctx->sel_pool_cap, (size_t)nb * Hkv, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(counts, ctx->d_pool_cnt, sizeof(int32_t) * nb * Hkv, cudaMemcpyDeviceToDevice, s);
    }
    if (e != cudaSuccess) return cuda_fail(ctx, e, "pooled pages copy");
    return kOk;
}

int32_t ep_sp_set_f32_attention(ep_sp_ctx* ctx, int32_t mode) {
    if (!ctx) return kInvalid;
    if (mode != 0 && mode != 1) return fail(ctx, kInvalid, "f32 attention mode must be 0 (f32) or 1 (f16 tensor cores)");
    if (ctx->f32_mode != mode) {
        ctx->f32_mode = mode;
        ctx->sel_valid = false;  // a prepared call's operands change
        std::fill(ctx->shadowed.begin(), ctx->shadowed.end(), 0);
    }
    return kOk;
}

int32_t ep_sp_get_f32_attention(const ep_sp_ctx* ctx) { return ctx ? ctx->f32_mode : 0; }

int32_t ep_sp_attention_grid(const ep_sp_ctx* ctx, int32_t n_tok, int32_t* ctas_per_head) {
    if (!ctx || !ctas_per_head || n_tok < 1) return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    *ctas_per_head = epsp::n_blocks_of(n_tok, ctx->q_subblock) *
                     epsp::attention_ctas_per_block(cf.n_head, cf.n_head_kv, n_tok, ctx->q_subblock, ctx->attn_tiles);
    return kOk;
}

// Cost of one K3 CTA in KV tiles (its kept segments, as the kernel walks
// them) plus a fixed share for setup, the Q load and the epilogue.  Measured
// on B200 (c4 shapes): K3 time is linear in the tiles with 0.4 tiles per CTA
// on top; splitting over n_parts > 1 GPUs adds the exchange epilogue, about
// 0.55 tiles for the own slot and 1.4 tiles per peer with peer stores, and
// about 0.8 tiles in all with one multicast store per chunk (a least-squares
// fit of the 8 ranks' K3 times against their tiles and CTAs on 8 GPUs).
int32_t ep_sp_balance_ctas(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t n_parts,
                           int32_t* cuts) {
    if (!ctx || !cuts || n_parts < 1 || layer < 0 || layer >= ctx->cfg.n_layer || n_tok < 1 || kv_len < n_tok)
        return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    const int32_t Hkv = cf.n_head_kv, G = cf.n_head / Hkv, T = 128 / G, P = cf.page_size;
    const int32_t SEG = P, SPT = 128 / SEG;
    const int32_t u0 = kv_len - n_tok;
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock), L = epsp::block_len(n_tok, ctx->q_subblock);
    const int32_t tpb = epsp::attention_ctas_per_block(cf.n_head, Hkv, n_tok, ctx->q_subblock, ctx->attn_tiles);
    const int32_t span = ctx->attn_tiles * T;  // tokens per CTA
    const bool active = gating_active(ctx);
    const epsp::GateParams gate = gate_of(ctx);
    const double kFixed =
        0.4 + (n_parts > 1 ? (ctx->xchg_mc != nullptr ? 0.8 : 0.55 + 1.4 * (n_parts - 1)) : 0.0);
    std::vector<double> prefix((size_t)Hkv * nb * tpb + 1, 0.0);
    size_t i = 0;
    for (int32_t h = 0; h < Hkv; ++h)
        for (int32_t b = 0; b < nb; ++b) {
            const int32_t b0 = u0 + b * L, b1 = std::min(u0 + n_tok, b0 + L);
            const int32_t kb = active ? budget_of(ctx, layer, gate.shared ? 0 : h) : -1;
            const epsp::BlockPlan pl = epsp::plan_block(gate, b0, b1, kb);
            const int32_t L0 = pl.gated ? pl.lsp * P : 0;
            for (int32_t c = 0; c < tpb; ++c, ++i) {
                const int32_t t0 = b0 + c * span;
                double cost = 0.0;
                if (t0 < b1) {
                    const int32_t t_end = std::min(t0 + span, b1);
                    const int32_t n_loc = (t_end - L0 + SEG - 1) / SEG;
                    const int32_t n_seg = pl.gated ? 1 + pl.k_sel + (pl.n_pool + SEG - 1) / SEG + n_loc : n_loc;
                    cost = (double)((n_seg + SPT - 1) / SPT) + kFixed;
                }
                prefix[i + 1] = prefix[i] + cost;
            }
        }
    const size_t total = i;
    cuts[0] = 0;
    size_t c = 0;
    for (int32_t r = 1; r < n_parts; ++r) {
        const double target = prefix[total] * r / n_parts;
        while (c < total && prefix[c + 1] <= target) ++c;
        // the CTA straddling the target goes to the side it mostly lies on
        if (c < total && target - prefix[c] > prefix[c + 1] - target) ++c;
        cuts[r] = (int32_t)std::max<size_t>(c, (size_t)cuts[r - 1]);
    }
    cuts[n_parts] = (int32_t)total;
    return kOk;
}

int32_t ep_sp_cta_work(const ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                       int32_t cta_end, double* out) {
    if (!ctx || !out || layer < 0 || layer >= ctx->cfg.n_layer || n_tok < 1 || kv_len < n_tok) return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    const int32_t Hkv = cf.n_head_kv, G = cf.n_head / Hkv, T = 128 / G, P = cf.page_size, d = cf.head_dim;
    const int32_t u0 = kv_len - n_tok;
    const int32_t L = epsp::block_len(n_tok, ctx->q_subblock);
    const int32_t tpb = epsp::attention_ctas_per_block(cf.n_head, Hkv, n_tok, ctx->q_subblock, ctx->attn_tiles);
    const int32_t span = ctx->attn_tiles * T;  // tokens per CTA
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    if (cta_begin < 0 || cta_end < cta_begin || cta_end > Hkv * nb * tpb) return kInvalid;
    const bool active = gating_active(ctx);
    const epsp::GateParams gate = gate_of(ctx);
    const double b_in = (double)esize(cf.dtype), b_out = (double)esize(cf.out_dtype);
    double keys = 0.0, rows = 0.0;
    for (int32_t id = cta_begin; id < cta_end; ++id) {
        const int32_t h = id / (nb * tpb), b = (id % (nb * tpb)) / tpb, c = id % tpb;
        const int32_t b0 = u0 + b * L, b1 = std::min(u0 + n_tok, b0 + L);
        const int32_t t0 = b0 + c * span, t1 = std::min(b1, t0 + span);
        if (t0 >= t1) continue;
        const int32_t kb = active ? budget_of(ctx, layer, gate.shared ? 0 : h) : -1;
        const epsp::BlockPlan pl = epsp::plan_block(gate, b0, b1, kb);
        // row i sees fixed + (i - b0 + 1) keys
        const double fixed =
            pl.gated ? (double)P + (double)pl.k_sel * P + (double)(b0 - pl.lsp * P) + pl.n_pool : (double)b0;
        const double n = t1 - t0, first = t0 - b0 + 1;
        keys += G * (n * fixed + n * first + n * (n - 1) / 2.0);
        rows += n * G;
    }
    out[0] = 4.0 * d * keys;                 // K3 flops
    out[1] = rows * d * (b_in + b_out);      // Q read + O written
    out[2] = keys;
    return kOk;
}

// ------------------------------------------------ head-parallel exchange --
int32_t ep_sp_xchg_alloc(ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, void** base, void* ipc_handle) {
    if (!ctx || !base) return kInvalid;
    if (rows < 1 || rows > ctx->cfg.max_ctx || n_slots < 1 || n_slots > kXchgMaxSlots)
        return fail(ctx, kInvalid, "exchange rows must be in [1, max_ctx] and slots in [1, 64]");
    if (ctx->cfg.out_dtype != EP_SP_F16 && ctx->cfg.out_dtype != EP_SP_BF16)
        return fail(ctx, kUnsupported, "the exchange needs a 16-bit out_dtype");
    if (ctx->xchg_base) return fail(ctx, kInvalid, "exchange buffer already allocated");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    const ep_sp_config& cf = ctx->cfg;
    const size_t heads = (size_t)ctx->n_head_kv_total * (cf.n_head / cf.n_head_kv);
    const size_t slot = ((size_t)rows * heads * cf.head_dim * esize(cf.out_dtype) + 4095) & ~(size_t)4095;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, kXchgHeader + slot * n_slots);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc exchange buffer");
    if ((e = cudaMemset(p, 0, kXchgHeader)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(ctx, e, "exchange counters");
    }
    if (ipc_handle) {
        cudaIpcMemHandle_t h;
        if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
            cudaFree(p);
            return cuda_fail(ctx, e, "cudaIpcGetMemHandle");
        }
        static_assert(sizeof(h) == EP_SP_XCHG_HANDLE_BYTES, "IPC handle size");
        std::memcpy(ipc_handle, &h, sizeof h);
    }
    ctx->xchg_base = p;
    ctx->xchg_rows = rows;
    ctx->xchg_slots = n_slots;
    ctx->xchg_slot_bytes = slot;
    ctx->xchg_ranks = 0;
    ctx->xchg_expected.assign(n_slots, 0);
    *base = p;
    return kOk;
}

int32_t ep_sp_xchg_open(ep_sp_ctx* ctx, const void* ipc_handle, void** base) {
    if (!ctx || !ipc_handle || !base) return kInvalid;
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof h);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaIpcOpenMemHandle");
    ctx->xchg_opened.push_back(p);
    *base = p;
    return kOk;
}

int32_t ep_sp_xchg_attach(ep_sp_ctx* ctx, int32_t n_ranks, int32_t rank, void* const* bases) {
    if (!ctx || !bases) return kInvalid;
    if (!ctx->xchg_base) return fail(ctx, kInvalid, "ep_sp_xchg_alloc first");
    if (ctx->xchg_ranks) return fail(ctx, kInvalid, "exchange already attached (allocate a new buffer to re-attach)");
    if (n_ranks < 1 || n_ranks > EP_SP_XCHG_MAX_RANKS || rank < 0 || rank >= n_ranks)
        return fail(ctx, kInvalid, "exchange ranks must be in [1, 8] and rank in [0, n_ranks)");
    if (bases[rank] != ctx->xchg_base) return fail(ctx, kInvalid, "bases[rank] must be this context's buffer");
    for (int32_t r = 0; r < n_ranks; ++r)
        if (!bases[r]) return fail(ctx, kInvalid, "null exchange base");
    ctx->xchg_bases.assign(bases, bases + n_ranks);
    ctx->xchg_ranks = n_ranks;
    ctx->xchg_rank = rank;
    return kOk;
}

int32_t ep_sp_xchg_attach_buffers(ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, int32_t n_ranks, int32_t rank,
                                  void* const* bases, void* mc_base) {
    if (!ctx || !bases) return kInvalid;
    if (ctx->xchg_base) return fail(ctx, kInvalid, "an exchange buffer is already attached");
    if (rows < 1 || rows > ctx->cfg.max_ctx || n_slots < 1 || n_slots > kXchgMaxSlots)
        return fail(ctx, kInvalid, "exchange rows must be in [1, max_ctx] and slots in [1, 64]");
    if (ctx->cfg.out_dtype != EP_SP_F16 && ctx->cfg.out_dtype != EP_SP_BF16)
        return fail(ctx, kUnsupported, "the exchange needs a 16-bit out_dtype");
    if (n_ranks < 1 || n_ranks > EP_SP_XCHG_MAX_RANKS || rank < 0 || rank >= n_ranks)
        return fail(ctx, kInvalid, "exchange ranks must be in [1, 8] and rank in [0, n_ranks)");
    for (int32_t r = 0; r < n_ranks; ++r)
        if (!bases[r] || (reinterpret_cast<uintptr_t>(bases[r]) & 4095))
            return fail(ctx, kInvalid, "exchange bases must be non-null and 4096-byte aligned");
    if (mc_base && (reinterpret_cast<uintptr_t>(mc_base) & 4095))
        return fail(ctx, kInvalid, "the multicast base must be 4096-byte aligned");
    int32_t rc = ensure_device(ctx);
    if (rc) return rc;
    const ep_sp_config& cf = ctx->cfg;
    const size_t heads = (size_t)ctx->n_head_kv_total * (cf.n_head / cf.n_head_kv);
    const size_t slot = ((size_t)rows * heads * cf.head_dim * esize(cf.out_dtype) + 4095) & ~(size_t)4095;
    // the counters of this rank's own buffer start at zero
    cudaError_t e = cudaMemset(bases[rank], 0, kXchgHeader);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "exchange counters");
    ctx->xchg_base = bases[rank];
    ctx->xchg_external = true;
    ctx->xchg_rows = rows;
    ctx->xchg_slots = n_slots;
    ctx->xchg_slot_bytes = slot;
    ctx->xchg_expected.assign(n_slots, 0);
    ctx->xchg_bases.assign(bases, bases + n_ranks);
    ctx->xchg_ranks = n_ranks;
    ctx->xchg_rank = rank;
    ctx->xchg_mc = mc_base;
    return kOk;
}

int32_t ep_sp_xchg_bytes(const ep_sp_ctx* ctx, int32_t rows, int32_t n_slots, size_t* bytes) {
    if (!ctx || !bytes || rows < 1 || n_slots < 1) return kInvalid;
    const ep_sp_config& cf = ctx->cfg;
    const size_t heads = (size_t)ctx->n_head_kv_total * (cf.n_head / cf.n_head_kv);
    const size_t slot = ((size_t)rows * heads * cf.head_dim * esize(cf.out_dtype) + 4095) & ~(size_t)4095;
    *bytes = kXchgHeader + slot * (size_t)n_slots;
    return kOk;
}

int32_t ep_sp_xchg_slot(const ep_sp_ctx* ctx, int32_t slot, void** data) {
    if (!ctx || !data || !ctx->xchg_base || slot < 0 || slot >= ctx->xchg_slots) return kInvalid;
    *data = static_cast<char*>(ctx->xchg_base) + kXchgHeader + (size_t)slot * ctx->xchg_slot_bytes;
    return kOk;
}

// (token, query head) rows the K3 CTAs of `aa` store.
uint64_t stored_rows(const ep_sp_ctx* ctx, const epsp::AttnArgs& aa) {
    const ep_sp_config& cf = ctx->cfg;
    const int32_t G = cf.n_head / cf.n_head_kv, T = 128 / G;
    const int32_t L = epsp::block_len(aa.n_tok, aa.q_subblock);
    const int32_t tpb = epsp::attention_ctas_per_block(cf.n_head, cf.n_head_kv, aa.n_tok, aa.q_subblock, aa.tiles_per_cta);
    const int32_t span = aa.tiles_per_cta * T;
    const int64_t per_head = (int64_t)aa.blk_count * tpb;
    const int64_t end = aa.cta_count > 0 ? aa.cta_begin + aa.cta_count : per_head * cf.n_head_kv;
    uint64_t rows = 0;
    for (int64_t id = aa.cta_begin; id < end; ++id) {
        const int32_t b = aa.blk_begin + (int32_t)((id % per_head) / tpb), c = (int32_t)(id % tpb);
        const int32_t b0 = aa.u0 + b * L, b1 = std::min(aa.u0 + aa.n_tok, b0 + L);
        const int32_t t0 = b0 + c * span;
        if (t0 < b1) rows += (uint64_t)(std::min(b1, t0 + span) - t0) * G;
    }
    return rows;
}

// Exchange-mode K3 of prepared arguments into slot `slot` of every attached
// rank's buffer, then the signal that adds its rows to every rank's counter.
int32_t launch_xchg(ep_sp_ctx* ctx, epsp::AttnArgs& aa, int32_t slot, void* stream) {
    const int32_t G = ctx->cfg.n_head / ctx->cfg.n_head_kv;
    aa.out_heads = ctx->n_head_kv_total * G;
    aa.out_head0 = ctx->cfg.kv_head_offset * G;
    aa.n_dest = ctx->xchg_ranks;
    unsigned long long* sig[epsp::kMaxDest];
    for (int32_t r = 0; r < ctx->xchg_ranks; ++r) {
        char* b = static_cast<char*>(ctx->xchg_bases[r]);
        aa.dest[r] = b + kXchgHeader + (size_t)slot * ctx->xchg_slot_bytes;
        sig[r] = reinterpret_cast<unsigned long long*>(b) + slot;
    }
    aa.mc_dest = ctx->xchg_mc ? static_cast<char*>(ctx->xchg_mc) + kXchgHeader + (size_t)slot * ctx->xchg_slot_bytes
                              : nullptr;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t rc = launch_attn(ctx, aa, s);
    if (rc) return rc;
    const uint64_t rows = stored_rows(ctx, aa);
    const cudaError_t e = timed(ctx, 5, s, [&] { return epsp::launch_exchange_signal(sig, ctx->xchg_ranks, rows, s); });
    if (e != cudaSuccess) return cuda_fail(ctx, e, "exchange signal");
    return kOk;
}

int32_t xchg_check(ep_sp_ctx* ctx, int32_t slot, int32_t n_tok) {
    if (!ctx->xchg_ranks) return fail(ctx, kInvalid, "exchange not attached");
    if (slot < 0 || slot >= ctx->xchg_slots) return fail(ctx, kInvalid, "exchange slot out of range");
    if (n_tok > ctx->xchg_rows) return fail(ctx, kInvalid, "n_tok exceeds the exchange buffer's rows");
    return kOk;
}

int32_t ep_sp_attend_rows_xchg(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t row_begin,
                               int32_t row_end, int32_t slot, void* stream) {
    if (!ctx) return kInvalid;
    int32_t rc = xchg_check(ctx, slot, n_tok);
    if (rc) return rc;
    epsp::AttnArgs aa;
    if ((rc = attn_args(ctx, layer, kv_len, n_tok, row_begin, row_end, aa))) return rc;
    return launch_xchg(ctx, aa, slot, stream);
}

int32_t ep_sp_attend_ctas_xchg(ep_sp_ctx* ctx, int32_t layer, int32_t kv_len, int32_t n_tok, int32_t cta_begin,
                               int32_t cta_end, int32_t slot, void* stream) {
    if (!ctx) return kInvalid;
    int32_t rc = xchg_check(ctx, slot, n_tok);
    if (rc) return rc;
    epsp::AttnArgs aa;
    if ((rc = cta_args(ctx, layer, kv_len, n_tok, cta_begin, cta_end, aa))) return rc;
    return launch_xchg(ctx, aa, slot, stream);
}

int32_t ep_sp_xchg_wait(ep_sp_ctx* ctx, int32_t slot, int32_t rows, void* stream) {
    if (!ctx) return kInvalid;
    if (!ctx->xchg_ranks) return fail(ctx, kInvalid, "exchange not attached");
    if (slot < 0 || slot >= ctx->xchg_slots) return fail(ctx, kInvalid, "exchange slot out of range");
    if (rows < 1 || rows > ctx->xchg_rows) return fail(ctx, kInvalid, "rows must be in [1, exchange rows]");
    const int32_t G = ctx->cfg.n_head / ctx->cfg.n_head_kv;
    ctx->xchg_expected[slot] += (uint64_t)rows * (uint64_t)ctx->n_head_kv_total * (uint64_t)G;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto* sig = reinterpret_cast<const unsigned long long*>(ctx->xchg_base) + slot;
    const cudaError_t e = timed(ctx, 5, s, [&] {
        return epsp::launch_exchange_wait(sig, ctx->xchg_expected[slot], ctx->d_err, ctx->timeout_ns, s);
    });
    if (e != cudaSuccess) return cuda_fail(ctx, e, "exchange wait");
    return kOk;
}

}  // extern "C"
