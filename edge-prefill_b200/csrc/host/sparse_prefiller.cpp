// sparse_prefiller.cpp -- the native chunk loop of SparsePrefiller for the
// bound-gated attention path (src/sparse_prefill.cpp:133-148 arming,
// :21-32/:235 prefill-mode guard, :252-262 unconditional disarm, :352-487 the
// ubatch loop with its chunk clamp and per-chunk audit).  The reference runs
// llama_decode per chunk (every layer inside); here every layer of the chunk
// is one ep_sp_attend_layer call on the caller's stream.
#include <cstdint>
#include <string>
#include <vector>

#include "epsp_host.h"

using namespace edge_prefill_b200;

namespace {

class PrefillModeGuard {
public:
    explicit PrefillModeGuard(ep_sp_ctx* c) : c_(c) { ep_sp_set_prefill_mode(c_, 1); }
    ~PrefillModeGuard() { ep_sp_set_prefill_mode(c_, 0); }

private:
    ep_sp_ctx* c_;
};

}  // namespace

extern "C" int32_t ep_sp_prefill(ep_sp_ctx* ctx, const ep_sp_prefill_options* opts, int32_t n_layers,
                                 const void* const* q, const void* const* k, const void* const* v, void* const* out,
                                 int32_t n_tokens, int32_t n_ubatch, ep_sp_prefill_stats* stats, void* stream) {
    if (!ctx || !opts || !stats) return static_cast<int32_t>(ErrorCode::InvalidArgument);
    if (n_layers < 1 || n_layers > ctx->cfg.n_layer || !q || !k || !v || !out)
        return static_cast<int32_t>(ErrorCode::InvalidArgument);
    if (n_tokens < 1 || n_tokens > ctx->cfg.max_ctx || n_ubatch < 1)
        return static_cast<int32_t>(ErrorCode::InvalidArgument);
    *stats = ep_sp_prefill_stats{};

    // Arm once per prefill; a rejected arming degrades (here: dense attention)
    // with a warning and never fails the request.
    bool bound_active = false;
    if (opts->enable_qg_bound) {
        const int32_t rc = ep_sp_set_qg_bound(ctx, 1, static_cast<int32_t>(opts->qg_sel_pages),
                                              static_cast<int32_t>(opts->qg_local_rows),
                                              static_cast<int32_t>(opts->qg_pool_pages));
        if (rc != 0) {
            log_warn("bound gating unavailable (rc " + std::to_string(rc) + "); running dense attention");
            stats->attn_fallback = 1;
        } else {
            bound_active = true;
            stats->query_gating = 1;
            stats->qg_groups = 1;
        }
    }

    // Gating is chunk-scoped, so the chunk never exceeds n_ubatch.
    uint32_t attn_chunk = opts->enable_chunking ? opts->chunk_size : 0;
    if (attn_chunk > static_cast<uint32_t>(n_ubatch)) {
        log_warn("attn chunk_size " + std::to_string(attn_chunk) + " exceeds n_ubatch " + std::to_string(n_ubatch) +
                 "; clamping to n_ubatch");
        attn_chunk = static_cast<uint32_t>(n_ubatch);
    }
    std::vector<Range> ranges;
    Status st = ChunkScheduler::plan(static_cast<uint32_t>(n_tokens), attn_chunk, static_cast<uint32_t>(n_ubatch),
                                     &ranges);
    int32_t rc = static_cast<int32_t>(st.code);
    if (st.ok()) {
        PrefillModeGuard guard(ctx);
        ep_sp_reset(ctx);
        stats->chunks = static_cast<uint32_t>(ranges.size());
        const size_t qrow = (size_t)ctx->cfg.n_head * ctx->cfg.head_dim;
        const size_t esz_in = ctx->cfg.dtype == EP_SP_F32 ? 4 : 2;
        const size_t esz_out = ctx->cfg.out_dtype == EP_SP_F32 ? 4 : 2;
        for (const Range& r : ranges) {
            for (int32_t l = 0; l < n_layers && rc == 0; ++l) {
                const char* ql = static_cast<const char*>(q[l]) + (size_t)r.begin * qrow * esz_in;
                char* ol = static_cast<char*>(out[l]) + (size_t)r.begin * qrow * esz_out;
                rc = ep_sp_attend_layer(ctx, l, ql, k[l], v[l], static_cast<int32_t>(r.end),
                                        static_cast<int32_t>(r.size()), ol, nullptr, nullptr, 0, stream);
            }
            if (rc != 0) break;
            // Audit of the gathered width (src/sparse_prefill.cpp:469-474), in rows.
            stats->chunk_attn_rows =
                bound_active ? (opts->qg_local_rows > 0 ? opts->qg_local_rows : r.size()) +
                                   static_cast<uint32_t>(ctx->cfg.page_size) * (1 + opts->qg_sel_pages)
                             : r.end;
        }
    }
    // Always restore the dense path.
    ep_sp_set_qg_bound(ctx, 0, 0, 0, 0);
    return rc;
}
