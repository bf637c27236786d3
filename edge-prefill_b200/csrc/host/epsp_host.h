// epsp_host.h -- C++17 host layer behind the C ABI (include/epsp.h).
//
// Mirrors the reference's operator surface for the page-gated path:
//   Status / ErrorCode            include/edge_prefill/status.h:7-34
//   ChunkScheduler::plan          src/chunk_scheduler.cpp:9-45
//   FfnSkipController             src/ffn_skip.cpp:41-117
//   SparsePrefiller (bound path)  src/sparse_prefill.cpp:39-294, 352-487
// and holds the per-context state the patched llama_context kept in its
// cparams (patch :567-584, :504-517).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../../../include/epsp.h"
#include "../epsp_plan.h"

namespace edge_prefill_b200 {

enum class ErrorCode : int32_t {
    Ok = 0,
    InvalidArgument = 2,
    ModelLoad = 3,
    Tokenize = 4,
    ContextInit = 5,
    Prefill = 6,
    Decode = 7,
    Cache = 8,
    Unsupported = 9,
    OutOfMemory = 10,
    Io = 11,
    Internal = 12,
    Unavailable = 13,
};

struct Status {
    ErrorCode code = ErrorCode::Ok;
    std::string message;
    bool ok() const noexcept { return code == ErrorCode::Ok; }
    static Status success() { return {}; }
    static Status error(ErrorCode c, std::string m) { return Status{c, std::move(m)}; }
};

const char* error_code_name(ErrorCode code);

struct Range {
    uint32_t begin = 0;
    uint32_t end = 0;
    uint32_t size() const { return end - begin; }
};

class ChunkScheduler {
public:
    static Status plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch, std::vector<Range>* out);
};

class FfnSkipController {
public:
    static Status auto_mask(int32_t n_layer, double ratio, uint64_t* out);
    static Status parse(const std::string& spec, int32_t n_layer, uint64_t* out, std::string* warning);
};

void log_warn(const std::string& msg);

}  // namespace edge_prefill_b200

// The opaque context of the C ABI.
struct ep_sp_ctx {
    ep_sp_config cfg{};
    int32_t n_head_kv_total = 0;

    // bound gating (llama_cparams prefill_qg_bound*, patch :567-584)
    int32_t qg_bound = 0;
    int32_t sel_pages = 8;
    int32_t local_pages = 0;
    int32_t pool_pages = 0;
    uint64_t epoch = 0;
    // extended semantics; defaults reproduce the reference
    int32_t per_kv_head = 0;
    int32_t q_subblock = 0;
    int32_t max_gather_rows = 4096;
    std::vector<int32_t> k_matrix;  // [n_layer][n_head_kv_total], empty = unset
    // prefill mode / FFN skip (ffn patch :9-21)
    int32_t prefill_mode = 0;
    uint64_t ffn_skip = 0;

    std::string last_error;

    // device state (reserved lazily)
    bool reserved = false;
    int32_t max_pages = 0;
    double* psum = nullptr;              // [n_layer][Hkv][max_pages][d]
    std::vector<int32_t> pooled;         // per (layer, KV head): pages [0, pooled) summed
    double* vsum = nullptr;              // V page sums for pooled rows (allocated on first use)
    std::vector<int32_t> v_pooled;       // per (layer, KV head): V pages [0, v_pooled) summed
    int32_t* d_pool = nullptr;           // pooled page lists [n_blocks][Hkv][pool_cap]
    size_t d_pool_elems = 0;
    int32_t* d_pool_cnt = nullptr;       // [n_blocks][Hkv]
    size_t d_pool_cnt_elems = 0;
    unsigned char* d_pkv = nullptr;      // pooled K rows then V rows [n_blocks * pool_stride][Hkv][d]
    size_t d_pkv_bytes = 0;
    std::vector<uint8_t> appended;       // per layer: cache written through ep_sp_append_kv
    int32_t* d_budget = nullptr;         // [n_layer][Hkv] armed budgets
    int32_t* d_dense = nullptr;          // [Hkv] all -1
    std::vector<int32_t> h_budget;       // host copy of d_budget
    uint64_t budget_epoch = ~0ull;       // epoch d_budget was built for
    int32_t* d_sel = nullptr;            // selection workspace
    size_t d_sel_elems = 0;
    int32_t* d_cnt = nullptr;
    size_t d_cnt_elems = 0;
    double* d_scores = nullptr;          // K2a page scores workspace
    size_t d_scores_elems = 0;
    int32_t* d_err = nullptr;            // device error word
    // f32 contexts: attention in fp32 on the CUDA cores (mode 0, the default)
    // or on f16 shadows for the tensor-core kernel (mode 1)
    int32_t f32_mode = 0;
    void* sh_q = nullptr;
    size_t sh_q_bytes = 0;
    void* sh_k = nullptr;                // [n_layer][max_ctx][Hkv][d] f16
    void* sh_v = nullptr;
    std::vector<int32_t> shadowed;       // per layer: rows [0, shadowed) converted
    uint64_t timeout_ns = 2000000000ull;
    int32_t attn_tiles = 2;              // query tiles per K3 CTA (ep_sp_set_attn_tiles)

    // the last selection (ep_sp_select_layer), consumed by ep_sp_attend_rows
    bool sel_valid = false;
    int32_t sel_layer = -1, sel_kv_len = 0, sel_n_tok = 0;
    uint64_t sel_epoch = 0;
    int32_t sel_head_begin = 0, sel_head_end = 0;  // KV heads the selection covers
    const int32_t* sel_ptr = nullptr;
    int32_t sel_cap_used = 1;
    const int32_t* sel_budget = nullptr;
    epsp::KvPaging paging;               // paged KV pools (ep_sp_set_paged_kv); block_rows 0: contiguous
    int32_t route_mode = 0;              // per-KV-head routing by score spread (ep_sp_set_head_routing)
    double route_threshold = 0.0;
    int32_t* d_route = nullptr;          // routed budgets [n_blocks][Hkv]
    size_t d_route_elems = 0;
    const int32_t* sel_cnt_attn = nullptr;       // counts K3 must read (routing), else null
    const int32_t* sel_pool_cnt_attn = nullptr;
    int32_t sel_pool_cap = 0;            // pooled lists of the last selection (0: none)
    int32_t sel_pool_stride = 0;
    int32_t sel_n_blocks = 0;
    const void* att_pk = nullptr;
    const void* att_pv = nullptr;
    const void* att_q = nullptr;
    const void* att_k = nullptr;
    const void* att_v = nullptr;
    int32_t att_dtype = 0;

    // kernel timing (ep_sp_profile_*)
    bool profiling = false;
    struct Ev {
        int kind;
        void* start;
        void* stop;
    };
    std::vector<Ev> events;       // recorded since the last enable
    std::vector<void*> event_pool;
    int64_t launches[EP_SP_NUM_KERNELS] = {0, 0, 0, 0, 0, 0};

    // head-parallel output exchange (ep_sp_xchg_*)
    void* xchg_base = nullptr;            // this rank's buffer: [header][slots]
    int32_t xchg_rows = 0, xchg_slots = 0;
    size_t xchg_slot_bytes = 0;
    int32_t xchg_ranks = 0, xchg_rank = -1;  // 0: not attached
    std::vector<void*> xchg_bases;        // every rank's buffer as mapped here
    std::vector<void*> xchg_opened;       // IPC mappings to close
    std::vector<uint64_t> xchg_expected;  // per slot: counter value once all calls so far landed
    void* xchg_mc = nullptr;              // multicast mapping of every rank's buffer (or null)
    bool xchg_external = false;           // buffers owned by the caller (ep_sp_xchg_attach_buffers)
};
