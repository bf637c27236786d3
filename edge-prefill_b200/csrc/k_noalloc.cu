// k_noalloc.cu -- page selection that allocates no device memory.
//
// Some callers cannot allocate device memory at the point where they need a
// page selection.  The typical one is an operator callback inside a graph
// executor such as ggml's (llama_decode's graph compute): the executor plans
// and reserves every buffer before the graph runs, hands the operator only its
// input and output tensors, and a cudaMalloc from inside the callback would
// implicitly synchronise the device and fall outside that memory plan.  Hosts
// with a fixed device-memory budget are in the same position.  For them this
// entry point runs the selection path (K1 page sums, then K2 score + top-k)
// with all its scratch in one file-scope device array of fixed size.
//
// Scratch layout (kNoAllocScratchBytes, allocated once per device when the
// library's module loads, held until the process exits):
//   [0, 4)            device error word (cleared at the start of every call;
//                     ep_sp_sync_status reads and clears it)
//   [256, 1280)       per-KV-head top-k budgets of the call (int32, <= 256 heads),
//                     written by a one-CTA kernel that receives them by value in
//                     its parameters, so no host buffer has to outlive the call
//   [2048, ...)       fp64 page sums [Hkv][n_scored_pages][d]
//   then              fp64 page scores [n_blocks][Hkv][n_scored_pages]
// Every call overwrites what it reads, so nothing depends on an earlier call's
// contents; but all calls share the array: two calls whose work overlaps on
// the GPU (different streams, or different host threads) race on it.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "epsp_kernels.h"
#include "epsp_plan.h"
#include "host/epsp_host.h"

namespace {

constexpr size_t kNoAllocScratchBytes = EP_SP_NOALLOC_SCRATCH_BYTES;
constexpr size_t kErrOffset = 0;
constexpr size_t kBudgetOffset = 256;
constexpr int kMaxHeads = 256;
constexpr size_t kPsumOffset = 2048;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The call's budgets travel in the kernel's parameters (copied at launch), not
// through a host-to-device copy of a host buffer.
struct NoAllocBegin {
    int32_t n_heads;
    int32_t budget[kMaxHeads];
};

__global__ void k_noalloc_begin(const __grid_constant__ NoAllocBegin a, int32_t* err, int32_t* budget) {
    for (int h = threadIdx.x; h < a.n_heads; h += blockDim.x) budget[h] = a.budget[h];
    if (threadIdx.x == 0) *err = 0;
}

// Device address of the scratch array per device ordinal, looked up once per
// device (with that device current) on the first call.  In host code the
// array's name is only a host-side stand-in, never a device address.
std::mutex g_mu;
std::vector<void*> g_scratch_addr;

int32_t scratch_for_current_device(void** out, std::string* why) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *why = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
        return EP_SP_UNAVAILABLE;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if ((int)g_scratch_addr.size() <= dev) g_scratch_addr.resize(dev + 1, nullptr);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            *why = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
            return EP_SP_INTERNAL;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return EP_SP_OK;
}

}  // namespace

namespace epsp {
// Reads and clears the no-allocation path's device error word on the current
// device.  *word = 0 when that device never ran the path.
cudaError_t noalloc_take_error_word(int32_t* word) {
    *word = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    void* p = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (dev < (int)g_scratch_addr.size()) p = g_scratch_addr[dev];
    }
    if (!p) return cudaSuccess;
    e = cudaMemcpy(word, static_cast<unsigned char*>(p) + kErrOffset, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && *word != 0) e = cudaMemset(static_cast<unsigned char*>(p) + kErrOffset, 0, sizeof(int32_t));
    return e;
}
}  // namespace epsp

extern "C" int32_t ep_sp_select_pages_noalloc(ep_sp_ctx* ctx, int32_t layer, const void* q, const void* k,
                                              int32_t kv_len, int32_t n_tok, int32_t* sel_pages,
                                              int32_t* sel_counts, int32_t sel_cap, void* stream) {
    if (!ctx) return EP_SP_INVALID_ARGUMENT;
    auto fail = [&](int32_t rc, const std::string& m) {
        ctx->last_error = m;
        return rc;
    };
    const ep_sp_config& cf = ctx->cfg;
    if (layer < 0 || layer >= cf.n_layer) return fail(EP_SP_INVALID_ARGUMENT, "layer out of range");
    if (!q || !k || !sel_pages || !sel_counts || sel_cap < 1) return fail(EP_SP_INVALID_ARGUMENT, "null tensor");
    if (n_tok < 1 || kv_len < n_tok || kv_len > cf.max_ctx) return fail(EP_SP_INVALID_ARGUMENT, "bad kv_len / n_tok");
    if (ctx->paging.block_rows > 0 && (int64_t)ctx->paging.n_entries * ctx->paging.block_rows < kv_len)
        return fail(EP_SP_INVALID_ARGUMENT, "the block table does not cover kv_len rows");
    if (cf.n_head_kv > kMaxHeads) return fail(EP_SP_INVALID_ARGUMENT, "more than 256 KV heads");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != cf.device)
        return fail(EP_SP_INVALID_ARGUMENT, "call with the context's device current");

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int32_t P = cf.page_size, Hkv = cf.n_head_kv, d = cf.head_dim;
    const int32_t u0 = kv_len - n_tok;
    const int32_t nb = epsp::n_blocks_of(n_tok, ctx->q_subblock);
    const int32_t L = epsp::block_len(n_tok, ctx->q_subblock);
    epsp::GateParams gate;
    gate.page_size = P;
    gate.local_pages = ctx->local_pages;
    gate.shared = ctx->per_kv_head ? 0 : 1;
    gate.max_gather_rows = ctx->max_gather_rows;
    const bool active = ctx->prefill_mode && ctx->qg_bound;

    if (active && gate.shared && Hkv < ctx->n_head_kv_total)
        return fail(EP_SP_UNSUPPORTED, "shared (reference) selection needs every KV head in one context");
    if (!active) {  // nothing is gated: every count is zero, as in ep_sp_attend_layer
        const cudaError_t e = cudaMemsetAsync(sel_counts, 0, sizeof(int32_t) * nb * Hkv, s);
        return e == cudaSuccess ? EP_SP_OK : fail(EP_SP_INTERNAL, cudaGetErrorString(e));
    }

    NoAllocBegin begin{};
    begin.n_heads = Hkv;
    int32_t* budget = begin.budget;
    for (int32_t h = 0; h < Hkv; ++h)
        budget[h] = ctx->k_matrix.empty()
                        ? ctx->sel_pages
                        : ctx->k_matrix[(size_t)layer * ctx->n_head_kv_total + cf.kv_head_offset + h];
    int32_t max_ksel = 0, max_lsp = 0;
    for (int32_t b = 0; b < nb; ++b) {
        const int32_t b0 = u0 + b * L, b1 = std::min(u0 + n_tok, b0 + L);
        for (int32_t h = 0; h < (gate.shared ? 1 : Hkv); ++h) {
            const epsp::BlockPlan pl = epsp::plan_block(gate, b0, b1, budget[h]);
            if (pl.gated && pl.k_sel > 0) {
                max_ksel = std::max(max_ksel, pl.k_sel);
                max_lsp = std::max(max_lsp, pl.lsp);
            }
        }
    }
    if (max_ksel > sel_cap) return fail(EP_SP_INVALID_ARGUMENT, "sel_cap smaller than a block's k_sel");
    const size_t psum_bytes = (size_t)Hkv * d * std::max(1, max_lsp) * sizeof(double);
    const size_t score_bytes = epsp::select_scores_elems(nb, Hkv, std::max(1, max_lsp)) * sizeof(double);
    const size_t need = kPsumOffset + psum_bytes + score_bytes;
    if (need > kNoAllocScratchBytes)
        return fail(EP_SP_INVALID_ARGUMENT, "page sums and scores of " + std::to_string(max_lsp) + " pages x " +
                                                std::to_string(Hkv) + " heads x d " + std::to_string(d) +
                                                " exceed the no-allocation scratch (" +
                                                std::to_string(kNoAllocScratchBytes) + " bytes)");
    if (max_ksel == 0) {
        const cudaError_t e = cudaMemsetAsync(sel_counts, 0, sizeof(int32_t) * nb * Hkv, s);
        return e == cudaSuccess ? EP_SP_OK : fail(EP_SP_INTERNAL, cudaGetErrorString(e));
    }

    void* base = nullptr;
    std::string why;
    const int32_t rc = scratch_for_current_device(&base, &why);
    if (rc != EP_SP_OK) return fail(rc, why);
    unsigned char* scratch = static_cast<unsigned char*>(base);
    int32_t* d_err = reinterpret_cast<int32_t*>(scratch + kErrOffset);
    int32_t* d_budget = reinterpret_cast<int32_t*>(scratch + kBudgetOffset);
    double* psum = reinterpret_cast<double*>(scratch + kPsumOffset);
    double* scores = reinterpret_cast<double*>(scratch + kPsumOffset + psum_bytes);

    k_noalloc_begin<<<1, 256, 0, s>>>(begin, d_err, d_budget);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(EP_SP_INTERNAL, cudaGetErrorString(e));

    // K1 over every page a block of this ubatch may score: pages [0, max_lsp).
    epsp::PoolArgs pa;
    pa.k = k;
    pa.dtype = cf.dtype;
    pa.n_head_kv = Hkv;
    pa.head_dim = d;
    pa.page_size = P;
    pa.page_begin = 0;
    pa.page_end = max_lsp;
    pa.max_pages = max_lsp;
    pa.psum = psum;
    pa.err = d_err;
    pa.timeout_ns = 2000000000ull;
    pa.paging = ctx->paging;
    e = epsp::launch_pool_pages(pa, s);
    if (e != cudaSuccess) return fail(EP_SP_INTERNAL, std::string("K1: ") + cudaGetErrorString(e));

    epsp::SelectArgs sa;
    sa.q = q;
    sa.dtype = cf.dtype;
    sa.n_head = cf.n_head;
    sa.n_head_kv = Hkv;
    sa.head_dim = d;
    sa.u0 = u0;
    sa.n_tok = n_tok;
    sa.q_subblock = ctx->q_subblock;
    sa.gate = gate;
    sa.k_budget = d_budget;
    sa.psum = psum;
    sa.max_pages = max_lsp;
    sa.sel = sel_pages;
    sa.cnt = sel_counts;
    sa.sel_cap = sel_cap;
    sa.err = d_err;
    sa.scores = scores;
    sa.max_cand = max_lsp - 1;
    sa.score_chunks = 0;
    e = epsp::launch_select_pages(sa, s);
    if (e != cudaSuccess) return fail(EP_SP_INTERNAL, std::string("K2: ") + cudaGetErrorString(e));
    return EP_SP_OK;
}
