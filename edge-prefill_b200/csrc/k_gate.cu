// k_gate.cu -- K1 page sums and K2 page scoring + top-k page select.
//
// K1 replaces the reference's per-ubatch re-scan of the whole K view
// (ggml_mul_mat(k_p, q_heads) + ggml_sum_rows, patch :1045-1050) by an
// incremental pooling: each ubatch sums only the pages it completes, once, into
// a persistent fp64 buffer laid out [Hkv][d][max_pages] so that K2 reads it
// coalesced.  HBM-bound: every K byte of the ubatch is read once with 16-byte
// vector loads.
//
// K2 restates patch :1040-1058: the gating query is the block's last row at
// the first query head of each KV group; score(page) = q . sum(K_page)
// (the 1/P of a page mean cancels in the ranking, patch :1046-1048); shared
// mode takes the MAX over KV heads (:1053-1055); pages 0 and >= lsp carry the
// -inf bias (:763-766) and are never candidates; top-k ranks by score
// descending with ties toward the lower page (a total order, so the selection
// is deterministic), and the list is emitted sorted by page.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cfloat>
#include <cmath>

#include "epsp_kernels.h"

namespace epsp {
namespace {

constexpr int kPoolThreads = 256;
constexpr int kSelectThreads = 512;
constexpr int kScoreThreads = 256;
constexpr int kScoreGroupCh = 16;  // channels per fma-chain group of a page score

template <int DT>
struct Vec16;  // 16-byte vector of the element type, converted exactly to fp64
template <>
struct Vec16<0> {
    static constexpr int N = 4;
    __device__ static void to_double(const uint4& u, double* out) {
        out[0] = (double)__uint_as_float(u.x);
        out[1] = (double)__uint_as_float(u.y);
        out[2] = (double)__uint_as_float(u.z);
        out[3] = (double)__uint_as_float(u.w);
    }
};
template <>
struct Vec16<1> {
    static constexpr int N = 8;
    __device__ static void to_double(const uint4& u, double* out) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = (double)__half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
            out[2 * i + 1] = (double)__half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
        }
    }
};
template <>
struct Vec16<2> {
    static constexpr int N = 8;
    __device__ static void to_double(const uint4& u, double* out) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = (double)__uint_as_float(w[i] << 16);
            out[2 * i + 1] = (double)__uint_as_float(w[i] & 0xffff0000u);
        }
    }
};

// One thread = (page, KV head, 16-byte channel chunk, 16-row group).  The
// group's rows are summed in ascending order, then thread g == 0 of the
// (page, head, chunk) adds the groups in ascending order.
template <int DT>
__global__ void __launch_bounds__(kPoolThreads) k1_pool_pages(PoolArgs a) {
    constexpr int VEC = Vec16<DT>::N;
    __shared__ double part[kPoolThreads][VEC];
    const int cpr = a.head_dim / VEC;               // chunks per row
    const int ng = a.page_size / kPageSumGroupRows; // row groups per page
    const int tpu = cpr * ng;                       // threads per (page, head)
    const int upc = kPoolThreads / tpu;
    const int tid = threadIdx.x;
    const int ul = tid / tpu;
    const int r = tid % tpu;
    const int g = r / cpr;
    const int c = r % cpr;
    const int hc = a.head_count > 0 ? a.head_count : a.n_head_kv;
    const int64_t n_units = (int64_t)(a.page_end - a.page_begin) * hc;
    const int64_t unit = (int64_t)blockIdx.x * upc + ul;
    const bool valid = ul < upc && unit < n_units;
    int page = 0, h = 0;
    if (valid) {
        page = a.page_begin + (int)(unit / hc);
        h = a.head_begin + (int)(unit % hc);
        constexpr int ESZ = DT == 0 ? 4 : 2;
        const char* base = static_cast<const char*>(a.k);
        const int64_t row0 = (int64_t)page * a.page_size + (int64_t)g * kPageSumGroupRows;
        const int64_t col = ((int64_t)h * a.head_dim + (int64_t)c * VEC) * ESZ;
        const int64_t row_bytes = (int64_t)a.n_head_kv * a.head_dim * ESZ;
        uint4 raw[kPageSumGroupRows];
        if (a.k_new == nullptr) {
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i)
                raw[i] = __ldg(reinterpret_cast<const uint4*>(base + (row0 + i) * row_bytes + col));
        } else {
            // append: the new rows come from k_new and are written to the cache
            const char* nb = static_cast<const char*>(a.k_new);
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i) {
                const int64_t r = row0 + i;
                raw[i] = r >= a.new_begin ? __ldg(reinterpret_cast<const uint4*>(nb + (r - a.new_begin) * row_bytes + col))
                                          : *reinterpret_cast<const uint4*>(base + r * row_bytes + col);
            }
            char* out = static_cast<char*>(a.k_store);
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i)
                if (row0 + i >= a.new_begin) *reinterpret_cast<uint4*>(out + (row0 + i) * row_bytes + col) = raw[i];
        }
        double acc[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = 0.0;
#pragma unroll
        for (int i = 0; i < kPageSumGroupRows; ++i) {
            double x[VEC];
            Vec16<DT>::to_double(raw[i], x);
#pragma unroll
            for (int v = 0; v < VEC; ++v) acc[v] = acc[v] + x[v];
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) part[tid][v] = acc[v];
    }
    __syncthreads();
    if (valid && g == 0) {
        const int first = ul * tpu + c;
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            double s = part[first][v];
            for (int gg = 1; gg < ng; ++gg) s = s + part[first + gg * cpr][v];
            a.psum[((int64_t)h * a.head_dim + (int64_t)c * VEC + v) * a.max_pages + page] = s;
        }
    }
}

__device__ __forceinline__ double load_q(const void* q, int dtype, int64_t i) {
    if (dtype == 0) return (double)static_cast<const float*>(q)[i];
    const unsigned short u = static_cast<const unsigned short*>(q)[i];
    if (dtype == 1) return (double)__half2float(__ushort_as_half(u));
    return (double)__uint_as_float((uint32_t)u << 16);
}

// Order-preserving 64-bit key of a finite double (-0.0 folded into +0.0 so
// that equal scores get equal keys): larger score <=> larger key; every
// finite score has a key above 0, which pads the sort.
__device__ __forceinline__ unsigned long long score_key(double s) {
    const unsigned long long u = (unsigned long long)__double_as_longlong(s + 0.0);
    return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

struct BlockGeom {
    BlockPlan plan;
    int h_first, h_count, k_sel;
};

__device__ __forceinline__ BlockGeom block_geom(const SelectArgs& a, int blk, int head) {
    const int L = block_len(a.n_tok, a.q_subblock);
    const int b0 = a.u0 + blk * L;
    const int b1 = min(a.u0 + a.n_tok, b0 + L);
    const bool shared = a.gate.shared != 0;
    BlockGeom g;
    g.plan = plan_block(a.gate, b0, b1, a.k_budget[shared ? 0 : head]);
    g.h_first = shared ? 0 : head;
    g.h_count = shared ? a.n_head_kv : 1;
    g.k_sel = g.plan.gated ? min(g.plan.k_sel, a.sel_cap) : 0;
    return g;
}

// K2a: page scores.  CTA = (gating block, 32-page chunk) x KV head (or x all
// heads in shared mode); one thread per (page, 16-channel group): the group's
// fp64 fma chain in channel order with the query group held in registers, then
// lane g == 0 of the page adds the groups in order.  Shared mode keeps the max
// over heads.  Scores land in a [n_blocks][Hkv][max_pages] workspace.
__global__ void __launch_bounds__(kScoreThreads) k2a_score_pages(SelectArgs a) {
    const int d = a.head_dim;
    const int n_grp = d / kScoreGroupCh;
    const int ppc = kScoreThreads / n_grp;  // pages per CTA
    const int blk = blockIdx.x / a.score_chunks;
    const int chunk = blockIdx.x % a.score_chunks;
    const int head = a.head_begin + blockIdx.y;
    const BlockGeom bg = block_geom(a, blk, head);
    if (bg.k_sel == 0) return;
    const int n_cand = bg.plan.lsp - 1;
    if (chunk * ppc >= n_cand) return;
    const int tid = threadIdx.x;
    const int g = tid % n_grp;
    const int i = chunk * ppc + tid / n_grp;  // candidate index (page i + 1)
    const int G = a.n_head / a.n_head_kv;
    const int64_t qrow = (int64_t)(bg.plan.b1 - 1 - a.u0) * a.n_head * d;
    double best = -INFINITY;
    for (int hl = 0; hl < bg.h_count; ++hl) {
        const int hh = bg.h_first + hl;
        double qv[kScoreGroupCh], v[kScoreGroupCh];
#pragma unroll
        for (int j = 0; j < kScoreGroupCh; ++j)
            qv[j] = load_q(a.q, a.dtype, qrow + (int64_t)(hh * G) * d + g * kScoreGroupCh + j);
        const double* ps = a.psum + ((int64_t)hh * d + g * kScoreGroupCh) * a.max_pages + (i + 1);
#pragma unroll
        for (int j = 0; j < kScoreGroupCh; ++j) v[j] = i < n_cand ? __ldg(ps + (int64_t)j * a.max_pages) : 0.0;
        double acc = 0.0;
#pragma unroll
        for (int j = 0; j < kScoreGroupCh; ++j) acc = fma(qv[j], v[j], acc);
        double total = acc;
        for (int gg = 1; gg < n_grp; ++gg) total = total + __shfl_down_sync(0xffffffffu, acc, gg, n_grp);
        if (total > best) best = total;  // max over heads: best = -inf; if (v > best) best = v
    }
    if (g == 0 && i < n_cand) a.scores[((int64_t)blk * a.n_head_kv + bg.h_first) * a.max_pages + i] = best;
}

// K2b: top-k of one (gating block, KV head) -- or block in shared mode.
// Bitonic sort in shared memory on (score key desc, page asc), which is a total
// order, so the k first entries are exactly the (score desc, ties -> lower
// page) top-k; they are then emitted in ascending page order.  The reference's
// off-by-one (k_sel = lsp > lsp - 1 candidates) prepends page 0.
__global__ void __launch_bounds__(kSelectThreads) k2b_select_pages(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int blk = blockIdx.x;
    const int head = a.head_begin + blockIdx.y;
    const int Hkv = a.n_head_kv;
    const int tid = threadIdx.x;
    const BlockGeom bg = block_geom(a, blk, head);
    if (bg.plan.gated && bg.plan.k_sel > a.sel_cap && tid == 0) atomicCAS(a.err, 0, kDevBadSelection);
    if (tid < bg.h_count) a.cnt[(int64_t)blk * Hkv + bg.h_first + tid] = bg.k_sel;
    if (bg.k_sel == 0) return;
    const int n_cand = bg.plan.lsp - 1;
    const int take = min(bg.k_sel, n_cand);
    const int extra = bg.k_sel - take;
    int np = 1;
    while (np < n_cand) np <<= 1;
    unsigned long long* key = reinterpret_cast<unsigned long long*>(smem_raw);  // [np]
    int* pg = reinterpret_cast<int*>(key + np);                                // [np]
    unsigned char* flag = reinterpret_cast<unsigned char*>(pg + np);            // [n_cand]
    __shared__ int warp_tot[kSelectThreads / 32];
    const double* sc = a.scores + ((int64_t)blk * Hkv + bg.h_first) * a.max_pages;

    if (take >= n_cand) {
        for (int i = tid; i < n_cand; i += blockDim.x) flag[i] = 1;
    } else {
        for (int i = tid; i < np; i += blockDim.x) {
            key[i] = i < n_cand ? score_key(sc[i]) : 0ull;
            pg[i] = i;
        }
        for (int i = tid; i < n_cand; i += blockDim.x) flag[i] = 0;
        __syncthreads();
        for (int k = 2; k <= np; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int i = tid; i < np; i += blockDim.x) {
                    const int ixj = i ^ j;
                    if (ixj > i) {
                        const unsigned long long ka = key[i], kb = key[ixj];
                        const int pa = pg[i], pb = pg[ixj];
                        const bool a_first = ka > kb || (ka == kb && pa < pb);
                        const bool desc = (i & k) == 0;  // this pair's run is sorted "first-order"
                        if (desc != a_first) {
                            key[i] = kb;
                            key[ixj] = ka;
                            pg[i] = pb;
                            pg[ixj] = pa;
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int r = tid; r < take; r += blockDim.x) flag[pg[r]] = 1;
    }
    __syncthreads();

    // Emit flagged pages in ascending page order: per-thread contiguous chunk,
    // block-wide exclusive scan of the chunk counts.
    const int lane = tid & 31, wid = tid >> 5;
    const int chunk = (n_cand + blockDim.x - 1) / blockDim.x;
    const int lo = min(n_cand, tid * chunk);
    const int hi = min(n_cand, lo + chunk);
    int mine = 0;
    for (int i = lo; i < hi; ++i) mine += flag[i];
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < wid; ++w) base += warp_tot[w];
    base += incl - mine + extra;
    for (int hl = 0; hl < bg.h_count; ++hl) {
        int32_t* out = a.sel + ((int64_t)blk * Hkv + bg.h_first + hl) * a.sel_cap;
        int pos = base;
        for (int i = lo; i < hi; ++i)
            if (flag[i]) out[pos++] = i + 1;
        if (extra > 0 && tid == 0) out[0] = 0;
    }
}

}  // namespace

cudaError_t launch_pool_pages(const PoolArgs& a, cudaStream_t s) {
    if (a.page_end <= a.page_begin) return cudaSuccess;
    const int vec = a.dtype == 0 ? 4 : 8;
    const int tpu = (a.head_dim / vec) * (a.page_size / kPageSumGroupRows);
    if (tpu > kPoolThreads || a.head_dim % vec || a.page_size % kPageSumGroupRows) return cudaErrorInvalidValue;
    const int upc = kPoolThreads / tpu;
    const int64_t units = (int64_t)(a.page_end - a.page_begin) * (a.head_count > 0 ? a.head_count : a.n_head_kv);
    const unsigned grid = (unsigned)((units + upc - 1) / upc);
    switch (a.dtype) {
        case 0: k1_pool_pages<0><<<grid, kPoolThreads, 0, s>>>(a); break;
        case 1: k1_pool_pages<1><<<grid, kPoolThreads, 0, s>>>(a); break;
        default: k1_pool_pages<2><<<grid, kPoolThreads, 0, s>>>(a); break;
    }
    return cudaGetLastError();
}

size_t select_scores_elems(int n_blocks, int n_head_kv, int max_pages) {
    return (size_t)n_blocks * n_head_kv * max_pages;
}

cudaError_t launch_select_pages(const SelectArgs& a, cudaStream_t s) {
    const int nb = n_blocks_of(a.n_tok, a.q_subblock);
    if (a.gate.shared && (a.head_begin != 0 || (a.head_count > 0 && a.head_count != a.n_head_kv)))
        return cudaErrorInvalidValue;  // the shared selection spans every KV head
    const int hg = a.gate.shared ? 1 : (a.head_count > 0 ? a.head_count : a.n_head_kv);
    int np = 1;
    while (np < a.max_cand) np <<= 1;
    const size_t smem = (size_t)np * (sizeof(unsigned long long) + sizeof(int)) + (size_t)a.max_cand + 16;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        int dev = 0;
        cudaGetDevice(&dev);
        // one bit per device ordinal < 32; atomic for host threads on several devices
        static std::atomic<unsigned> attr_set_mask{0};
        if (dev >= 32 || !(attr_set_mask.load(std::memory_order_acquire) & (1u << dev))) {
            cudaError_t e = cudaFuncSetAttribute(k2b_select_pages, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024);
            if (e != cudaSuccess) return e;
            if (dev < 32) attr_set_mask.fetch_or(1u << dev, std::memory_order_release);
        }
    }
    if (a.max_cand > 0) {
        const int ppc = kScoreThreads / (a.head_dim / kScoreGroupCh);
        SelectArgs sa = a;
        sa.score_chunks = (a.max_cand + ppc - 1) / ppc;
        k2a_score_pages<<<dim3(nb * sa.score_chunks, hg), kScoreThreads, 0, s>>>(sa);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    k2b_select_pages<<<dim3(nb, hg), kSelectThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace epsp
