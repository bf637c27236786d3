// k_gate.cu -- K1 page sums and K2 page scoring + top-k page select.
//
// K1 replaces the reference's per-ubatch re-scan of the whole K view
// (ggml_mul_mat(k_p, q_heads) + ggml_sum_rows, patch :1045-1050) by an
// incremental pooling: each ubatch sums only the pages it completes, once, into
// a persistent fp64 buffer laid out [Hkv][max_pages][d] (a page's d sums are
// one contiguous row, written by consecutive threads and read by K2 as whole
// 128-byte groups).  HBM-bound: every K byte of the ubatch is read once.  For
// 16-bit caches K1 is a persistent kernel with one CTA per SM: a producer
// thread streams 128-row spans of one KV head into a ring of shared-memory
// stages with TMA (no multicast), and teams of consumer threads sum them in
// fp64 as the spans land, so several spans per SM are always in flight.
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
#include <algorithm>
#include <cmath>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "epsp_kernels.h"
#include "tc100.cuh"

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

// Direct variant (f32 caches and the fused append): one thread = (page, KV
// head, 16-byte channel chunk, 16-row group).  The group's rows are summed in
// ascending order, then thread g == 0 of the (page, head, chunk) adds the
// groups in ascending order.
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
        // the 16-row group lies inside one page, hence inside one block of a paged pool
        bool bad = false;
        const int64_t prow0 = phys_row(a.paging, (int32_t)row0, bad);
        if (bad && a.err) atomicCAS(a.err, 0, kDevBadBlockTable);
        const int64_t col = ((int64_t)h * a.head_dim + (int64_t)c * VEC) * ESZ;
        const int64_t row_bytes = (int64_t)a.n_head_kv * a.head_dim * ESZ;
        uint4 raw[kPageSumGroupRows];
        if (a.k_new == nullptr) {
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i)
                raw[i] = __ldg(reinterpret_cast<const uint4*>(base + (prow0 + i) * row_bytes + col));
        } else {
            // append: the new rows come from k_new and are written to the cache
            const char* nb = static_cast<const char*>(a.k_new);
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i) {
                const int64_t r = row0 + i;
                raw[i] = r >= a.new_begin ? __ldg(reinterpret_cast<const uint4*>(nb + (r - a.new_begin) * row_bytes + col))
                                          : *reinterpret_cast<const uint4*>(base + (prow0 + i) * row_bytes + col);
            }
            char* out = static_cast<char*>(a.k_store);
            if (!bad) {
#pragma unroll
                for (int i = 0; i < kPageSumGroupRows; ++i)
                    if (row0 + i >= a.new_begin) *reinterpret_cast<uint4*>(out + (prow0 + i) * row_bytes + col) = raw[i];
            }
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
            a.psum[((int64_t)h * a.max_pages + page) * a.head_dim + (int64_t)c * VEC + v] = s;
        }
    }
}

// ---- K1, TMA-staged variant (16-bit caches, plain pooling) ----------------
// Work item = (KV head, 128-row span of the pooled rows), head-major; CTA b
// takes items b, b + gridDim.x, ...  Stage = the span's [128 rows][d] of one
// head as two TMA boxes of [128 rows][64 channels] (128-byte rows, no
// swizzle).  A consumer team (one thread per (16-byte chunk, 16-row group) of
// a span) sums its 16 rows in ascending order from 0.0 in fp64, releases the
// stage, then its first d threads add the groups of each page in ascending
// order and store the page's d sums as one contiguous row: the page-sum
// contract of the direct variant and of the oracle.
constexpr int kSpanRows = 128;
constexpr int kPoolTmaProducer = 32;  // warp 0: lane 0 issues the copies

template <int D>
struct PoolTma {
    static constexpr int kChunks = D / 8;                       // 16-byte chunks per row
    static constexpr int kTeam = kChunks * (kSpanRows / kPageSumGroupRows);  // threads per span
    static constexpr int kTeams = 256 / kTeam;                  // spans summed at once
    static constexpr int kStages = D == 128 ? 6 : 8;            // a multiple of kTeams
    static constexpr int kStageBytes = kSpanRows * D * 2;
    static constexpr int kHalfBytes = kSpanRows * 128;          // one [128][64] box
    static constexpr int kPartBytes = kTeam * 8 * (int)sizeof(double);
    static constexpr int kOffPart = kStages * kStageBytes;
    static constexpr int kOffBar = kOffPart + kTeams * kPartBytes;
    static constexpr int kBytes = kOffBar + 2 * kStages * 8 + 16;
    static constexpr int kThreads = kPoolTmaProducer + kTeams * kTeam;
    static_assert(kStages % kTeams == 0, "each team reuses its own stages");
};

template <int DT, int D>
__global__ void __launch_bounds__(PoolTma<D>::kThreads, 1)
    k1_pool_pages_tma(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ PoolArgs a) {
    using LY = PoolTma<D>;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_dyn + 127) & ~(uintptr_t)127);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY::kOffBar);
    uint64_t* empty = full + LY::kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + LY::kStages);

    const int P = a.page_size;
    const int hc = a.head_count > 0 ? a.head_count : a.n_head_kv;
    const int64_t rows = (int64_t)(a.page_end - a.page_begin) * P;
    const int n_span = (int)((rows + kSpanRows - 1) / kSpanRows);
    const int64_t n_items = (int64_t)n_span * hc;
    // this CTA's items: blockIdx.x + k * gridDim.x, k < my_items
    const int my_items = n_items > blockIdx.x ? (int)((n_items - 1 - blockIdx.x) / gridDim.x) + 1 : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < LY::kStages; ++i) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], LY::kTeam);
        }
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch_desc(&tmK);
    }
    __syncthreads();

    if (threadIdx.x < kPoolTmaProducer) {
        if (threadIdx.x == 0) {
            int issued = 0;
            bool ok = true;
            for (int k = 0; k < my_items && ok; ++k) {
                const int st = k % LY::kStages;
                const uint32_t par = ((k / LY::kStages) & 1) ^ 1;
                if (!tc::mbar_wait(&empty[st], par, a.timeout_ns) || *abort_flag) {
                    ok = false;
                    break;
                }
                const int64_t item = blockIdx.x + (int64_t)k * gridDim.x;
                const int h = a.head_begin + (int)(item / n_span);
                const int row0 = a.page_begin * P + (int)(item % n_span) * kSpanRows;
                unsigned char* dst = smem + st * LY::kStageBytes;
                tc::mbar_arrive_expect_tx(&full[st], LY::kStageBytes);
                if (a.paging.block_rows <= 0) {
#pragma unroll
                    for (int hf = 0; hf < D / 64; ++hf)
                        tc::tma_load_3d(dst + hf * LY::kHalfBytes, &tmK, &full[st], hf * 64, h, row0);
                } else {
                    // paged pool: the map's box is one page; each page of the span
                    // comes from its own block (pages past the pooled range and
                    // bad table entries read rows past the pool: zeros)
                    for (int pr = 0; pr < kSpanRows; pr += P) {
                        bool bad = false;
                        int prow = a.paging.pool_rows;  // out of the map: zero fill
                        if (row0 + pr < a.page_end * P) {
                            prow = phys_row(a.paging, row0 + pr, bad);
                            if (bad) {
                                if (a.err) atomicCAS(a.err, 0, kDevBadBlockTable);
                                prow = a.paging.pool_rows;
                            }
                        }
#pragma unroll
                        for (int hf = 0; hf < D / 64; ++hf)
                            tc::tma_load_3d(dst + hf * LY::kHalfBytes + pr * 128, &tmK, &full[st], hf * 64, h, prow);
                    }
                }
                issued = k + 1;
            }
            if (!ok) {
                if (a.err) atomicCAS(a.err, 0, kDevWaitPoolProducer);
                *abort_flag = 1;
            }
            // copies still in flight must land before the CTA exits
            for (int k = issued - LY::kStages; k < issued; ++k)
                if (k >= 0) tc::mbar_wait(&full[k % LY::kStages], (k / LY::kStages) & 1, a.timeout_ns);
        }
    } else {
        const int ct = threadIdx.x - kPoolTmaProducer;
        const int team = ct / LY::kTeam;
        const int tt = ct % LY::kTeam;
        const int c = tt % LY::kChunks;   // 16-byte chunk of the row
        const int g = tt / LY::kChunks;   // 16-row group of the span
        double* part = reinterpret_cast<double*>(smem + LY::kOffPart + team * LY::kPartBytes);
        for (int k = team; k < my_items; k += LY::kTeams) {
            const int st = k % LY::kStages;
            const bool w = tc::mbar_wait(&full[st], (k / LY::kStages) & 1, a.timeout_ns);
            if (!w && a.err) atomicCAS(a.err, 0, kDevWaitPool);
            // one decision for the whole team (its threads' waits are bounded
            // separately), so no thread is left behind at the team's barriers
            if (!tc::named_bar_and(1 + team, LY::kTeam, w && !*abort_flag)) {
                *abort_flag = 1;
                break;
            }
            const unsigned char* src = smem + st * LY::kStageBytes + (c >> 3) * LY::kHalfBytes + (c & 7) * 16;
            double acc[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) acc[v] = 0.0;
#pragma unroll
            for (int i = 0; i < kPageSumGroupRows; ++i) {
                const uint4 u = *reinterpret_cast<const uint4*>(src + (g * kPageSumGroupRows + i) * 128);
                double x[8];
                Vec16<DT>::to_double(u, x);
#pragma unroll
                for (int v = 0; v < 8; ++v) acc[v] = acc[v] + x[v];
            }
            tc::mbar_arrive(&empty[st]);  // the stage may be refilled
#pragma unroll
            for (int v = 0; v < 8; ++v) part[g * D + c * 8 + v] = acc[v];
            tc::named_bar_sync(1 + team, LY::kTeam);
            const int64_t item = blockIdx.x + (int64_t)k * gridDim.x;
            const int h = a.head_begin + (int)(item / n_span);
            const int page0 = a.page_begin + (int)(item % n_span) * (kSpanRows / P);
            const int n_pg = min(kSpanRows / P, a.page_end - page0);
            const int gpp = P / kPageSumGroupRows;  // groups per page
            for (int idx = tt; idx < n_pg * D; idx += LY::kTeam) {
                const int pl = idx / D, ch = idx % D;
                double sum = part[(pl * gpp) * D + ch];
                for (int gg = 1; gg < gpp; ++gg) sum = sum + part[(pl * gpp + gg) * D + ch];
                a.psum[((int64_t)h * a.max_pages + page0 + pl) * D + ch] = sum;
            }
            tc::named_bar_sync(1 + team, LY::kTeam);  // part is rewritten by the next span
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

// Geometry of (block, head); routed = true applies the routing's effective
// budget (K2r's output) to k_sel and to the pooled count that follows it.
__device__ __forceinline__ BlockGeom block_geom(const SelectArgs& a, int blk, int head, bool routed = false) {
    const int L = block_len(a.n_tok, a.q_subblock);
    const int b0 = a.u0 + blk * L;
    const int b1 = min(a.u0 + a.n_tok, b0 + L);
    const bool shared = a.gate.shared != 0;
    BlockGeom g;
    g.plan = plan_block(a.gate, b0, b1, a.k_budget[shared ? 0 : head]);
    if (routed && a.route_mode != 0 && g.plan.gated && g.plan.lsp >= 2) {
        const int n_cand = g.plan.lsp - 1;
        g.plan.k_sel = a.route_k[(int64_t)blk * a.n_head_kv + head];
        const int left = n_cand - min(g.plan.k_sel, n_cand);
        g.plan.n_pool = min(a.gate.pool_pages, left);
    }
    g.h_first = shared ? 0 : head;
    g.h_count = shared ? a.n_head_kv : 1;
    g.k_sel = g.plan.gated ? min(g.plan.k_sel, a.sel_cap) : 0;
    return g;
}

// Pages this block ranks: the selection plus the pooled pages (when asked).
__device__ __forceinline__ int ranked_pages(const SelectArgs& a, const BlockGeom& bg) {
    return bg.k_sel + (a.pool != nullptr ? bg.plan.n_pool : 0);
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
    if (ranked_pages(a, bg) == 0) return;
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
        const double* ps = a.psum + ((int64_t)hh * a.max_pages + (i + 1)) * d + g * kScoreGroupCh;
#pragma unroll
        for (int j = 0; j < kScoreGroupCh; j += 2) {
            const double2 p2 = i < n_cand ? __ldg(reinterpret_cast<const double2*>(ps + j)) : make_double2(0.0, 0.0);
            v[j] = p2.x;
            v[j + 1] = p2.y;
        }
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
// off-by-one (k_sel = lsp > lsp - 1 candidates) prepends page 0.  With pooled
// rows armed, the n_pool entries ranked right after the selection are emitted
// (ascending) as the block's pooled pages.
__global__ void __launch_bounds__(kSelectThreads) k2b_select_pages(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int blk = blockIdx.x;
    const int head = a.head_begin + blockIdx.y;
    const int Hkv = a.n_head_kv;
    const int tid = threadIdx.x;
    const BlockGeom bg = block_geom(a, blk, head, true);
    const int n_pool = a.pool != nullptr ? bg.plan.n_pool : 0;
    if (bg.plan.gated && bg.plan.k_sel > a.sel_cap && tid == 0) atomicCAS(a.err, 0, kDevBadSelection);
    if (n_pool > a.pool_cap && tid == 0) atomicCAS(a.err, 0, kDevBadSelection);
    if (tid < bg.h_count) {
        a.cnt[(int64_t)blk * Hkv + bg.h_first + tid] = bg.k_sel;
        if (a.pool != nullptr) a.pool_cnt[(int64_t)blk * Hkv + bg.h_first + tid] = min(n_pool, a.pool_cap);
    }
    if (bg.k_sel == 0 && n_pool == 0) return;
    const int n_cand = bg.plan.lsp - 1;
    const int take = min(bg.k_sel, n_cand);
    const int extra = bg.k_sel - take;
    const int m = min(n_pool, a.pool_cap);
    int np = 1;
    while (np < n_cand) np <<= 1;
    unsigned long long* key = reinterpret_cast<unsigned long long*>(smem_raw);  // [np]
    int* pg = reinterpret_cast<int*>(key + np);                                // [np]
    unsigned char* flag = reinterpret_cast<unsigned char*>(pg + np);            // [n_cand]: 1 selected, 2 pooled
    __shared__ unsigned long long warp_tot[kSelectThreads / 32];
    const double* sc = a.scores + ((int64_t)blk * Hkv + bg.h_first) * a.max_pages;

    if (take >= n_cand) {
        for (int i = tid; i < n_cand; i += blockDim.x) flag[i] = 1;  // every candidate selected, none left to pool
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
        for (int r = tid; r < take + m; r += blockDim.x) flag[pg[r]] = r < take ? 1 : 2;
    }
    __syncthreads();

    // Emit flagged pages in ascending page order: per-thread contiguous chunk,
    // block-wide exclusive scan of the chunk counts (selected in the low 32
    // bits, pooled in the high 32).
    const int lane = tid & 31, wid = tid >> 5;
    const int chunk = (n_cand + blockDim.x - 1) / blockDim.x;
    const int lo = min(n_cand, tid * chunk);
    const int hi = min(n_cand, lo + chunk);
    unsigned long long mine = 0;
    for (int i = lo; i < hi; ++i) mine += flag[i] == 1 ? 1ull : (flag[i] == 2 ? (1ull << 32) : 0ull);
    unsigned long long incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    unsigned long long base = 0;
    for (int w = 0; w < wid; ++w) base += warp_tot[w];
    base += incl - mine;
    const int sbase = (int)(base & 0xffffffffull) + extra;
    const int pbase = (int)(base >> 32);
    for (int hl = 0; hl < bg.h_count; ++hl) {
        int32_t* out = a.sel + ((int64_t)blk * Hkv + bg.h_first + hl) * a.sel_cap;
        int32_t* pout = a.pool != nullptr ? a.pool + ((int64_t)blk * Hkv + bg.h_first + hl) * a.pool_cap : nullptr;
        int pos = sbase, ppos = pbase;
        for (int i = lo; i < hi; ++i) {
            if (flag[i] == 1) out[pos++] = i + 1;
            else if (flag[i] == 2) pout[ppos++] = i + 1;
        }
        if (extra > 0 && tid == 0) out[0] = 0;
    }
}

// K2r: per-KV-head routing of one gating block by the live page-score spread
// (AR006 head routing): warp w takes KV head w of the range; its lane 0 walks
// the block's candidate scores in ascending page order (max, and the fp64 sum
// from 0.0 for the mean, of u = score / page_size), spread = (max - mean) /
// (|mean| + eps); spread < threshold marks a streaming head (budget 0).  Mode
// 2 then gives the streaming heads' pages to the retrieval heads in equal
// shares (the remainder to the lowest-index ones), capped at the candidates.
// The result, the effective budgets, goes to route_k for K2b and K3.
__global__ void __launch_bounds__(1024) k2r_route_heads(SelectArgs a) {
    __shared__ int k_base[32], k_stream[32];
    const int blk = blockIdx.x;
    const int hc = a.head_count > 0 ? a.head_count : a.n_head_kv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int hl = warp; hl < hc; hl += blockDim.x >> 5) {
        const int h = a.head_begin + hl;
        const BlockGeom bg = block_geom(a, blk, h);
        const int n_cand = bg.plan.lsp - 1;
        int kin = bg.plan.gated ? bg.plan.k_sel : 0;
        int streaming = 0;
        if (lane == 0 && bg.plan.gated && n_cand >= 1) {
            const double* sc = a.scores + ((int64_t)blk * a.n_head_kv + h) * a.max_pages;
            const double inv_p = 1.0 / (double)a.gate.page_size;  // a power of two: exact
            double mx = -INFINITY, sum = 0.0;
            for (int i = 0; i < n_cand; ++i) {
                const double u = sc[i] * inv_p;
                mx = fmax(mx, u);
                sum = sum + u;
            }
            const double mean = sum / (double)n_cand;
            const double spread = (mx - mean) / (fabs(mean) + kRouteEps);
            streaming = spread < a.route_threshold ? 1 : 0;
        }
        if (lane == 0) {
            a.route_k[(int64_t)blk * a.n_head_kv + h] = streaming ? 0 : kin;
            if (hl < 32) {
                k_base[hl] = kin;
                k_stream[hl] = streaming;
            }
        }
    }
    if (a.route_mode != 2 || hc > 32) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        int freed = 0, n_ret = 0;
        for (int hl = 0; hl < hc; ++hl) {
            if (k_stream[hl]) freed += k_base[hl];
            else ++n_ret;
        }
        if (n_ret == 0 || freed == 0) return;
        const BlockGeom bg = block_geom(a, blk, a.head_begin);
        const int n_cand = bg.plan.lsp - 1;
        int rank = 0;
        for (int hl = 0; hl < hc; ++hl) {
            if (k_stream[hl]) continue;
            const int k = min(n_cand, k_base[hl] + freed / n_ret + (rank < freed % n_ret ? 1 : 0));
            a.route_k[(int64_t)blk * a.n_head_kv + a.head_begin + hl] = k;
            ++rank;
        }
    }
}

// K2c: pooled rows.  CTA = (gating block, KV head); the row's d channels are
// consecutive threads, so sums are read and rows written coalesced.
__global__ void __launch_bounds__(256) k2c_build_pooled(const __grid_constant__ PoolRowArgs a) {
    const int blk = blockIdx.x;
    const int h = a.head_begin + blockIdx.y;
    const int d = a.head_dim;
    const int cnt = min(__ldg(a.pool_cnt + (int64_t)blk * a.n_head_kv + h), a.pool_cap);
    const int32_t* list = a.pool + ((int64_t)blk * a.n_head_kv + h) * a.pool_cap;
    const double inv_p = 1.0 / (double)a.page_size;  // a power of two: exact
    for (int idx = threadIdx.x; idx < a.pool_stride * d; idx += blockDim.x) {
        const int j = idx / d, c = idx % d;
        float kf = 0.f, vf = 0.f;
        if (j < cnt) {
            const int page = __ldg(list + j);
            const int64_t off = ((int64_t)h * a.max_pages + page) * d + c;
            kf = (float)(__ldg(a.ksum + off) * inv_p);
            vf = (float)(__ldg(a.vsum + off) * inv_p);
        }
        const int64_t o = (((int64_t)blk * a.pool_stride + j) * a.n_head_kv + h) * d + c;
        if (a.out_dtype == 0) {
            static_cast<float*>(a.pk)[o] = kf;
            static_cast<float*>(a.pv)[o] = vf;
        } else if (a.out_dtype == 1) {
            static_cast<__half*>(a.pk)[o] = __float2half_rn(kf);
            static_cast<__half*>(a.pv)[o] = __float2half_rn(vf);
        } else {
            static_cast<__nv_bfloat16*>(a.pk)[o] = __float2bfloat16_rn(kf);
            static_cast<__nv_bfloat16*>(a.pv)[o] = __float2bfloat16_rn(vf);
        }
    }
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
    PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
    if (!f) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
            fn.store(f, std::memory_order_release);
        }
    }
    return f;
}

template <int DT, int D>
cudaError_t launch_pool_tma(const PoolArgs& a, cudaStream_t s) {
    using LY = PoolTma<D>;
    auto enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    // K as [rows][Hkv][d] 16-bit, box [128 rows][1 head][64 channels]; rows
    // past page_end * P are outside the map (zeros, never summed).  A paged
    // pool is mapped whole with a box of one page.
    CUtensorMap m;
    const bool paged = a.paging.block_rows > 0;
    const cuuint64_t rows_mapped = paged ? (cuuint64_t)a.paging.pool_rows : (cuuint64_t)a.page_end * a.page_size;
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)a.n_head_kv, rows_mapped};
    const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)D * a.n_head_kv * 2};
    const cuuint32_t box[3] = {64, 1, paged ? (cuuint32_t)std::min(a.page_size, kSpanRows) : (cuuint32_t)kSpanRows};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&m, DT == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(a.k), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    const int smem = LY::kBytes + 128;
    static std::atomic<unsigned> set_mask{0};  // one bit per device ordinal < 32
    if (dev >= 32 || !(set_mask.load(std::memory_order_acquire) & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(k1_pool_pages_tma<DT, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) set_mask.fetch_or(1u << dev, std::memory_order_release);
    }
    const int64_t rows = (int64_t)(a.page_end - a.page_begin) * a.page_size;
    const int64_t items = (rows + kSpanRows - 1) / kSpanRows * (a.head_count > 0 ? a.head_count : a.n_head_kv);
    const unsigned grid = (unsigned)std::min<int64_t>(items, sms);
    k1_pool_pages_tma<DT, D><<<grid, LY::kThreads, smem, s>>>(m, a);
    return cudaGetLastError();
}

cudaError_t launch_pool_pages(const PoolArgs& a, cudaStream_t s) {
    if (a.page_end <= a.page_begin) return cudaSuccess;
    // 16-bit caches without the append: the TMA-staged persistent kernel
    const bool aligned = (reinterpret_cast<uintptr_t>(a.k) & 15) == 0;
    if (a.k_new == nullptr && a.dtype != 0 && aligned && a.page_size % kPageSumGroupRows == 0 && a.timeout_ns > 0) {
        if (a.head_dim == 128) return a.dtype == 2 ? launch_pool_tma<2, 128>(a, s) : launch_pool_tma<1, 128>(a, s);
        if (a.head_dim == 64) return a.dtype == 2 ? launch_pool_tma<2, 64>(a, s) : launch_pool_tma<1, 64>(a, s);
    }
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
    constexpr size_t kSelectSmemMax = 227 * 1024 - 256;  // room for the kernel's static shared memory
    if (smem > kSelectSmemMax) return cudaErrorInvalidValue;
    if (smem > 48 * 1024 - 256) {
        int dev = 0;
        cudaGetDevice(&dev);
        // one bit per device ordinal < 32; atomic for host threads on several devices
        static std::atomic<unsigned> attr_set_mask{0};
        if (dev >= 32 || !(attr_set_mask.load(std::memory_order_acquire) & (1u << dev))) {
            cudaError_t e = cudaFuncSetAttribute(k2b_select_pages, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kSelectSmemMax);
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
    if (a.route_mode != 0) {
        if (a.gate.shared || a.route_k == nullptr) return cudaErrorInvalidValue;
        const int hc = a.head_count > 0 ? a.head_count : a.n_head_kv;
        if (a.route_mode == 2 && hc > 32) return cudaErrorNotSupported;
        k2r_route_heads<<<nb, std::min(1024, 32 * hc), 0, s>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    k2b_select_pages<<<dim3(nb, hg), kSelectThreads, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_build_pooled_rows(const PoolRowArgs& a, cudaStream_t s) {
    const int hc = a.head_count > 0 ? a.head_count : a.n_head_kv;
    if (a.n_blocks < 1 || hc < 1 || a.pool_stride < 1) return cudaErrorInvalidValue;
    k2c_build_pooled<<<dim3(a.n_blocks, hc), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace epsp
