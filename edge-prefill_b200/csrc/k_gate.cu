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

#include <cfloat>
#include <cmath>

#include "epsp_kernels.h"

namespace epsp {
namespace {

constexpr int kPoolThreads = 256;
constexpr int kSelectThreads = 256;

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
    const int64_t n_units = (int64_t)(a.page_end - a.page_begin) * a.n_head_kv;
    const int64_t unit = (int64_t)blockIdx.x * upc + ul;
    const bool valid = ul < upc && unit < n_units;
    int page = 0, h = 0;
    if (valid) {
        page = a.page_begin + (int)(unit / a.n_head_kv);
        h = (int)(unit % a.n_head_kv);
        constexpr int ESZ = DT == 0 ? 4 : 2;
        const char* base = static_cast<const char*>(a.k);
        const int64_t row0 = (int64_t)page * a.page_size + (int64_t)g * kPageSumGroupRows;
        uint4 raw[kPageSumGroupRows];
#pragma unroll
        for (int i = 0; i < kPageSumGroupRows; ++i) {
            const int64_t off = (((row0 + i) * a.n_head_kv + h) * a.head_dim + (int64_t)c * VEC) * ESZ;
            raw[i] = __ldg(reinterpret_cast<const uint4*>(base + off));
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
// that equal scores get equal keys): larger score <=> larger key.
__device__ __forceinline__ unsigned long long score_key(double s) {
    const unsigned long long u = (unsigned long long)__double_as_longlong(s + 0.0);
    return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

// One CTA per (gating block, KV head) -- or per block in shared mode.
//   1. scores: one thread per candidate page, fp64 fma chain over channels in
//      ascending order; channel values are loaded 16 at a time (independent
//      loads issued together) so the chain is not serialised on L2 latency;
//   2. selection: MSB-first radix select (8 passes of 8 bits) on the score
//      keys finds the k-th largest key T; keys > T are selected, and of the
//      keys == T the lowest pages fill the remaining slots -- exactly the
//      (score desc, page asc) order;
//   3. output: flagged pages in ascending page order (block-wide scan).
__global__ void __launch_bounds__(kSelectThreads) k2_select_pages(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int blk = blockIdx.x;
    const int head = blockIdx.y;  // per-head mode only
    const int Hkv = a.n_head_kv;
    const int d = a.head_dim;
    const int G = a.n_head / Hkv;
    const int L = block_len(a.n_tok, a.q_subblock);
    const int b0 = a.u0 + blk * L;
    const int b1 = min(a.u0 + a.n_tok, b0 + L);
    const bool shared = a.gate.shared != 0;
    const int kb = a.k_budget[shared ? 0 : head];
    const BlockPlan plan = plan_block(a.gate, b0, b1, kb);
    const int h_first = shared ? 0 : head;
    const int h_count = shared ? Hkv : 1;
    const int tid = threadIdx.x;

    int k_sel = plan.gated ? plan.k_sel : 0;
    if (k_sel > a.sel_cap) {  // the host checks this; never write past the list
        if (tid == 0) atomicCAS(a.err, 0, kDevBadSelection);
        k_sel = a.sel_cap;
    }
    if (tid < h_count) a.cnt[(int64_t)blk * Hkv + h_first + tid] = k_sel;
    if (k_sel == 0) return;

    const int n_cand = plan.lsp - 1;  // pages 1 .. lsp-1
    double* qd = reinterpret_cast<double*>(smem_raw);             // [h_count][d]
    double* sc = qd + (size_t)h_count * d;                         // [n_cand]
    unsigned char* flag = reinterpret_cast<unsigned char*>(sc + (n_cand > 0 ? n_cand : 1));
    __shared__ int warp_tot[kSelectThreads / 32];
    __shared__ int hist[256];
    __shared__ int pick_bin, pick_above;

    const int64_t qrow = (int64_t)(b1 - 1 - a.u0) * a.n_head * d;
    for (int i = tid; i < h_count * d; i += blockDim.x) {
        const int hh = h_first + i / d;
        qd[i] = load_q(a.q, a.dtype, qrow + (int64_t)(hh * G) * d + (i % d));
    }
    __syncthreads();

    constexpr int CH = 16;
    for (int i = tid; i < n_cand; i += blockDim.x) {
        const int page = i + 1;
        double best = -INFINITY;
        for (int hl = 0; hl < h_count; ++hl) {
            const double* ps = a.psum + (int64_t)(h_first + hl) * d * a.max_pages + page;
            const double* qv = qd + hl * d;
            double acc = 0.0;
            for (int c0 = 0; c0 < d; c0 += CH) {
                double v[CH];
#pragma unroll
                for (int j = 0; j < CH; ++j) v[j] = __ldg(ps + (int64_t)(c0 + j) * a.max_pages);
#pragma unroll
                for (int j = 0; j < CH; ++j) acc = fma(qv[c0 + j], v[j], acc);
            }
            if (acc > best) best = acc;
        }
        sc[i] = best;
    }
    __syncthreads();

    const int take = min(k_sel, n_cand);
    const int extra = k_sel - take;  // reference off-by-one: page 0 (lowest -inf id) fills
    const int lane = tid & 31, wid = tid >> 5;
    if (take >= n_cand) {
        for (int i = tid; i < n_cand; i += blockDim.x) flag[i] = 1;
    } else {
        unsigned long long prefix = 0, pmask = 0;
        int k_rem = take;
        for (int pass = 7; pass >= 0; --pass) {
            const int shift = pass * 8;
            for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
            __syncthreads();
            for (int i = tid; i < n_cand; i += blockDim.x) {
                const unsigned long long key = score_key(sc[i]);
                if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
            }
            __syncthreads();
            if (wid == 0) {
                int loc[8], sum = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    loc[j] = hist[255 - 8 * lane - j];
                    sum += loc[j];
                }
                int incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const int excl = incl - sum;
                if (excl < k_rem && k_rem <= incl) {
                    int acc = excl;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (acc + loc[j] >= k_rem) {
                            pick_bin = 255 - 8 * lane - j;
                            pick_above = acc;
                            break;
                        }
                        acc += loc[j];
                    }
                }
            }
            __syncthreads();
            k_rem -= pick_above;
            prefix |= (unsigned long long)pick_bin << shift;
            pmask |= 0xFFull << shift;
        }
        // prefix == key of the take-th largest score; k_rem of its ties are taken.
        const int chunk = (n_cand + blockDim.x - 1) / blockDim.x;
        const int lo = min(n_cand, tid * chunk);
        const int hi = min(n_cand, lo + chunk);
        int eq = 0;
        for (int i = lo; i < hi; ++i) eq += score_key(sc[i]) == prefix;
        int incl = eq;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) warp_tot[wid] = incl;
        __syncthreads();
        int before = incl - eq;
        for (int w = 0; w < wid; ++w) before += warp_tot[w];
        for (int i = lo; i < hi; ++i) {
            const unsigned long long key = score_key(sc[i]);
            unsigned char f = key > prefix;
            if (key == prefix) f = (before++ < k_rem);
            flag[i] = f;
        }
        __syncthreads();
    }
    __syncthreads();

    // Emit flagged pages in ascending page order: per-thread contiguous chunk,
    // block-wide exclusive scan of the chunk counts.
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
    for (int hl = 0; hl < h_count; ++hl) {
        int32_t* out = a.sel + ((int64_t)blk * Hkv + h_first + hl) * a.sel_cap;
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
    const int64_t units = (int64_t)(a.page_end - a.page_begin) * a.n_head_kv;
    const unsigned grid = (unsigned)((units + upc - 1) / upc);
    switch (a.dtype) {
        case 0: k1_pool_pages<0><<<grid, kPoolThreads, 0, s>>>(a); break;
        case 1: k1_pool_pages<1><<<grid, kPoolThreads, 0, s>>>(a); break;
        default: k1_pool_pages<2><<<grid, kPoolThreads, 0, s>>>(a); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_select_pages(const SelectArgs& a, cudaStream_t s) {
    const int nb = n_blocks_of(a.n_tok, a.q_subblock);
    const int h_count = a.gate.shared ? a.n_head_kv : 1;
    const size_t smem = (size_t)h_count * a.head_dim * sizeof(double) + (size_t)a.max_pages * sizeof(double) +
                        (size_t)a.max_pages + 16;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        int dev = 0;
        cudaGetDevice(&dev);
        static unsigned attr_set_mask = 0;  // one bit per device ordinal < 32
        if (dev >= 32 || !(attr_set_mask & (1u << dev))) {
            cudaError_t e = cudaFuncSetAttribute(k2_select_pages, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024);
            if (e != cudaSuccess) return e;
            if (dev < 32) attr_set_mask |= 1u << dev;
        }
    }
    dim3 grid(nb, a.gate.shared ? 1 : a.n_head_kv);
    k2_select_pages<<<grid, kSelectThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace epsp
