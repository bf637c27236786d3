// k_attn_f32.cu -- K3 for f32 Q/K/V: the same page-gated sparse attention in
// fp32 on the CUDA cores.
//
// The reference attends an f32 KV cache in f32 (build_attn_mha after the
// gathers cast back to the source type, patch :1081-1093); the tensor-core
// kernel (k_attn.cu) takes 16-bit operands only.  Rather than narrowing f32
// inputs, this kernel keeps every operand, product, score, exponential and
// accumulator in fp32.  It walks the same kept set as K3 -- sink page, the
// selected pages, the local window cut causally at each query's own row --
// straight from the KV cache, and covers the same CTA grid: K3 CTA id `id`
// (head-major [Hkv][blocks][ctas_per_block], NT query tiles of 128 / G tokens)
// is split into subs_per_cta(NT) sub-CTAs of 64 query rows, so every entry point that
// takes K3 CTA ranges works unchanged.
//
// Sub-CTA: 128 threads, two per query row (each holds half of the row's q and
// O in registers); K/V rows arrive in 32-row chunks staged in shared memory
// with 16-byte loads.  Per chunk each thread pair scores the 32 keys (fp32 FMA
// chain over its channels, pair combined by one shuffle), then an online
// softmax in base 2 (running max, rescale of O and l when it grows) adds
// p * v in fp32.  The tensor cores are not used: this path trades speed for
// f32 arithmetic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>

#include "epsp_kernels.h"

namespace epsp {
namespace {

constexpr int kRowsPerSub = 64;   // query rows of one sub-CTA
constexpr int kSubThreads = 128;  // two threads per row
constexpr int kChunk = 32;        // KV rows staged per step (divides every page size)

__host__ __device__ constexpr int subs_per_cta(int nt) { return nt * 128 / kRowsPerSub; }

template <int D, int NT>
__global__ void __launch_bounds__(kSubThreads, D == 128 ? 2 : 3) k3f_sparse_attention(const __grid_constant__ AttnArgs a) {
    constexpr int HALF = D / 2;
    constexpr int SUBS = subs_per_cta(NT);
    __shared__ __align__(16) float ks[kChunk][D];
    __shared__ __align__(16) float vs[kChunk][D];

    const int Hkv = a.n_head_kv;
    const int G = a.n_head / Hkv;
    const int T = 128 / G;
    const int L = block_len(a.n_tok, a.q_subblock);
    const int tpb = (L + NT * T - 1) / (NT * T);
    // the K3 CTA this sub-CTA belongs to (same id order as k_attn.cu)
    const int n_cta = (int)(gridDim.x / SUBS);
    const int cta = (int)(blockIdx.x / SUBS), sub = (int)(blockIdx.x % SUBS);
    const int id = a.cta_begin + (n_cta - 1 - cta);
    const int h = id / (a.blk_count * tpb);
    const int blk = a.blk_begin + (id % (a.blk_count * tpb)) / tpb;
    const int b0 = a.u0 + blk * L;
    const int b1 = min(a.u0 + a.n_tok, b0 + L);
    const int t0 = b0 + (id % tpb) * NT * T;
    if (t0 >= b1) return;
    const int t_end = min(t0 + NT * T, b1);
    const int rows_cta = (t_end - t0) * G;  // token-major rows: row = token * G + g
    const int r_first = sub * kRowsPerSub;
    if (r_first >= rows_cta) return;

    const BlockPlan plan = plan_block(a.gate, b0, b1, __ldg(a.k_budget + h));
    const int P = a.gate.page_size;
    const int64_t bh = (int64_t)blk * Hkv + h;  // K2's counts replace the plan's when given (head routing)
    const int k_sel = plan.gated ? (a.cnt != nullptr ? min(__ldg(a.cnt + bh), a.sel_cap) : plan.k_sel) : 0;
    const int L0 = plan.gated ? plan.lsp * P : 0;
    const int32_t* sel = a.sel + ((int64_t)blk * Hkv + h) * a.sel_cap;
    // kept chunks: sink page, selected pages, pooled rows, local window [L0, t_end)
    const int cpp = P / kChunk;
    const int n_fixed = plan.gated ? cpp * (1 + k_sel) : 0;
    const int n_pool = (plan.gated && a.pk != nullptr)
                           ? (a.pool_cnt != nullptr ? min(__ldg(a.pool_cnt + bh), a.pool_stride) : plan.n_pool)
                           : 0;
    const int n_pch = (n_pool + kChunk - 1) / kChunk;
    const int n_chunks = n_fixed + n_pch + (t_end - L0 + kChunk - 1) / kChunk;

    const int tid = threadIdx.x;
    const int row = r_first + (tid >> 1);
    const int half = tid & 1;
    const bool active = row < rows_cta;
    const int t = active ? t0 + row / G : -1;
    const int hq = h * G + (active ? row % G : 0);

    const float qs = a.kq_scale * 1.4426950408889634f;  // scores in log2 units
    float q[HALF], o[HALF];
    {
        const float* qp = static_cast<const float*>(a.q) + ((int64_t)(active ? t - a.u0 : 0) * a.n_head + hq) * D +
                          half * HALF;
#pragma unroll
        for (int c = 0; c < HALF; c += 4) {
            const float4 v4 = active ? __ldg(reinterpret_cast<const float4*>(qp + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
            q[c] = v4.x * qs;
            q[c + 1] = v4.y * qs;
            q[c + 2] = v4.z * qs;
            q[c + 3] = v4.w * qs;
        }
#pragma unroll
        for (int c = 0; c < HALF; ++c) o[c] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    bool bad = false;
    const int64_t row_stride = (int64_t)Hkv * D;
    const float* kbase = static_cast<const float*>(a.k) + (int64_t)h * D;
    const float* vbase = static_cast<const float*>(a.v) + (int64_t)h * D;

    for (int ci = 0; ci < n_chunks; ++ci) {
        int r;           // first KV row of the chunk (in the cache, or in the pooled rows)
        int pvalid = 0;  // > 0: a chunk of pooled rows with that many valid rows
        if (ci >= n_fixed && ci < n_fixed + n_pch) {
            const int pc = ci - n_fixed;
            r = blk * a.pool_stride + pc * kChunk;
            pvalid = min(kChunk, n_pool - pc * kChunk);
        } else if (ci < n_fixed) {
            const int pi = ci / cpp;  // 0: sink page, then the selected pages
            int page = 0;
            if (pi > 0) {
                page = __ldg(sel + pi - 1);
                if (page < 0 || (page + 1) * P > a.kv_len) {
                    bad = true;
                    page = -1;
                }
            }
            r = page < 0 ? -1 : page * P + (ci % cpp) * kChunk;
        } else {
            r = L0 + (ci - n_fixed - n_pch) * kChunk;
        }
        __syncthreads();  // the previous chunk is consumed
        if (r >= 0) {
            const float* kb = pvalid > 0 ? static_cast<const float*>(a.pk) + (int64_t)h * D : kbase;
            const float* vb = pvalid > 0 ? static_cast<const float*>(a.pv) + (int64_t)h * D : vbase;
            int n_rows = pvalid > 0 ? pvalid : a.kv_len - r;
            // a cache chunk lies in one page, hence in one block of a paged pool
            int src = r;
            if (pvalid == 0 && a.paging.block_rows > 0) {
                bool badt = false;
                src = phys_row(a.paging, r, badt);
                if (badt) {
                    bad = true;
                    n_rows = 0;
                }
            }
            for (int i = tid; i < kChunk * D / 4; i += kSubThreads) {
                const int rr = i / (D / 4), c4 = i % (D / 4);
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
                if (rr < n_rows) {
                    kv = __ldg(reinterpret_cast<const float4*>(kb + (int64_t)(src + rr) * row_stride) + c4);
                    vv = __ldg(reinterpret_cast<const float4*>(vb + (int64_t)(src + rr) * row_stride) + c4);
                }
                reinterpret_cast<float4*>(&ks[rr][0])[c4] = kv;
                reinterpret_cast<float4*>(&vs[rr][0])[c4] = vv;
            }
        }
        __syncthreads();
        // last visible key of this chunk for this row (causal; pooled rows are
        // visible to every row; absent chunk: none)
        const int lim = (r < 0 || !active) ? -1 : (pvalid > 0 ? pvalid - 1 : min(kChunk - 1, t - r));
        const int lim_w = __reduce_max_sync(0xffffffffu, lim);
        for (int j0 = 0; j0 <= lim_w; j0 += 8) {
            float s[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float* kr = &ks[j0 + u][half * HALF];
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < HALF; c += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                    acc = fmaf(q[c], k4.x, acc);
                    acc = fmaf(q[c + 1], k4.y, acc);
                    acc = fmaf(q[c + 2], k4.z, acc);
                    acc = fmaf(q[c + 3], k4.w, acc);
                }
                acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                s[u] = (j0 + u <= lim) ? acc : -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int u = 1; u < 8; ++u) mx = fmaxf(mx, s[u]);
            const float m_new = fmaxf(m, mx);
            if (m_new == -INFINITY) continue;  // nothing visible yet for this row
            const float alpha = exp2f(m - m_new);  // 0 on the first visible keys
            m = m_new;
            l *= alpha;
#pragma unroll
            for (int c = 0; c < HALF; ++c) o[c] *= alpha;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float p = exp2f(s[u] - m);
                l += p;
                const float* vr = &vs[j0 + u][half * HALF];
#pragma unroll
                for (int c = 0; c < HALF; c += 4) {
                    const float4 v4 = *reinterpret_cast<const float4*>(vr + c);
                    o[c] = fmaf(p, v4.x, o[c]);
                    o[c + 1] = fmaf(p, v4.y, o[c + 1]);
                    o[c + 2] = fmaf(p, v4.z, o[c + 2]);
                    o[c + 3] = fmaf(p, v4.w, o[c + 3]);
                }
            }
        }
    }
    if (bad && tid == 0) atomicCAS(a.err, 0, kDevBadSelection);
    if (!active) return;
    const float inv_l = 1.f / l;
    const int out_heads = a.out_heads > 0 ? a.out_heads : a.n_head;
    const int64_t off = ((int64_t)(t - a.u0) * out_heads + a.out_head0 + hq) * D + half * HALF;
    if (a.out_dtype == 0) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
        for (int c = 0; c < HALF; c += 4)
            dst[c / 4] = make_float4(o[c] * inv_l, o[c + 1] * inv_l, o[c + 2] * inv_l, o[c + 3] * inv_l);
    } else if (a.out_dtype == 1) {
        __half2* dst = reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + off);
#pragma unroll
        for (int c = 0; c < HALF; c += 2) dst[c / 2] = __floats2half2_rn(o[c] * inv_l, o[c + 1] * inv_l);
    } else {
        __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + off);
#pragma unroll
        for (int c = 0; c < HALF; c += 2) dst[c / 2] = __floats2bfloat162_rn(o[c] * inv_l, o[c + 1] * inv_l);
    }
}

template <int D, int NT>
cudaError_t launch_f32_t(const AttnArgs& a, cudaStream_t s) {
    const int G = a.n_head / a.n_head_kv;
    const int T = 128 / G;
    const int L = block_len(a.n_tok, a.q_subblock);
    const int tpb = (L + NT * T - 1) / (NT * T);
    const int64_t total = (int64_t)a.n_head_kv * a.blk_count * tpb;
    const int64_t count = a.cta_count > 0 ? a.cta_count : total - a.cta_begin;
    if (a.cta_begin < 0 || count < 1 || a.cta_begin + count > total) return cudaErrorInvalidValue;
    const int64_t grid = count * subs_per_cta(NT);
    if (grid > 0x7fffffff) return cudaErrorInvalidValue;
    k3f_sparse_attention<D, NT><<<(unsigned)grid, kSubThreads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_sparse_attention_f32(const AttnArgs& a, cudaStream_t s) {
    if (a.dtype != 0) return cudaErrorInvalidValue;
    if (a.n_head % a.n_head_kv || 128 / (a.n_head / a.n_head_kv) < 1) return cudaErrorNotSupported;
    if (a.n_dest > 0) return cudaErrorNotSupported;  // the exchange stores 16-bit tiles from K3 only
    if (a.tiles_per_cta != 1 && a.tiles_per_cta != 2) return cudaErrorInvalidValue;
    if (a.gate.page_size % kChunk) return cudaErrorNotSupported;
    const bool two = a.tiles_per_cta == 2;
    if (a.head_dim == 128) return two ? launch_f32_t<128, 2>(a, s) : launch_f32_t<128, 1>(a, s);
    if (a.head_dim == 64) return two ? launch_f32_t<64, 2>(a, s) : launch_f32_t<64, 1>(a, s);
    return cudaErrorNotSupported;
}

}  // namespace epsp
