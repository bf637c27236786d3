// k_ffn.cu -- K4: FFN-skip row compaction and scatter.
//
// The reference skips a layer's FFN for every row by returning
// ggml_scale(cur, 0) in build_ffn (patches/llama-prefill-ffn-skip.patch
// :146-149: the residual add survives, the FFN contributes zero), and drops
// non-selected tokens from the batch host-side (src/sparse_prefill.cpp
// :214-232).  Generalised to rows: only the kept rows are gathered into a
// dense [n_keep][hidden] block for the FFN GEMMs, and the FFN output is added
// back into their residual rows; every other row keeps its residual unchanged,
// exactly the zero-contribution semantics.  Pure data movement: HBM-bound.
// The scan reads the mask as 16-byte vectors in one CTA; the gather and the
// scatter-add give each kept row to one warp, whose lanes keep 8 16-byte loads
// in flight (no per-element index division).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "epsp_kernels.h"

namespace epsp {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kRowWarps = 8;  // rows copied at once per CTA (one warp per row)
constexpr int kRowUnroll = 8; // 16-byte loads in flight per lane

// Nonzero bytes of a 32-bit word.
__device__ __forceinline__ int nonzero_bytes(uint32_t w) {
    return __popc((((w & 0x7f7f7f7fu) + 0x7f7f7f7fu) | w) & 0x80808080u);
}

// Single CTA: ordered stream compaction of the keep mask -> row ids, count.
// Each thread owns a contiguous run of rows (a multiple of 16 bytes of the
// mask, read as 16-byte vectors when the mask is 16-byte aligned), counts its
// kept rows, a block-wide exclusive scan gives its first output slot, and it
// writes its kept row ids in row order.
__global__ void __launch_bounds__(kScanThreads) k4_scan_keep(const uint8_t* keep, int32_t n_rows, int32_t skip,
                                                             int32_t* row_ids, int32_t* n_keep) {
    __shared__ int warp_tot[kScanThreads / 32];
    if (skip) {
        if (threadIdx.x == 0) *n_keep = 0;
        return;
    }
    const int chunk = ((n_rows + kScanThreads - 1) / kScanThreads + 15) & ~15;
    const int lo = min(n_rows, (int)threadIdx.x * chunk);
    const int hi = min(n_rows, lo + chunk);
    const bool vec = (reinterpret_cast<uintptr_t>(keep) & 15) == 0;
    int mine = 0;
    int r = lo;
    if (vec)
        for (; r + 16 <= hi; r += 16) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(keep + r));
            mine += nonzero_bytes(u.x) + nonzero_bytes(u.y) + nonzero_bytes(u.z) + nonzero_bytes(u.w);
        }
    for (; r < hi; ++r) mine += keep[r] != 0;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        int v = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        warp_tot[lane] = v;  // inclusive totals
    }
    __syncthreads();
    int pos = (wid ? warp_tot[wid - 1] : 0) + incl - mine;
    if (mine > 0) {
        r = lo;
        if (vec)
            for (; r + 16 <= hi; r += 16) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(keep + r));
                if ((u.x | u.y | u.z | u.w) == 0) continue;
                const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if ((w4[i >> 2] >> (8 * (i & 3))) & 0xffu) row_ids[pos++] = r + i;
            }
        for (; r < hi; ++r)
            if (keep[r]) row_ids[pos++] = r;
    }
    if (threadIdx.x == kScanThreads - 1) *n_keep = warp_tot[kScanThreads / 32 - 1];
}

// Gather kept rows: x_kept[i] = x[row_ids[i]], one warp per row (grid-stride
// over rows), kRowUnroll 16-byte loads in flight per lane before the stores.
__global__ void __launch_bounds__(kRowWarps * 32) k4_gather_rows(const uint4* __restrict__ x, uint4* __restrict__ x_kept,
                                                                 const int32_t* __restrict__ row_ids,
                                                                 const int32_t* __restrict__ n_keep, int32_t cpr) {
    const int n = *n_keep;
    const int lane = threadIdx.x & 31;
    for (int i = blockIdx.x * kRowWarps + (threadIdx.x >> 5); i < n; i += gridDim.x * kRowWarps) {
        const uint4* src = x + (int64_t)__ldg(row_ids + i) * cpr;
        uint4* dst = x_kept + (int64_t)i * cpr;
        for (int c0 = 0; c0 < cpr; c0 += 32 * kRowUnroll) {
            uint4 v[kRowUnroll];
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < cpr) v[u] = __ldg(src + c);
            }
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < cpr) dst[c] = v[u];
            }
        }
    }
}

template <int DT>
__device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
    if constexpr (DT == 2) {
        const float lo = __uint_as_float(a << 16) + __uint_as_float(b << 16);
        const float hi = __uint_as_float(a & 0xffff0000u) + __uint_as_float(b & 0xffff0000u);
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        const float lo = __half2float(__ushort_as_half((unsigned short)(a & 0xffffu))) +
                         __half2float(__ushort_as_half((unsigned short)(b & 0xffffu)));
        const float hi = __half2float(__ushort_as_half((unsigned short)(a >> 16))) +
                         __half2float(__ushort_as_half((unsigned short)(b >> 16)));
        return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
    }
}

template <int DT>
__device__ __forceinline__ uint4 add16(uint4 x, const uint4& f) {
    if constexpr (DT == 0) {
        x.x = __float_as_uint(__uint_as_float(x.x) + __uint_as_float(f.x));
        x.y = __float_as_uint(__uint_as_float(x.y) + __uint_as_float(f.y));
        x.z = __float_as_uint(__uint_as_float(x.z) + __uint_as_float(f.z));
        x.w = __float_as_uint(__uint_as_float(x.w) + __uint_as_float(f.w));
    } else {
        x.x = add2<DT>(x.x, f.x);
        x.y = add2<DT>(x.y, f.y);
        x.z = add2<DT>(x.z, f.z);
        x.w = add2<DT>(x.w, f.w);
    }
    return x;
}

// residual[row_ids[i]] += ffn_out[i] (fp32 add, rounded to the element type):
// one warp per kept row, kRowUnroll chunks of both operands in flight per lane.
template <int DT>
__global__ void __launch_bounds__(kRowWarps * 32) k4_scatter_add(const uint4* __restrict__ ffn_out,
                                                                 uint4* __restrict__ residual,
                                                                 const int32_t* __restrict__ row_ids,
                                                                 const int32_t* __restrict__ n_keep, int32_t cpr) {
    const int n = *n_keep;
    const int lane = threadIdx.x & 31;
    for (int i = blockIdx.x * kRowWarps + (threadIdx.x >> 5); i < n; i += gridDim.x * kRowWarps) {
        const uint4* src = ffn_out + (int64_t)i * cpr;
        uint4* dst = residual + (int64_t)__ldg(row_ids + i) * cpr;
        for (int c0 = 0; c0 < cpr; c0 += 32 * kRowUnroll) {
            uint4 f[kRowUnroll], x[kRowUnroll];
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < cpr) {
                    f[u] = __ldg(src + c);
                    x[u] = dst[c];
                }
            }
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < cpr) dst[c] = add16<DT>(x[u], f[u]);
            }
        }
    }
}

// Plain row copy (16-byte vectors, grid-stride): the KV append's V rows and
// the K rows outside completed pages, on the SMs rather than a copy engine.
__global__ void k_copy16(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __ldg(src + i);
}

// A finite input whose f16 rounding overflows to +-inf records kDevF16Range
// (the tensor-core mode cannot represent it; the f32 mode can).
__global__ void k_f32_to_f16(const float* __restrict__ src, __half* __restrict__ dst, int64_t n, int32_t* err) {
    bool over = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float x = src[i];
        const __half hx = __float2half_rn(x);
        over |= __hisinf(hx) != 0 && isfinite(x);
        dst[i] = hx;
    }
    if (__any_sync(0xffffffffu, over) && (threadIdx.x & 31) == 0) atomicCAS(err, 0, kDevF16Range);
}

unsigned stream_grid(cudaStream_t) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return (unsigned)sms * 8;  // 8 x 256 threads resident per SM
}

// Row copy into a paged pool: logical rows [row_begin, row_begin + n_rows)
// of the destination go to their table rows; a bad table entry records the
// error and skips the row.
__global__ void k_copy_rows_paged(const uint4* __restrict__ src, uint4* __restrict__ dst, int32_t row_begin,
                                  int32_t n_rows, int32_t cpr, KvPaging pg, int32_t* err) {
    const int64_t total = (int64_t)n_rows * cpr;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t r = (int32_t)(i / cpr), c = (int32_t)(i % cpr);
        bool bad = false;
        const int32_t pr = phys_row(pg, row_begin + r, bad);
        if (bad) {
            if (err) atomicCAS(err, 0, kDevBadBlockTable);
            continue;
        }
        dst[(int64_t)pr * cpr + c] = __ldg(src + i);
    }
}

}  // namespace

cudaError_t launch_copy_rows_paged(const void* src, void* dst_pool, int32_t row_begin, int32_t n_rows, size_t row_bytes,
                                   const KvPaging& pg, int32_t* err, cudaStream_t s) {
    if (n_rows <= 0) return cudaSuccess;
    if (row_bytes % 16 || (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst_pool)) & 15)
        return cudaErrorInvalidValue;
    const int32_t cpr = (int32_t)(row_bytes / 16);
    const int64_t total = (int64_t)n_rows * cpr;
    const unsigned grid = (unsigned)std::min<int64_t>(stream_grid(s), (total + 255) / 256);
    k_copy_rows_paged<<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst_pool), row_begin,
                                           n_rows, cpr, pg, err);
    return cudaGetLastError();
}

cudaError_t launch_ffn_compact(const FfnCompactArgs& a, cudaStream_t s) {
    if ((a.hidden * a.elem_bytes) % 16) return cudaErrorInvalidValue;
    k4_scan_keep<<<1, kScanThreads, 0, s>>>(a.keep, a.n_rows, a.skip_layer, a.row_ids, a.n_keep);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.skip_layer) return e;
    const int cpr = a.hidden * a.elem_bytes / 16;
    const unsigned grid = std::max(1u, std::min<unsigned>(stream_grid(s) / 2, (unsigned)((a.n_rows + kRowWarps - 1) / kRowWarps)));
    k4_gather_rows<<<grid, kRowWarps * 32, 0, s>>>(static_cast<const uint4*>(a.x), static_cast<uint4*>(a.x_kept),
                                                  a.row_ids, a.n_keep, cpr);
    return cudaGetLastError();
}

cudaError_t launch_ffn_scatter(const FfnScatterArgs& a, cudaStream_t s) {
    const int esz = a.dtype == 0 ? 4 : 2;
    if ((a.hidden * esz) % 16) return cudaErrorInvalidValue;
    const int cpr = a.hidden * esz / 16;
    const uint4* f = static_cast<const uint4*>(a.ffn_out);
    uint4* r = static_cast<uint4*>(a.residual);
    const unsigned grid = std::max(1u, std::min<unsigned>(stream_grid(s) / 2, (unsigned)((a.n_rows + kRowWarps - 1) / kRowWarps)));
    switch (a.dtype) {
        case 0: k4_scatter_add<0><<<grid, kRowWarps * 32, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
        case 1: k4_scatter_add<1><<<grid, kRowWarps * 32, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
        default: k4_scatter_add<2><<<grid, kRowWarps * 32, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_copy_rows(const void* src, void* dst, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return cudaSuccess;
    if (bytes % 16 || (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15)
        return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s);
    const int64_t n16 = (int64_t)(bytes / 16);
    const unsigned grid = (unsigned)std::min<int64_t>(stream_grid(s), (n16 + 255) / 256);
    k_copy16<<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16);
    return cudaGetLastError();
}

cudaError_t launch_convert_f32_to_f16(const float* src, void* dst, int64_t n, int32_t* err, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    k_f32_to_f16<<<stream_grid(s), 256, 0, s>>>(src, static_cast<__half*>(dst), n, err);
    return cudaGetLastError();
}

}  // namespace epsp
