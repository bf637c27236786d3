// k_ffn.cu -- K4: FFN-skip row compaction and scatter.
//
// The reference skips a layer's FFN for every row by returning
// ggml_scale(cur, 0) in build_ffn (patches/llama-prefill-ffn-skip.patch
// :146-149: the residual add survives, the FFN contributes zero), and drops
// non-selected tokens from the batch host-side (src/sparse_prefill.cpp
// :214-232).  Generalised to rows: only the kept rows are gathered into a
// dense [n_keep][hidden] block for the FFN GEMMs, and the FFN output is added
// back into their residual rows; every other row keeps its residual unchanged,
// exactly the zero-contribution semantics.  Pure data movement: HBM-bound,
// 16-byte vector loads/stores, grid sized to the SM count.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "epsp_kernels.h"

namespace epsp {
namespace {

constexpr int kScanThreads = 1024;

// Single CTA: ordered stream compaction of the keep mask -> row ids, count.
__global__ void __launch_bounds__(kScanThreads) k4_scan_keep(const uint8_t* keep, int32_t n_rows, int32_t skip,
                                                             int32_t* row_ids, int32_t* n_keep) {
    __shared__ int warp_tot[kScanThreads / 32];
    if (skip) {
        if (threadIdx.x == 0) *n_keep = 0;
        return;
    }
    const int chunk = (n_rows + kScanThreads - 1) / kScanThreads;
    const int lo = min(n_rows, (int)threadIdx.x * chunk);
    const int hi = min(n_rows, lo + chunk);
    int mine = 0;
    for (int r = lo; r < hi; ++r) mine += keep[r] != 0;
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
    for (int r = lo; r < hi; ++r)
        if (keep[r]) row_ids[pos++] = r;
    if (threadIdx.x == kScanThreads - 1) *n_keep = warp_tot[kScanThreads / 32 - 1];
}

// Gather kept rows: x_kept[i] = x[row_ids[i]], 16-byte chunks, grid-stride.
__global__ void __launch_bounds__(256) k4_gather_rows(const uint4* __restrict__ x, uint4* __restrict__ x_kept,
                                                      const int32_t* __restrict__ row_ids,
                                                      const int32_t* __restrict__ n_keep, int32_t chunks_per_row) {
    const int64_t total = (int64_t)(*n_keep) * chunks_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / chunks_per_row;
        const int64_t c = i - r * chunks_per_row;
        const int64_t src = (int64_t)__ldg(row_ids + r) * chunks_per_row + c;
        x_kept[i] = __ldg(x + src);
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
        const __half2 ha = *reinterpret_cast<const __half2*>(&a);
        const __half2 hb = *reinterpret_cast<const __half2*>(&b);
        const float2 fa = __half22float2(ha), fb = __half22float2(hb);
        __half2 v = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

// residual[row_ids[i]] += ffn_out[i] (fp32 add, rounded to the element type).
template <int DT>
__global__ void __launch_bounds__(256) k4_scatter_add(const uint4* __restrict__ ffn_out, uint4* __restrict__ residual,
                                                      const int32_t* __restrict__ row_ids,
                                                      const int32_t* __restrict__ n_keep, int32_t chunks_per_row) {
    const int64_t total = (int64_t)(*n_keep) * chunks_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / chunks_per_row;
        const int64_t c = i - r * chunks_per_row;
        const int64_t dst = (int64_t)__ldg(row_ids + r) * chunks_per_row + c;
        const uint4 f = __ldg(ffn_out + i);
        uint4 x = residual[dst];
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
        residual[dst] = x;
    }
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

}  // namespace

cudaError_t launch_ffn_compact(const FfnCompactArgs& a, cudaStream_t s) {
    if ((a.hidden * a.elem_bytes) % 16) return cudaErrorInvalidValue;
    k4_scan_keep<<<1, kScanThreads, 0, s>>>(a.keep, a.n_rows, a.skip_layer, a.row_ids, a.n_keep);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.skip_layer) return e;
    const int cpr = a.hidden * a.elem_bytes / 16;
    k4_gather_rows<<<stream_grid(s), 256, 0, s>>>(static_cast<const uint4*>(a.x), static_cast<uint4*>(a.x_kept),
                                                  a.row_ids, a.n_keep, cpr);
    return cudaGetLastError();
}

cudaError_t launch_ffn_scatter(const FfnScatterArgs& a, cudaStream_t s) {
    const int esz = a.dtype == 0 ? 4 : 2;
    if ((a.hidden * esz) % 16) return cudaErrorInvalidValue;
    const int cpr = a.hidden * esz / 16;
    const uint4* f = static_cast<const uint4*>(a.ffn_out);
    uint4* r = static_cast<uint4*>(a.residual);
    switch (a.dtype) {
        case 0: k4_scatter_add<0><<<stream_grid(s), 256, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
        case 1: k4_scatter_add<1><<<stream_grid(s), 256, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
        default: k4_scatter_add<2><<<stream_grid(s), 256, 0, s>>>(f, r, a.row_ids, a.n_keep, cpr); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_convert_f32_to_f16(const float* src, void* dst, int64_t n, int32_t* err, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    k_f32_to_f16<<<stream_grid(s), 256, 0, s>>>(src, static_cast<__half*>(dst), n, err);
    return cudaGetLastError();
}

}  // namespace epsp
