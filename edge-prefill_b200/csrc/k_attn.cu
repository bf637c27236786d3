// k_attn.cu -- K3: page-gated sparse flash attention on sm_100a tensor cores.
//
// Replaces patch :1002-1092 of the reference: the K/V/mask row gathers
// (ggml_get_rows + concat, which materialise copies) and the non-flash
// build_attn_mha over the union.  Here the kept set -- sink page, the selected
// pages, the local window up to the query's own row -- is streamed page by page
// straight from the KV cache into shared memory by TMA and consumed by tcgen05
// MMAs; no copy of K, V or the mask is ever written.  Causality is computed
// from row indices, not read from a mask tensor.
//
// CTA = one (gating block, pair of query tiles, KV head).  A query tile
// packs the G query heads of the KV head: 128 MMA rows = T tokens x G heads
// (T = 128 / G); the CTA owns tiles A = tokens [t0, t0+T) and B = [t0+T,
// t0+2T), so every K/V byte brought on chip serves 2 x G query rows.
//
// Warp roles (384 threads):
//   warp 0   TMA producer: Q of both tiles once; then per KV tile the K and V
//            segments into a 2-stage ring (K and V have their own barriers).
//   warp 1   TMEM owner + MMA issuer (the whole warp runs the loop, one elected
//            lane issues): S = Q K^T (smem x smem), O += P V with P in TMEM.
//            Issue order per KV tile j: PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1),
//            so the tensor core works on one tile while the other's softmax runs;
//            each PV is issued in two halves (KV rows 0-63 once the softmax has
//            stored the first half of P, rows 64-127 once it has stored all of it).
//   warps 4-7 softmax of tile A, warps 8-11 softmax of tile B: each thread owns
//            one query row (one TMEM lane): online softmax in fp32 on exp2
//            (a quarter of the exponentials on the FMA pipe), P written back
//            over S in TMEM as 16-bit, O rescaled in TMEM only when the running
//            max grows by more than 8 (log2 units), and the epilogue O / l.
// TMEM columns: S_A [0,128) S_B [128,256) O_A [256,256+D) O_B [256+D,256+2D);
// P_A / P_B occupy the first 64 columns of S_A / S_B (the next QK into that S
// is issued after the PV that reads the P, and tcgen05 MMAs of one CTA run in
// issue order).  setmaxnreg moves registers from warpgroup 0 to the softmax
// warpgroups.
// Every mbarrier wait is bounded by %globaltimer; a timeout records an error
// word, unwinds, drains in-flight copies/MMAs and frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <climits>
#include <cmath>
#include <cstring>

#include "epsp_kernels.h"
#include "tc100.cuh"

namespace epsp {
namespace {

// NT query tiles per CTA: NT = 2 ping-pongs two tiles on the tensor core in
// one CTA (384 threads, one CTA per SM); NT = 1 runs one tile per CTA with two
// CTAs per SM (256 threads), so one CTA computes while the other drains its
// epilogue.
template <int NT>
__host__ __device__ constexpr int threads_of() { return NT == 2 ? 384 : 256; }
constexpr int kSoftmaxWarpThreads = 128;  // one warpgroup per query tile
constexpr int BM = 128;                  // query rows per tile (TMEM lanes)
constexpr int BN = 128;                  // KV rows per tile
constexpr int kHalfBytes = 128 * 128;    // [128 rows][64 x 16-bit] swizzled sub-tile
__host__ __device__ constexpr uint32_t kColS(int tile) { return tile ? 128u : 0u; }
template <int NT>
__host__ __device__ constexpr uint32_t tmem_cols_of() { return NT == 2 ? 512u : 256u; }
// setmaxnreg splits of the launch's register pool (threads x registers at
// launch: 384 x 168 for NT = 2, 256 x 128 for NT = 1):
//   NT = 2: 128 x 136 + 256 x 184 = 64,512 <= 64,512
//   NT = 1: 128 x 96 + 128 x 160 = 32,768 <= 32,768
// WG0 (producer, MMA) 136 / softmax 184 registers: with 96 / 200 ptxas
// spilled in the producer and MMA loops and the kernel ran 3.5 % slower;
// 152 / 176 measured within 0.5 % of 136 / 184.
#ifndef K3_REGS_WG0
#define K3_REGS_WG0 136
#endif
#ifndef K3_REGS_SOFTMAX
#define K3_REGS_SOFTMAX 184
#endif
template <int NT>
__host__ __device__ constexpr int regs_wg0_of() { return NT == 2 ? K3_REGS_WG0 : 96; }
template <int NT>
__host__ __device__ constexpr int regs_softmax_of() { return NT == 2 ? K3_REGS_SOFTMAX : 160; }
static_assert(128 * K3_REGS_WG0 + 256 * K3_REGS_SOFTMAX <= 384 * 168, "setmaxnreg split above the launch's pool");
// One exponential pair in this many goes to the FMA pipe (exp2_poly2), the
// rest to MUFU ex2; measured best of 2, 3, 4 and 8 on B200 (2: -13 %, 3: -2 %,
// 8: -7 % against 4).
#ifndef K3_KSTAGES
#define K3_KSTAGES 2
#endif
#ifndef K3_POLY_EVERY
#define K3_POLY_EVERY 4
#endif
constexpr int kPolyEvery = K3_POLY_EVERY;

template <int D, int NT>
struct Layout {
    static constexpr int kHalves = D / 64;
    static constexpr int kQBytes = kHalves * kHalfBytes;      // one query tile
    static constexpr int kStageBytes = kHalves * kHalfBytes;  // one K or V tile
    // ring depths (a third K stage fits in shared memory with two query
    // tiles but measured 0.6 % slower)
    static constexpr int kStagesK = NT == 2 ? K3_KSTAGES : 1;
    static constexpr int kStagesV = NT;
    static constexpr int kOffQ = 0;                           // Q of the NT tiles
    static constexpr int kOffK = kOffQ + NT * kQBytes;
    static constexpr int kOffV = kOffK + kStagesK * kStageBytes;
    static constexpr int kOffBar = kOffV + kStagesV * kStageBytes;
    static constexpr int kBytes = kOffBar + 256;
    static constexpr uint32_t kColO(int tile) { return NT * 128 + tile * D; }
};

enum Bar { kQFull = 0, kKFull = 1, kKEmpty = 4, kVFull = 7, kVEmpty = 9, kSFull = 11, kPFull = 13, kPVDone = 15, kDone = 17, kPHalf = 18, kNumBars = 20 };

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float max3f(float x, float y, float z) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
    return r;
}

// 2^x on the FMA pipe for a pair (used for part of the softmax so that the
// MUFU pipe is not the only exp2 unit).  x is clamped to >= -120 (so that
// 2^n * p(r) stays a normal float; masked -inf entries give ~1e-36), split as
// x = n + r with n = round(x) (added to 1.5 * 2^23, the integer lands in the
// low mantissa bits) and r in [-0.5, 0.5]; 2^r comes from a degree-3
// polynomial fitted here for minimum relative error on that interval (max
// relative error 7.5e-5, far below the 2^-9 of the 16-bit P it feeds), and n
// is added into the exponent field.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    x.x = fmaxf(x.x, -120.0f);
    x.y = fmaxf(x.y, -120.0f);
    const float2 tt = __fadd2_rn(x, magic);
    const float2 n = __fadd2_rn(tt, make_float2(-12582912.0f, -12582912.0f));
    const float2 r = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
    float2 p = __ffma2_rn(make_float2(0.05517132207751274f, 0.05517132207751274f), r,
                          make_float2(0.24261054396629333f, 0.24261054396629333f));
    p = __ffma2_rn(p, r, make_float2(0.6932609677314758f, 0.6932609677314758f));
    p = __ffma2_rn(p, r, make_float2(0.9999281167984009f, 0.9999281167984009f));
    const int ex = __float_as_int(tt.x) << 23, ey = __float_as_int(tt.y) << 23;
    return make_float2(__int_as_float(__float_as_int(p.x) + ex), __int_as_float(__float_as_int(p.y) + ey));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

// Kept-set geometry of one CTA: the ordered list of SEG-row segments
// (sink page, selected pages, pooled rows, local window cut at the tile's
// last token).
#ifdef K3_TRACE
// Diagnostic build only: per-tile clock64 stamps of the first 64 CTAs.
__device__ unsigned int g_k3_trace[64 * 3 * 64 * 8];
#define K3T(role, j, ev)                                                                                  \
    do {                                                                                                  \
        if (blockIdx.x < 64 && (j) < 64 && lane == 0)                                                     \
            g_k3_trace[((blockIdx.x * 3 + (role)) * 64 + (j)) * 8 + (ev)] = (unsigned)(clock64() - t_start); \
    } while (0)
#else
#define K3T(role, j, ev) \
    do {                 \
    } while (0)
#endif

struct Segs {
    int gated, P, sps, k_sel, L0, n_seg, kv_len;
    int n_pool, n_pseg, prow0;  // pooled rows, their segments, first row in pk / pv
    const int32_t* sel;
};

// Segment i: row >= 0 is its first row in the KV cache (causal) or, when
// pooled > 0, in the pooled rows (pooled = its valid rows, all visible);
// row < 0: absent (past the kept set, or a bad selection).
struct SegRef {
    int row, pooled;
};

template <int SEG>
__device__ __forceinline__ SegRef seg_ref(const Segs& s, int i, bool& bad) {
    if (i >= s.n_seg) return {-1, 0};
    if (!s.gated) return {i * SEG, 0};
    if (i < s.sps) return {i * SEG, 0};
    int j = i - s.sps;
    if (j < s.k_sel * s.sps) {
        const int page = __ldg(s.sel + j / s.sps);
        const int r = page * s.P + (j % s.sps) * SEG;
        if (page < 0 || r + SEG > s.kv_len) {
            bad = true;
            return {-1, 0};
        }
        return {r, 0};
    }
    j -= s.k_sel * s.sps;
    if (j < s.n_pseg) return {s.prow0 + j * SEG, min(SEG, s.n_pool - j * SEG)};
    j -= s.n_pseg;
    return {s.L0 + j * SEG, 0};
}

template <bool BF16, int D, int SEG, bool XCHG, int NT>
__global__ void __launch_bounds__(threads_of<NT>(), NT == 2 ? 1 : 2)
    k3_sparse_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmPK,
                        const __grid_constant__ CUtensorMap tmPV, const __grid_constant__ AttnArgs a) {
    using LY = Layout<D, NT>;
    constexpr int SPT = BN / SEG;  // segments per KV tile
    constexpr int kThreads = threads_of<NT>();
    constexpr int KSK = LY::kStagesK;
    constexpr int KSV = LY::kStagesV;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::kOffBar + kNumBars * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::kOffBar + kNumBars * 8 + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int Hkv = a.n_head_kv;
    const int G = a.n_head / Hkv;
    const int T = BM / G;  // tokens per query tile
    const int L = block_len(a.n_tok, a.q_subblock);
    const int tpb = (L + NT * T - 1) / (NT * T);  // CTAs per gating block
    // CTA id in the call's head-major grid [Hkv][blk_count][tpb]; the range
    // [cta_begin, cta_begin + gridDim.x) runs backwards so the heavier CTAs
    // (late gating blocks) start first and the cheap ones fill the tail.
    const int id = a.cta_begin + (int)(gridDim.x - 1 - blockIdx.x);
    const int h = id / (a.blk_count * tpb);
    const int blk = a.blk_begin + (id % (a.blk_count * tpb)) / tpb;
    const int b0 = a.u0 + blk * L;
    const int b1 = min(a.u0 + a.n_tok, b0 + L);
    const int t0 = b0 + (id % tpb) * NT * T;
    if (t0 >= b1) return;  // whole CTA: tail of a short last block
    const int t_end = min(t0 + NT * T, b1);  // last token of the CTA + 1

    const BlockPlan plan = plan_block(a.gate, b0, b1, __ldg(a.k_budget + h));
    Segs sg;
    sg.gated = plan.gated;
    sg.P = a.gate.page_size;
    sg.sps = a.gate.page_size / SEG;
    // K2's counts replace the plan's when given (head routing changes them)
    const int64_t bh = (int64_t)blk * Hkv + h;
    sg.k_sel = plan.gated ? (a.cnt != nullptr ? min(__ldg(a.cnt + bh), a.sel_cap) : plan.k_sel) : 0;
    sg.L0 = plan.gated ? plan.lsp * a.gate.page_size : 0;
    sg.kv_len = a.kv_len;
    sg.sel = a.sel + ((int64_t)blk * Hkv + h) * a.sel_cap;
    sg.n_pool = (plan.gated && a.pk != nullptr)
                    ? (a.pool_cnt != nullptr ? min(__ldg(a.pool_cnt + bh), a.pool_stride) : plan.n_pool)
                    : 0;
    sg.n_pseg = (sg.n_pool + SEG - 1) / SEG;
    sg.prow0 = blk * a.pool_stride;
    {
        const int n_loc = (t_end - sg.L0 + SEG - 1) / SEG;
        sg.n_seg = plan.gated ? sg.sps + sg.k_sel * sg.sps + sg.n_pseg + n_loc : n_loc;
    }
    const int n_tiles = (sg.n_seg + SPT - 1) / SPT;

    // ------------------------------------------------------------- setup --
    if (threadIdx.x == 0) {
        for (int i = 0; i < kNumBars; ++i) tc::mbar_init(&bars[i], 1);
        tc::mbar_init(&bars[kPFull + 0], kSoftmaxWarpThreads);
        tc::mbar_init(&bars[kPFull + 1], kSoftmaxWarpThreads);
        tc::mbar_init(&bars[kPHalf + 0], kSoftmaxWarpThreads);
        tc::mbar_init(&bars[kPHalf + 1], kSoftmaxWarpThreads);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch_desc(&tmQ);
        tc::tma_prefetch_desc(&tmK);
        tc::tma_prefetch_desc(&tmV);
        if (sg.n_pool > 0) {
            tc::tma_prefetch_desc(&tmPK);
            tc::tma_prefetch_desc(&tmPV);
        }
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, tmem_cols_of<NT>());
        tc::tmem_relinquish();
    }
    // Q rows past T*G are never written by TMA: zero them so no stale shared
    // memory reaches the tensor cores.
    {
        const int rows_used = T * G;
        if (rows_used < BM) {
            const int n16 = (BM - rows_used) * 8;  // 16-byte chunks per half
            for (int i = threadIdx.x; i < n16 * NT * LY::kHalves; i += kThreads) {
                const int hf = i / n16, k = i % n16;  // hf: (tile, half)
                uint4* p = reinterpret_cast<uint4*>(smem + LY::kOffQ + hf * kHalfBytes + rows_used * 128) + k;
                *p = make_uint4(0, 0, 0, 0);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint64_t tmo = a.timeout_ns;
#ifdef K3_TRACE
    const long long t_start = clock64();
#endif

    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(regs_wg0_of<NT>()));
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(regs_softmax_of<NT>()));
    }

    if (warp == 0) {
        // ------------------------------------------------------ producer --
        // Lane 0 of warp 0 loads Q and both rings.  (Loading the V ring from
        // warp 2 in a loop of its own measured 0.5-1 % slower.)
        if (lane == 0) {
            bool ok = true;
            const int qbytes = NT * LY::kHalves * 64 * 2 * T * G;
            tc::mbar_arrive_expect_tx(&bars[kQFull], qbytes);
#pragma unroll
            for (int tile = 0; tile < NT; ++tile)
#pragma unroll
                for (int hf = 0; hf < LY::kHalves; ++hf)
                    tc::tma_load_3d(smem + LY::kOffQ + tile * LY::kQBytes + hf * kHalfBytes, &tmQ, &bars[kQFull],
                                    hf * 64, h * G, t0 + tile * T - a.u0);
            bool bad = false;
            int kt = 0, vt = 0;  // K / V tiles whose copies were issued
            int where = 0, wj = 0;
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int sk = j % KSK, sv = j % KSV;
                const uint32_t park = ((j / KSK) & 1) ^ 1, parv = ((j / KSV) & 1) ^ 1;
                int rows[SPT];
                bool pooled[SPT];
#pragma unroll
                for (int q = 0; q < SPT; ++q) {
                    const SegRef sr = seg_ref<SEG>(sg, j * SPT + q, bad);
                    pooled[q] = sr.row >= 0 && sr.pooled > 0;
                    if (a.paging.block_rows <= 0) {
                        rows[q] = sr.row < 0 ? 0 : sr.row;  // absent segment: load rows [0,SEG), masked later
                    } else if (sr.row < 0) {
                        rows[q] = a.paging.pool_rows;  // absent: past the pool, zeros
                    } else if (pooled[q]) {
                        rows[q] = sr.row;
                    } else {
                        bool badt = false;  // a cache segment lies in one page, hence one block
                        rows[q] = phys_row(a.paging, sr.row, badt);
                        if (badt) {
                            atomicCAS(a.err, 0, kDevBadBlockTable);
                            rows[q] = a.paging.pool_rows;
                        }
                    }
                }
                if (!tc::mbar_wait(&bars[kKEmpty + sk], park, tmo)) { ok = false; where = 0x11; wj = j; break; }
                tc::mbar_arrive_expect_tx(&bars[kKFull + sk], LY::kStageBytes);
#pragma unroll
                for (int q = 0; q < SPT; ++q)
#pragma unroll
                    for (int hf = 0; hf < LY::kHalves; ++hf)
                        tc::tma_load_3d(smem + LY::kOffK + sk * LY::kStageBytes + hf * kHalfBytes + q * SEG * 128,
                                        pooled[q] ? &tmPK : &tmK, &bars[kKFull + sk], hf * 64, h, rows[q]);
                kt = j + 1;
                if (!tc::mbar_wait(&bars[kVEmpty + sv], parv, tmo)) { ok = false; where = 0x12; wj = j; break; }
                tc::mbar_arrive_expect_tx(&bars[kVFull + sv], LY::kStageBytes);
#pragma unroll
                for (int q = 0; q < SPT; ++q)
#pragma unroll
                    for (int hf = 0; hf < LY::kHalves; ++hf)
                        tc::tma_load_3d(smem + LY::kOffV + sv * LY::kStageBytes + hf * kHalfBytes + q * SEG * 128,
                                        pooled[q] ? &tmPV : &tmV, &bars[kVFull + sv], hf * 64, h, rows[q]);
                vt = j + 1;
            }
            if (bad) atomicCAS(a.err, 0, kDevBadSelection);
            if (!ok) {
                report_error(a.err, kDevWaitProducer, where, wj);
                *abort_flag = 1;
            }
            // Drain: copies still in flight must land before the CTA exits (the
            // ring-depth most recent tiles of each ring; older ones were consumed).
            for (int j = kt - KSK; j < kt; ++j)
                if (j >= 0) tc::mbar_wait(&bars[kKFull + j % KSK], (j / KSK) & 1, tmo);
            for (int j = vt - KSV; j < vt; ++j)
                if (j >= 0) tc::mbar_wait(&bars[kVFull + j % KSV], (j / KSV) & 1, tmo);
            tc::mbar_wait(&bars[kQFull], 0, tmo);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        // The whole warp runs the loop; one elected lane issues each MMA.
        constexpr uint32_t idesc_qk = tc::make_idesc_f16(BF16, BM, BN, false);
        constexpr uint32_t idesc_pv = tc::make_idesc_f16(BF16, BM, D, true);
        const uint64_t dq0 = tc::make_sdesc_sw128(tc::smem_u32(smem + LY::kOffQ), 16, 1024);
        const uint64_t dk0 = tc::make_sdesc_sw128(tc::smem_u32(smem + LY::kOffK), 16, 1024);
        const uint64_t dv0 = tc::make_sdesc_sw128(tc::smem_u32(smem + LY::kOffV), kHalfBytes, 1024);
        const bool leader = tc::elect_one();
        auto wait_all = [&](uint64_t* bar, uint32_t par) -> bool {
            const bool w = tc::mbar_wait(bar, par, tmo);
            return __all_sync(0xffffffffu, w);
        };
        auto qk = [&](int tile, int j) {  // S_tile = Q_tile K_j^T (K of stage j & 1)
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t off = (uint64_t)(((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4);
                    tc::mma_ss(tmem + kColS(tile), dq0 + (uint64_t)((tile * LY::kQBytes) >> 4) + off,
                               dk0 + (uint64_t)(((j % KSK) * LY::kStageBytes) >> 4) + off, idesc_qk, kk > 0 ? 1u : 0u);
                }
                tc::mma_commit(&bars[kSFull + tile]);
            }
            __syncwarp();
        };
        // O_tile += P_tile V_j over KV rows [64 part, 64 part + 64); the
        // second part commits PVDone
        auto pv = [&](int tile, int j, int part) {
            const int k0 = part * (BN / 32), k1 = k0 + BN / 32;
            if (leader) {
#pragma unroll
                for (int kk = k0; kk < k1; ++kk) {
                    // MN-major V: 16 KV rows (2 atoms of 8 x 128 B) per step; the
                    // D/64 column chunks sit kHalfBytes apart (LBO).
                    const uint64_t dv = dv0 + (uint64_t)(((j % KSV) * LY::kStageBytes + kk * 16 * 128) >> 4);
                    tc::mma_ts(tmem + LY::kColO(tile), tmem + kColS(tile) + kk * 8, dv, idesc_pv,
                               (j > 0 || kk > 0) ? 1u : 0u);
                }
                if (part != 0) tc::mma_commit(&bars[kPVDone + tile]);
            }
            __syncwarp();
        };
        auto commit = [&](int bar) {
            if (leader) tc::mma_commit(&bars[bar]);
            __syncwarp();
        };
        bool ok = wait_all(&bars[kQFull], 0);
        if (ok) ok = wait_all(&bars[kKFull + 0], 0);
        if (ok) {
            tc::fence_after_sync();
            qk(0, 0);
            if constexpr (NT == 2) qk(1, 0);
            commit(kKEmpty + 0);
        }
        int mma_j = 0;
        for (int j = 0; j < n_tiles && ok; ++j) {
            const int s = j % KSV;               // V stage of tile j
            const int jn = j + 1, sn = jn % KSK;  // K stage of tile j + 1
            mma_j = j;
            K3T(2, j, 0);
            if (!(ok = wait_all(&bars[kPHalf + 0], j & 1))) break;
            K3T(2, j, 1);
            if (!(ok = wait_all(&bars[kVFull + s], (j / KSV) & 1))) break;
            K3T(2, j, 2);
            if (a.paging.block_rows > 0) {
                // A paged pool's block holds whatever its rows past kv_len last
                // held: zero those V rows (their P is 0, and 0 * NaN is not 0)
                // before the tensor core reads them.
                bool any = false;
#pragma unroll
                for (int q = 0; q < SPT; ++q) {
                    bool bad = false;
                    const SegRef sr = seg_ref<SEG>(sg, j * SPT + q, bad);
                    if (sr.row < 0 || sr.pooled > 0 || sr.row + SEG <= a.kv_len) continue;
                    const int first = a.kv_len - sr.row;  // rows [first, SEG) of the segment
                    for (int i = lane; i < (SEG - first) * 8 * LY::kHalves; i += 32) {
                        const int hf = i / ((SEG - first) * 8), rem = i % ((SEG - first) * 8);
                        *reinterpret_cast<uint4*>(smem + LY::kOffV + s * LY::kStageBytes + hf * kHalfBytes +
                                                  (q * SEG + first + rem / 8) * 128 + (rem % 8) * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                    any = true;
                }
                if (any) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            tc::fence_after_sync();
            // the first half of P is in TMEM: its PV runs while the softmax
            // finishes the second half
            pv(0, j, 0);
            if (!(ok = wait_all(&bars[kPFull + 0], j & 1))) break;
            K3T(2, j, 3);
            tc::fence_after_sync();
            pv(0, j, 1);
            if constexpr (NT == 2) {
                if (jn < n_tiles) {
                    if (!(ok = wait_all(&bars[kKFull + sn], (jn / KSK) & 1))) break;
                    K3T(2, j, 4);
                    tc::fence_after_sync();
                    qk(0, jn);
                }
                if (!(ok = wait_all(&bars[kPHalf + 1], j & 1))) break;
                K3T(2, j, 5);
                tc::fence_after_sync();
                pv(1, j, 0);
                if (!(ok = wait_all(&bars[kPFull + 1], j & 1))) break;
                K3T(2, j, 6);
                tc::fence_after_sync();
                pv(1, j, 1);
                commit(kVEmpty + s);
                if (jn < n_tiles) {
                    qk(1, jn);
                    commit(kKEmpty + sn);
                }
            } else {
                commit(kVEmpty + s);
                if (jn < n_tiles) {
                    if (!(ok = wait_all(&bars[kKFull + sn], (jn / KSK) & 1))) break;
                    tc::fence_after_sync();
                    qk(0, jn);
                    commit(kKEmpty + sn);
                }
            }
        }
        if (!ok && lane == 0) {
            report_error(a.err, kDevWaitMma, 0x20, mma_j);
            *abort_flag = 1;
        }
        // Every MMA issued must retire before TMEM is freed.
        commit(kDone);
        wait_all(&bars[kDone], 0);
    } else if (warp >= 4) {
        // ------------------------------------------------------- softmax --
        const int tile = (warp - 4) >> 2;       // 0: tile A, 1: tile B
        const int wq = warp & 3;                // TMEM lane quadrant
        const int row = wq * 32 + lane;         // query row of the tile
        const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
        const int tt0 = t0 + tile * T;          // first token of this tile
        const bool row_used = row < T * G;
        const int t = row_used ? tt0 + row / G : INT_MAX;
        const float sl2 = a.kq_scale * 1.4426950408889634f;
        const float2 sl2_2 = make_float2(sl2, sl2);
        const uint32_t s_col = kColS(tile);
        const uint32_t o_col = LY::kColO(tile);
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        int sm_j = 0;
        // Segment ranges of the kept set, for the masks without reading the
        // page list per tile: a selected page lies wholly before the local
        // window, so it is visible to every row of the block.  One scan of the
        // list per CTA checks that; a list with an absent, out-of-range or
        // late page takes the per-segment path (seg_ref) instead.
        const int e_sink = sg.gated ? sg.sps : 0;
        const int e_sel = e_sink + (sg.gated ? sg.k_sel * sg.sps : 0);
        const int e_pool = e_sel + (sg.gated ? sg.n_pseg : 0);
        bool list_fast = true;
        if (sg.gated) {
            const int lim_row = min(sg.kv_len, sg.L0);
            for (int i = lane; i < sg.k_sel; i += 32) {
                const int page = __ldg(sg.sel + i);
                if (page < 0 || (int64_t)page * sg.P + sg.P > lim_row) list_fast = false;
            }
            list_fast = __all_sync(0xffffffffu, list_fast);
        }
        for (int j = 0; j < n_tiles; ++j) {
            sm_j = j;
            if ((warp & 3) == 0) K3T(tile, j, 0);
            bool w = tc::mbar_wait(&bars[kSFull + tile], j & 1, tmo);
            if ((warp & 3) == 0) K3T(tile, j, 1);
            if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
            tc::fence_after_sync();
            // Causal / absent-segment mask limits, only on tiles that need it.
            int lim[SPT];
            bool masked = false;
            {
                bool bad = false;
#pragma unroll
                for (int q = 0; q < SPT; ++q) {
                    const int idx = j * SPT + q;
                    SegRef sr;
                    if (!list_fast) {
                        sr = seg_ref<SEG>(sg, idx, bad);
                    } else if (idx >= sg.n_seg) {
                        sr = {-1, 0};
                    } else if (idx < e_sink || !sg.gated) {
                        sr = {idx * SEG, 0};
                    } else if (idx < e_sel) {
                        lim[q] = SEG - 1;  // a selected page: before the block, never masked
                        continue;
                    } else if (idx < e_pool) {
                        sr = {sg.prow0 + (idx - e_sel) * SEG, min(SEG, sg.n_pool - (idx - e_sel) * SEG)};
                    } else {
                        sr = {sg.L0 + (idx - e_pool) * SEG, 0};
                    }
                    const int r = sr.row;
                    if (r >= 0 && sr.pooled > 0) {  // pooled rows: visible to every row of the block
                        if (sr.pooled < SEG) masked = true;
                        lim[q] = sr.pooled - 1;
                    } else {
                        if (r < 0 || r + SEG - 1 > tt0) masked = true;
                        lim[q] = r < 0 ? -1 : (t >= r + SEG - 1 ? SEG - 1 : t - r);
                    }
                }
            }
            // Pass 1: row max over the 128 columns, 64 at a time, the second
            // half first so that the first half stays in registers for pass 2.
            auto load_half = [&](int hh, uint32_t (&s)[64]) {
                tc::tmem_ld32(tmem + lane_addr + s_col + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
                tc::tmem_ld32(tmem + lane_addr + s_col + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
                tc::tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        const int c = 64 * hh + i;
                        if ((c % SEG) > lim[c / SEG]) s[i] = __float_as_uint(-INFINITY);
                    }
                }
            };
            auto half_max = [&](const uint32_t (&s)[64]) -> float {
                float mt[22];
#pragma unroll
                for (int i = 0; i < 21; ++i)
                    mt[i] = max3f(__uint_as_float(s[3 * i]), __uint_as_float(s[3 * i + 1]), __uint_as_float(s[3 * i + 2]));
                mt[21] = __uint_as_float(s[63]);
#pragma unroll
                for (int i = 0; i < 7; ++i) mt[i] = max3f(mt[3 * i], mt[3 * i + 1], mt[3 * i + 2]);
                mt[7] = mt[21];
                return max3f(max3f(mt[0], mt[1], mt[2]), max3f(mt[3], mt[4], mt[5]), fmaxf(mt[6], mt[7]));
            };
            uint32_t s0[64];  // columns [0, 64), kept for pass 2
            float mx;
            {
                uint32_t s1[64];
                load_half(1, s1);
                mx = half_max(s1);
            }
            load_half(0, s0);
            mx = fmaxf(mx, half_max(s0));

            if ((warp & 3) == 0) K3T(tile, j, 2);
            const float m_new = fmaxf(m_run, mx * sl2);
            bool need;
            float m_use;
            if (j == 0) {
                m_use = m_new;
                need = false;
            } else {
                need = m_new > m_run + 8.0f;
                m_use = need ? m_new : m_run;
            }
            const float2 nm2 = make_float2(-m_use, -m_use);
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
            // Pass 2: exponentials, 64 columns at a time; P of columns [64hh,
            // 64hh+64) goes to TMEM columns [32hh, 32hh+32) of S, which pass 2
            // has already consumed: the first half from the registers pass 1
            // left, then the second half loaded again.
            auto exp_half = [&](int hh, const uint32_t (&s)[64]) {
                uint32_t pk[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[2 * c]), __uint_as_float(s[2 * c + 1])),
                                                sl2_2, nm2);
                    float2 p;
                    if ((c % kPolyEvery) == kPolyEvery - 1) {
                        p = exp2_poly2(x);  // a share of the pairs on the FMA pipe
                    } else {
                        p.x = ex2(x.x);
                        p.y = ex2(x.y);
                    }
                    acc[c & 3] = __fadd2_rn(acc[c & 3], p);
                    pk[c] = pack2<BF16>(p.x, p.y);
                }
                tc::tmem_st32(tmem + lane_addr + s_col + 32 * hh, pk);
            };

            float alpha = 1.f;
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // O may only be touched once PV(j-1) of this tile has retired
                // (it has: S(j) is committed after it, but the wait is cheap
                // on this rare path).
                w = tc::mbar_wait(&bars[kPVDone + tile], (j - 1) & 1, tmo);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                {
                    alpha = need ? ex2(m_run - m_use) : 1.f;
                    tc::fence_after_sync();
#pragma unroll
                    for (int i = 0; i < D / 32; ++i) {
                        uint32_t o[32];
                        tc::tmem_ld32(tmem + lane_addr + o_col + 32 * i, o);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                        tc::tmem_st32(tmem + lane_addr + o_col + 32 * i, o);
                    }
                    load_half(0, s0);  // reloaded rather than held across the rescale (register pressure)
                }
            }
            // O is rescaled (if at all) before any PV of this tile: signal the
            // first half of P as soon as it is in TMEM, then the second
            exp_half(0, s0);
            if ((warp & 3) == 0) K3T(tile, j, 5);
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(&bars[kPHalf + tile]);
            if ((warp & 3) == 0) K3T(tile, j, 3);
            {
                uint32_t s1[64];
                load_half(1, s1);
                if ((warp & 3) == 0) K3T(tile, j, 6);
                exp_half(1, s1);
                if ((warp & 3) == 0) K3T(tile, j, 7);
            }
            const float2 s01 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
            l_run = l_run * alpha + (s01.x + s01.y);
            m_run = m_use;
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(&bars[kPFull + tile]);
            if ((warp & 3) == 0) K3T(tile, j, 4);
        }
        if (ok) {
            bool w = tc::mbar_wait(&bars[kPVDone + tile], (n_tiles - 1) & 1, tmo);
            ok = __all_sync(0xffffffffu, w);
        }
        if (!ok) {
            if (lane == 0) report_error(a.err, kDevWaitSoftmax, 0x30 + 0x10 * tile, sm_j);
            *abort_flag = 1;
        }
        // ------------------------------------------------------ epilogue --
        const int g = row % G;
        const bool store = row_used && t < min(tt0 + T, b1);
        if constexpr (!XCHG) {
            if (ok) {
                tc::fence_after_sync();
                const float inv_l = 1.f / l_run;
                const int out_heads = a.out_heads > 0 ? a.out_heads : a.n_head;
                const int64_t out_off = ((int64_t)(t - a.u0) * out_heads + a.out_head0 + (int64_t)h * G + g) * D;
#pragma unroll
                for (int i = 0; i < D / 32; ++i) {
                    uint32_t o[32];
                    tc::tmem_ld32(tmem + lane_addr + o_col + 32 * i, o);
                    tc::tmem_wait_ld();
                    if (store) {
                        if (a.out_dtype == 0) {
                            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + out_off + 32 * i);
#pragma unroll
                            for (int c = 0; c < 8; ++c)
                                dst[c] = make_float4(__uint_as_float(o[4 * c]) * inv_l,
                                                     __uint_as_float(o[4 * c + 1]) * inv_l,
                                                     __uint_as_float(o[4 * c + 2]) * inv_l,
                                                     __uint_as_float(o[4 * c + 3]) * inv_l);
                        } else {
                            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + out_off + 32 * i);
                            const bool obf = a.out_dtype == 2;
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                uint32_t w4[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float x0 = __uint_as_float(o[8 * c + 2 * e]) * inv_l;
                                    const float x1 = __uint_as_float(o[8 * c + 2 * e + 1]) * inv_l;
                                    w4[e] = obf ? pack2<true>(x0, x1) : pack2<false>(x0, x1);
                                }
                                dst[c] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                            }
                        }
                    }
                }
            }
        } else {
            // Exchange: the tile (16-bit) is staged in the 128-byte-swizzled
            // layout of the Q tile it overwrites (every QK of this tile has
            // retired) and stored from there to each destination, unless it
            // straddles the end of its gating block inside the call (the rows
            // past it belong to another CTA): then each thread stores its own row.
            const int64_t out_off = ((int64_t)(t - a.u0) * a.out_heads + a.out_head0 + (int64_t)h * G + g) * D;
            const bool staged = tt0 + T <= b1 || b1 == a.u0 + a.n_tok;
            unsigned char* stage = smem + LY::kOffQ + tile * LY::kQBytes;
            if (ok) {
                tc::fence_after_sync();
                const float inv_l = 1.f / l_run;
                const bool obf = a.out_dtype == 2;
#pragma unroll
                for (int i = 0; i < D / 32; ++i) {
                    uint32_t o[32];
                    tc::tmem_ld32(tmem + lane_addr + o_col + 32 * i, o);
                    tc::tmem_wait_ld();
                    if (!staged && !store) continue;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t w4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float x0 = __uint_as_float(o[8 * c + 2 * e]) * inv_l;
                            const float x1 = __uint_as_float(o[8 * c + 2 * e + 1]) * inv_l;
                            w4[e] = obf ? pack2<true>(x0, x1) : pack2<false>(x0, x1);
                        }
                        const uint4 v4 = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                        if (staged) {
                            const int chunk = (i & 1) * 4 + c;
                            *reinterpret_cast<uint4*>(stage + (i >> 1) * kHalfBytes + row * 128 +
                                                      ((chunk ^ (row & 7)) << 4)) = v4;
                        } else if (a.mc_dest != nullptr) {
                            tc::multimem_st16(reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.mc_dest) + out_off +
                                                                       32 * i) + c, v4);
                        } else {
                            for (int r = 0; r < a.n_dest; ++r)
                                reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.dest[r]) + out_off + 32 * i)[c] = v4;
                        }
                    }
                }
            }
            // Stores of the staged tile by the warpgroup's threads, coalesced:
            // a warp writes 512 contiguous bytes of one token's G x D output
            // per instruction to each destination, in a per-tile rotated rank
            // order so the ranks' CTAs spread over every peer's links.  (TMA
            // tile stores would queue behind the SM's K/V loads.)  Nothing
            // waits for them here: the kernel's completion orders them before
            // the signal kernel that follows on the stream.
            if (staged) {
                tc::named_bar_sync(1 + tile, kSoftmaxWarpThreads);  // every thread of the warpgroup, aborted or not
                if (tt0 < b1) {
                    const int tid = (int)threadIdx.x - (tile + 1) * kSoftmaxWarpThreads;
                    const int n_tt = min(T, b1 - tt0);
                    constexpr int kCh = D / 8;  // 16-byte chunks per head row
                    const int cpt = G * kCh;    // chunks per token
                    const int total = n_tt * cpt;
                    const int r0 = (int)((blockIdx.x * 2u + tile) % (unsigned)a.n_dest);
                    for (int c = tid; c < total; c += kSoftmaxWarpThreads) {
                        const int tl = c / cpt, cc = c % cpt;
                        const int gg = cc / kCh, dc = cc % kCh;
                        const int srow = tl * G + gg;
                        const uint4 v = *reinterpret_cast<const uint4*>(stage + (dc >> 3) * kHalfBytes + srow * 128 +
                                                                        (((dc & 7) ^ (srow & 7)) << 4));
                        const int64_t off = ((int64_t)(tt0 - a.u0 + tl) * a.out_heads + a.out_head0 + (int64_t)h * G) *
                                                D * 2 + (int64_t)cc * 16;
                        if (a.mc_dest != nullptr) {
                            tc::multimem_st16(static_cast<char*>(a.mc_dest) + off, v);
                        } else {
                            for (int i = 0; i < a.n_dest; ++i) {
                                const int r = r0 + i < a.n_dest ? r0 + i : r0 + i - a.n_dest;
                                *reinterpret_cast<uint4*>(static_cast<char*>(a.dest[r]) + off) = v;
                            }
                        }
                    }
                }
            }
            // multicast stores are performed at system scope before the
            // signal kernel that follows on the stream adds to the counters
            if (a.mc_dest != nullptr) __threadfence_system();
        }
    }

    // ------------------------------------------------------------ teardown --
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, tmem_cols_of<NT>());
    }
}

#ifdef K3_TRACE
}  // namespace
}  // namespace epsp
extern "C" int ep_k3_trace_read(void* host, size_t bytes) {
    return (int)cudaMemcpyFromSymbol(host, epsp::g_k3_trace, bytes);
}
namespace epsp {
namespace {
#endif
// ---------------------------------------------------------------- host side --
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 3-D map over [dim2][dim1][dim0] 16-bit elements, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, bool bf16, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t box0,
              uint32_t box1, uint32_t box2) {
    auto enc = get_encode();
    if (!enc) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
    const cuuint32_t box[3] = {box0, box1, box2};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <bool BF16, int D, int SEG, bool XCHG, int NT>
cudaError_t launch_t(const AttnArgs& a, cudaStream_t s) {
    constexpr int SEGX = SEG;  // TMA box rows: one segment (a page)
    const int G = a.n_head / a.n_head_kv;
    const int T = BM / G;
    CUtensorMap mq, mk, mv, mpk, mpv;
    if (!make_map(&mq, a.q, BF16, D, a.n_head, a.n_tok, 64, G, T)) return cudaErrorInvalidValue;
    const uint64_t kv_rows = a.paging.block_rows > 0 ? (uint64_t)a.paging.pool_rows : (uint64_t)a.kv_len;
    if (!make_map(&mk, a.k, BF16, D, a.n_head_kv, kv_rows, 64, 1, SEGX)) return cudaErrorInvalidValue;
    if (!make_map(&mv, a.v, BF16, D, a.n_head_kv, kv_rows, 64, 1, SEGX)) return cudaErrorInvalidValue;
    if (a.pk != nullptr) {
        // pooled rows [blocks * pool_stride][Hkv][d], loaded SEG rows at a time like the cache
        if (a.pool_stride % SEG || a.pool_rows_total < a.pool_stride) return cudaErrorInvalidValue;
        if (!make_map(&mpk, a.pk, BF16, D, a.n_head_kv, a.pool_rows_total, 64, 1, SEGX)) return cudaErrorInvalidValue;
        if (!make_map(&mpv, a.pv, BF16, D, a.n_head_kv, a.pool_rows_total, 64, 1, SEGX)) return cudaErrorInvalidValue;
    } else {
        mpk = mk;  // never read: no pooled segment exists
        mpv = mv;
    }
    const int smem = Layout<D, NT>::kBytes + 1024;
    int dev = 0;
    cudaGetDevice(&dev);
    // one bit per device ordinal < 32 whose attribute is set; atomic, since
    // host threads driving different devices launch concurrently
    static std::atomic<unsigned> set_mask{0};
    if (dev >= 32 || !(set_mask.load(std::memory_order_acquire) & (1u << dev))) {
        const cudaError_t e = cudaFuncSetAttribute(k3_sparse_attention<BF16, D, SEG, XCHG, NT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 32) set_mask.fetch_or(1u << dev, std::memory_order_release);
    }
    const int L = block_len(a.n_tok, a.q_subblock);
    const int tpb = (L + NT * T - 1) / (NT * T);
    const int64_t total = (int64_t)a.n_head_kv * a.blk_count * tpb;
    const int64_t count = a.cta_count > 0 ? a.cta_count : total - a.cta_begin;
    if (a.cta_begin < 0 || count < 1 || a.cta_begin + count > total || total > INT_MAX) return cudaErrorInvalidValue;
    dim3 grid((unsigned)count);
    k3_sparse_attention<BF16, D, SEG, XCHG, NT><<<grid, threads_of<NT>(), smem, s>>>(mq, mk, mv, mpk, mpv, a);
    return cudaGetLastError();
}

template <bool BF16, int D>
cudaError_t launch_seg(const AttnArgs& a, cudaStream_t s) {
    const bool x = a.n_dest > 0;
    if (a.tiles_per_cta == 1) {
        switch (a.gate.page_size) {
            case 32: return x ? launch_t<BF16, D, 32, true, 1>(a, s) : launch_t<BF16, D, 32, false, 1>(a, s);
            case 64: return x ? launch_t<BF16, D, 64, true, 1>(a, s) : launch_t<BF16, D, 64, false, 1>(a, s);
            case 128: return x ? launch_t<BF16, D, 128, true, 1>(a, s) : launch_t<BF16, D, 128, false, 1>(a, s);
            default: return cudaErrorNotSupported;
        }
    }
    switch (a.gate.page_size) {
        case 32: return x ? launch_t<BF16, D, 32, true, 2>(a, s) : launch_t<BF16, D, 32, false, 2>(a, s);
        case 64: return x ? launch_t<BF16, D, 64, true, 2>(a, s) : launch_t<BF16, D, 64, false, 2>(a, s);
        case 128: return x ? launch_t<BF16, D, 128, true, 2>(a, s) : launch_t<BF16, D, 128, false, 2>(a, s);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace

int attention_smem_bytes(int head_dim) {
    return head_dim == 64 ? Layout<64, 2>::kBytes + 1024 : Layout<128, 2>::kBytes + 1024;
}

int attention_ctas_per_block(int n_head, int n_head_kv, int n_tok, int q_subblock, int tiles_per_cta) {
    const int T = BM / (n_head / n_head_kv);
    const int L = block_len(n_tok, q_subblock);
    return (L + tiles_per_cta * T - 1) / (tiles_per_cta * T);
}

cudaError_t launch_sparse_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    if (a.n_dest < 0 || a.n_dest > kMaxDest) return cudaErrorInvalidValue;
    if (a.n_dest > 0 && a.out_dtype != 1 && a.out_dtype != 2) return cudaErrorNotSupported;
    if (a.tiles_per_cta != 1 && a.tiles_per_cta != 2) return cudaErrorInvalidValue;
    if (BM / (a.n_head / a.n_head_kv) < 1) return cudaErrorNotSupported;
    if (a.dtype != 1 && a.dtype != 2) return cudaErrorNotSupported;
    const bool bf16 = a.dtype == 2;
    if (a.head_dim == 128) return bf16 ? launch_seg<true, 128>(a, s) : launch_seg<false, 128>(a, s);
    if (a.head_dim == 64) return bf16 ? launch_seg<true, 64>(a, s) : launch_seg<false, 64>(a, s);
    return cudaErrorNotSupported;
}

}  // namespace epsp
