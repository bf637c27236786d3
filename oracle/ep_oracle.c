/*
 * ep_oracle.c -- CPU oracle (test infrastructure, never shipped).
 * See ep_oracle.h for the contract and the reference lines each part restates.
 */
#include "ep_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* scalar conversions                                                        */
/* ------------------------------------------------------------------------ */

float epo_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float epo_f16_to_f32(uint16_t h) {
    const int s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    float v;
    if (e == 0) {
        v = ldexpf((float)m, -24);
    } else if (e == 31) {
        v = m ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(m + 1024), e - 25);
    }
    return s ? -v : v;
}

uint16_t epo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    }
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb; /* round to nearest, ties to even */
    return (uint16_t)(u >> 16);
}

uint16_t epo_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t absu = u & 0x7fffffffu;
    if (absu >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (absu > 0x7f800000u ? 0x200u : 0u));
    }
    const int32_t exp = (int32_t)(absu >> 23) - 127;
    uint32_t mant = absu & 0x7fffffu;
    if (exp > 15) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (exp >= -14) {
        /* normal half: 10 mantissa bits, round the low 13 bits */
        uint32_t h = ((uint32_t)(exp + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* carry may reach inf */
        return (uint16_t)(sign | h);
    }
    if (exp < -25) return sign; /* underflows to zero (below half of min subnormal) */
    /* subnormal half: value = m * 2^-24 with m = round(|f| * 2^24); |f| * 2^24 is
     * the 24-bit mantissa shifted right by (-exp - 1) bits. */
    mant |= 0x800000u;
    const int drop = -exp - 1; /* 14..24 */
    uint32_t h = mant >> drop;
    const uint32_t rem = mant & ((1u << drop) - 1u);
    const uint32_t half = 1u << (drop - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

static inline double load_elem(const void* base, int32_t dtype, size_t i) {
    switch (dtype) {
        case EPO_F32: return (double)((const float*)base)[i];
        case EPO_F16: return (double)epo_f16_to_f32(((const uint16_t*)base)[i]);
        default: return (double)epo_bf16_to_f32(((const uint16_t*)base)[i]);
    }
}

/* ------------------------------------------------------------------------ */
/* block geometry: patch :976-993 (graph), :754-792 (set_input), :925-933     */
/* ------------------------------------------------------------------------ */

void epo_plan_block(const epo_params* p, int32_t b0, int32_t b1, int32_t k_budget,
                    epo_block_plan* out) {
    const int64_t P = p->page_size;
    const int64_t n_blk = (int64_t)b1 - b0;
    const int64_t N = b1;
    const int64_t W = p->local_pages > 0 ? (int64_t)p->local_pages * P : n_blk;
    int64_t start_row = N - n_blk - W;
    if (start_row < 0) start_row = 0;
    const int64_t lsp = start_row / P;
    const int64_t n_pages = N / P;
    out->b0 = b0;
    out->b1 = b1;
    out->lsp = (int32_t)lsp;
    out->gated = (k_budget >= 0 && n_pages > 0 && lsp > 0) ? 1 : 0;
    if (!out->gated) {
        out->k_sel = 0;
        out->n_local = (int32_t)N;
        return;
    }
    const int64_t n_local = P + N - lsp * P;
    int64_t k_sel = k_budget;
    if (p->shared) {
        if (k_sel > lsp) k_sel = lsp; /* reference formula, patch :990-992 */
    } else {
        if (k_sel > lsp - 1) k_sel = lsp - 1; /* only pages 1..lsp-1 are selectable */
    }
    if (p->max_gather_rows > 0) {
        int64_t cap = (p->max_gather_rows - n_local) / P;
        if (p->max_gather_rows - n_local < 0) cap = 0;
        if (k_sel > cap) k_sel = cap;
    }
    if (k_sel < 0) k_sel = 0;
    out->k_sel = (int32_t)k_sel;
    out->n_local = (int32_t)n_local;
}

/* ------------------------------------------------------------------------ */
/* chunk plan: src/chunk_scheduler.cpp:9-45                                   */
/* ------------------------------------------------------------------------ */

int32_t epo_chunk_plan(uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                       uint32_t* ranges, int32_t cap) {
    if (!ranges || n_tokens == 0 || n_ubatch == 0) return -2;
    int32_t n = 0;
    if (chunk_size != 0 && chunk_size >= n_tokens) {
        if (cap < 1) return -2;
        ranges[0] = 0;
        ranges[1] = n_tokens;
        return 1;
    }
    uint32_t eff = chunk_size == 0 ? n_ubatch : chunk_size;
    if (eff > n_ubatch) eff = n_ubatch;
    if (eff > n_tokens) eff = n_tokens;
    if (eff == 0) eff = 1;
    for (uint32_t b = 0; b < n_tokens; b += eff) {
        if (n >= cap) return -2;
        const uint32_t e = (n_tokens - b < eff) ? n_tokens : b + eff;
        ranges[2 * n] = b;
        ranges[2 * n + 1] = e;
        ++n;
    }
    return n;
}

int32_t epo_list_blocks(const epo_params* p, uint32_t n_tokens, uint32_t chunk_size,
                        uint32_t n_ubatch, int32_t* blocks, int32_t cap) {
    const int32_t max_ranges = (int32_t)(n_tokens / (n_ubatch ? 1 : 1)) + 1;
    uint32_t* ranges = (uint32_t*)malloc(sizeof(uint32_t) * 2 * (size_t)max_ranges);
    if (!ranges) return -10;
    const int32_t nr = epo_chunk_plan(n_tokens, chunk_size, n_ubatch, ranges, max_ranges);
    if (nr < 0) {
        free(ranges);
        return nr;
    }
    int32_t nb = 0;
    for (int32_t i = 0; i < nr; ++i) {
        const uint32_t c0 = ranges[2 * i], c1 = ranges[2 * i + 1];
        const uint32_t step = p->q_subblock > 0 ? (uint32_t)p->q_subblock : (c1 - c0);
        for (uint32_t b = c0; b < c1; b += step) {
            const uint32_t e = (c1 - b < step) ? c1 : b + step;
            if (blocks) {
                if (nb >= cap) {
                    free(ranges);
                    return -2;
                }
                blocks[2 * nb] = (int32_t)b;
                blocks[2 * nb + 1] = (int32_t)e;
            }
            ++nb;
        }
    }
    free(ranges);
    return nb;
}

int32_t epo_count_blocks(const epo_params* p, uint32_t n_tokens, uint32_t chunk_size,
                         uint32_t n_ubatch) {
    return epo_list_blocks(p, n_tokens, chunk_size, n_ubatch, NULL, 0);
}

/* ------------------------------------------------------------------------ */
/* page sums (fp64, ascending row order)                                      */
/* ------------------------------------------------------------------------ */

void epo_page_sums(const void* k, int32_t dtype, int32_t n_rows, int32_t n_head_kv,
                   int32_t head_dim, int32_t page_size, double* out) {
    /* Contract: rows are summed sequentially in groups of EPO_GROUP_ROWS
     * (starting from 0.0), then the groups of the page are added in ascending
     * order starting from group 0's sum. */
    const int32_t n_pages = n_rows / page_size;
    const int32_t ng = page_size / EPO_GROUP_ROWS;
    for (int32_t h = 0; h < n_head_kv; ++h) {
        for (int32_t pg = 0; pg < n_pages; ++pg) {
            double* dst = out + ((size_t)h * n_pages + pg) * head_dim;
            for (int32_t c = 0; c < head_dim; ++c) {
                double total = 0.0;
                for (int32_t g = 0; g < ng; ++g) {
                    double gs = 0.0;
                    const int32_t r0 = pg * page_size + g * EPO_GROUP_ROWS;
                    for (int32_t r = r0; r < r0 + EPO_GROUP_ROWS; ++r)
                        gs = gs + load_elem(k, dtype, ((size_t)r * n_head_kv + h) * head_dim + c);
                    total = (g == 0) ? gs : total + gs;
                }
                dst[c] = total;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* scoring + top-k: patch :1035-1058                                          */
/* ------------------------------------------------------------------------ */

static double page_score(const epo_params* p, const void* q_last, int32_t dtype,
                         const double* psum, int32_t stride, int32_t h, int32_t page) {
    /* Contract: channels in groups of EPO_GROUP_CH; each group is an fma chain
     * in ascending channel order starting from 0.0; the group partials are
     * added in ascending group order starting from group 0's. */
    const int32_t d = p->head_dim;
    const int32_t G = p->n_head / p->n_head_kv;
    const size_t qoff = (size_t)(h * G) * d;
    const double* s = psum + ((size_t)h * stride + page) * d;
    double total = 0.0;
    for (int32_t g = 0; g < d / EPO_GROUP_CH; ++g) {
        double acc = 0.0;
        for (int32_t c = g * EPO_GROUP_CH; c < (g + 1) * EPO_GROUP_CH; ++c)
            acc = fma(load_elem(q_last, dtype, qoff + c), s[c], acc);
        total = (g == 0) ? acc : total + acc;
    }
    return total;
}

typedef struct {
    double score;
    int32_t page;
} scored_page;

static int cmp_rank(const void* a, const void* b) {
    const scored_page* x = (const scored_page*)a;
    const scored_page* y = (const scored_page*)b;
    if (x->score > y->score) return -1;
    if (x->score < y->score) return 1;
    return (x->page < y->page) ? -1 : (x->page > y->page);
}

static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

/* Candidates 1..lsp-1 scored (per head, or the MAX over heads when head < 0)
 * and sorted by rank (score descending, ties -> lower page).  Caller frees. */
static scored_page* rank_candidates(const epo_params* p, const epo_block_plan* plan, const void* q_last,
                                    int32_t dtype, const double* psum, int32_t n_pages_stride, int32_t head,
                                    double* scores_out) {
    const int32_t n_cand = plan->lsp - 1;
    scored_page* cand = (scored_page*)malloc(sizeof(scored_page) * (size_t)(n_cand > 0 ? n_cand : 1));
    for (int32_t i = 0; i < n_cand; ++i) {
        const int32_t page = i + 1;
        double s;
        if (head >= 0) {
            s = page_score(p, q_last, dtype, psum, n_pages_stride, head, page);
        } else {
            s = -INFINITY;
            for (int32_t h = 0; h < p->n_head_kv; ++h) {
                const double v = page_score(p, q_last, dtype, psum, n_pages_stride, h, page);
                if (v > s) s = v;
            }
        }
        cand[i].score = s;
        cand[i].page = page;
        if (scores_out) scores_out[page] = s;
    }
    if (scores_out) scores_out[0] = -INFINITY;
    qsort(cand, (size_t)(n_cand > 0 ? n_cand : 0), sizeof(scored_page), cmp_rank);
    return cand;
}

void epo_route_block(const epo_params* p, const epo_block_plan* plan, const void* q_last, int32_t dtype,
                     const double* psum, int32_t n_pages_stride, const int32_t* k_in, int32_t* k_out,
                     double* spread_out) {
    const int32_t Hkv = p->n_head_kv;
    const int32_t n_cand = plan->lsp - 1;
    for (int32_t h = 0; h < Hkv; ++h) k_out[h] = k_in[h];
    if (!plan->gated || n_cand < 1 || p->route_mode == 0) return;
    int32_t n_ret = 0, freed = 0;
    int32_t* streaming = (int32_t*)calloc((size_t)Hkv, sizeof(int32_t));
    for (int32_t h = 0; h < Hkv; ++h) {
        double mx = -INFINITY, sum = 0.0;
        for (int32_t page = 1; page <= n_cand; ++page) {
            const double u = page_score(p, q_last, dtype, psum, n_pages_stride, h, page) / (double)p->page_size;
            if (u > mx) mx = u;
            sum = sum + u;
        }
        const double mean = sum / (double)n_cand;
        const double spread = (mx - mean) / (fabs(mean) + EPO_ROUTE_EPS);
        if (spread_out) spread_out[h] = spread;
        if (spread < p->route_threshold) {
            streaming[h] = 1;
            freed += k_in[h];
            k_out[h] = 0;
        } else {
            ++n_ret;
        }
    }
    if (p->route_mode == 2 && n_ret > 0 && freed > 0) {
        int32_t rank = 0;
        for (int32_t h = 0; h < Hkv; ++h) {
            if (streaming[h]) continue;
            int32_t k = k_in[h] + freed / n_ret + (rank < freed % n_ret ? 1 : 0);
            if (k > n_cand) k = n_cand;
            k_out[h] = k;
            ++rank;
        }
    }
    free(streaming);
}

int32_t epo_pool_block(const epo_params* p, const epo_block_plan* plan,
                       const void* q_last, int32_t dtype, const double* psum,
                       int32_t n_pages_stride, int32_t head, int32_t* out_pages) {
    if (!plan->gated || p->pool_pages <= 0) return 0;
    const int32_t n_cand = plan->lsp - 1;
    const int32_t take = plan->k_sel < n_cand ? plan->k_sel : n_cand;
    int32_t m = n_cand - take;
    if (m > p->pool_pages) m = p->pool_pages;
    if (m <= 0) return 0;
    scored_page* cand = rank_candidates(p, plan, q_last, dtype, psum, n_pages_stride, head, NULL);
    for (int32_t i = 0; i < m; ++i) out_pages[i] = cand[take + i].page;
    qsort(out_pages, (size_t)m, sizeof(int32_t), cmp_i32);
    free(cand);
    return m;
}

double epo_pool_elem(double page_sum, int32_t page_size, int32_t dtype) {
    const float f = (float)(page_sum / (double)page_size);
    if (dtype == EPO_F32) return (double)f;
    if (dtype == EPO_F16) return (double)epo_f16_to_f32(epo_f32_to_f16(f));
    return (double)epo_bf16_to_f32(epo_f32_to_bf16(f));
}

int32_t epo_select_block(const epo_params* p, const epo_block_plan* plan,
                         const void* q_last, int32_t dtype, const double* psum,
                         int32_t n_pages_stride, int32_t head, int32_t* out_pages,
                         double* scores_out) {
    if (!plan->gated) return 0;
    const int32_t lsp = plan->lsp;
    const int32_t n_cand = lsp - 1;
    scored_page* cand = rank_candidates(p, plan, q_last, dtype, psum, n_pages_stride, head, scores_out);
    int32_t n = 0;
    for (int32_t i = 0; i < n_cand && n < plan->k_sel; ++i) out_pages[n++] = cand[i].page;
    /* reference off-by-one: the remaining picks are -inf pages, lowest id first
     * ({0} then lsp, lsp+1, ...). */
    int32_t extra = 0;
    while (n < plan->k_sel) {
        out_pages[n++] = (extra == 0) ? 0 : lsp + extra - 1;
        ++extra;
    }
    qsort(out_pages, (size_t)n, sizeof(int32_t), cmp_i32);
    free(cand);
    return n;
}

/* ------------------------------------------------------------------------ */
/* parallel-for                                                               */
/* ------------------------------------------------------------------------ */

typedef void (*pf_body)(void* ctx, int64_t i);

typedef struct {
    pf_body body;
    void* ctx;
    int64_t n;
    int64_t next;
    pthread_mutex_t mu;
} pf_state;

static void* pf_worker(void* arg) {
    pf_state* st = (pf_state*)arg;
    for (;;) {
        pthread_mutex_lock(&st->mu);
        const int64_t i = st->next++;
        pthread_mutex_unlock(&st->mu);
        if (i >= st->n) break;
        st->body(st->ctx, i);
    }
    return NULL;
}

static void parallel_for(int64_t n, int32_t n_threads, pf_body body, void* ctx) {
    if (n_threads <= 1 || n <= 1) {
        for (int64_t i = 0; i < n; ++i) body(ctx, i);
        return;
    }
    pf_state st;
    st.body = body;
    st.ctx = ctx;
    st.n = n;
    st.next = 0;
    pthread_mutex_init(&st.mu, NULL);
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int32_t t = 0; t < n_threads; ++t) pthread_create(&th[t], NULL, pf_worker, &st);
    for (int32_t t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    free(th);
    pthread_mutex_destroy(&st.mu);
}

/* ------------------------------------------------------------------------ */
/* one layer: chunk loop + selection + attention over the kept union          */
/* (patch :1002-1016 local gather, :1060-1078 union, :1092 attention)         */
/* ------------------------------------------------------------------------ */

typedef struct {
    const epo_params* p;
    const int32_t* k_budget;
    const void* q;
    const void* k;
    const void* v;
    int32_t dtype;
    const int32_t* blocks; /* [nb][2] */
    int32_t nb;
    epo_block_plan* plans; /* [nb][Hkv] */
    int32_t* sel;          /* [nb][Hkv][sel_cap] */
    int32_t* cnt;          /* [nb][Hkv] */
    int32_t sel_cap;
    const double* psum;
    const double* vsum;    /* V page sums (pooled rows), or NULL */
    int32_t* pool;         /* [nb][Hkv][pool_cap] */
    int32_t* pool_cnt;     /* [nb][Hkv] */
    int32_t pool_cap;
    int32_t n_pages;
    double* out;
    const int32_t* rows;
    int32_t* row_block;    /* block index of each query row */
    double kq_scale;
} layer_job;

static void select_body(void* vctx, int64_t i) {
    layer_job* J = (layer_job*)vctx;
    const epo_params* p = J->p;
    const int32_t Hkv = p->n_head_kv;
    const int32_t b = (int32_t)(i / Hkv), h = (int32_t)(i % Hkv);
    const epo_block_plan* plan = &J->plans[(size_t)b * Hkv + h];
    const int32_t b1 = J->blocks[2 * b + 1];
    const size_t qrow = (size_t)(b1 - 1) * p->n_head * p->head_dim;
    const size_t esz = J->dtype == EPO_F32 ? 4 : 2;
    const void* q_last = (const char*)J->q + qrow * esz;
    int32_t* dst = J->sel + ((size_t)b * Hkv + h) * J->sel_cap;
    int32_t* pdst = J->pool + ((size_t)b * Hkv + h) * J->pool_cap;
    if (p->shared) {
        if (h != 0) return; /* head 0 computes the shared lists; copied below */
        const int32_t n = epo_select_block(p, plan, q_last, J->dtype, J->psum, J->n_pages, -1, dst, NULL);
        const int32_t m = epo_pool_block(p, plan, q_last, J->dtype, J->psum, J->n_pages, -1, pdst);
        for (int32_t hh = 0; hh < Hkv; ++hh) {
            J->cnt[(size_t)b * Hkv + hh] = n;
            J->pool_cnt[(size_t)b * Hkv + hh] = m;
            if (hh) {
                memcpy(J->sel + ((size_t)b * Hkv + hh) * J->sel_cap, dst, sizeof(int32_t) * (size_t)n);
                memcpy(J->pool + ((size_t)b * Hkv + hh) * J->pool_cap, pdst, sizeof(int32_t) * (size_t)m);
            }
        }
    } else {
        J->cnt[(size_t)b * Hkv + h] =
            epo_select_block(p, plan, q_last, J->dtype, J->psum, J->n_pages, h, dst, NULL);
        J->pool_cnt[(size_t)b * Hkv + h] = epo_pool_block(p, plan, q_last, J->dtype, J->psum, J->n_pages, h, pdst);
    }
}

static void attend_body(void* vctx, int64_t i) {
    layer_job* J = (layer_job*)vctx;
    const epo_params* p = J->p;
    const int32_t Hq = p->n_head, Hkv = p->n_head_kv, d = p->head_dim, P = p->page_size;
    const int32_t G = Hq / Hkv;
    const int32_t t = J->rows ? J->rows[i / Hq] : (int32_t)(i / Hq);
    const int32_t hq = (int32_t)(i % Hq);
    const int32_t h = hq / G;
    const int32_t b = J->row_block[t];
    const epo_block_plan* plan = &J->plans[(size_t)b * Hkv + h];
    const int32_t* sel = J->sel + ((size_t)b * Hkv + h) * J->sel_cap;
    const int32_t nsel = J->cnt[(size_t)b * Hkv + h];

    /* kept multiset of rows (sink, selected pages, local window; causal) */
    int32_t n_keep = 0;
    int32_t* keep;
    if (!plan->gated) {
        keep = (int32_t*)malloc(sizeof(int32_t) * (size_t)(t + 1));
        for (int32_t r = 0; r <= t; ++r) keep[n_keep++] = r;
    } else {
        const int32_t lo = plan->lsp * P;
        keep = (int32_t*)malloc(sizeof(int32_t) * (size_t)(P + nsel * P + (t - lo + 1)));
        for (int32_t r = 0; r < P; ++r) keep[n_keep++] = r;
        for (int32_t s = 0; s < nsel; ++s)
            for (int32_t r = sel[s] * P; r < sel[s] * P + P; ++r)
                if (r <= t) keep[n_keep++] = r;
        for (int32_t r = lo; r <= t; ++r) keep[n_keep++] = r;
    }
    /* pooled rows of this block and head (patch :1595-1715 semantics): one
     * row per pooled page, the page means, visible to every query row */
    const int32_t n_pool = (plan->gated && J->vsum) ? J->pool_cnt[(size_t)b * Hkv + h] : 0;
    const int32_t* pool = J->pool + ((size_t)b * Hkv + h) * J->pool_cap;
    const size_t qoff = ((size_t)t * Hq + hq) * d;
    double* qv = (double*)malloc(sizeof(double) * (size_t)d);
    for (int32_t c = 0; c < d; ++c) qv[c] = load_elem(J->q, J->dtype, qoff + c);
    double* sc = (double*)malloc(sizeof(double) * (size_t)(n_keep + n_pool));
    double m = -INFINITY;
    for (int32_t j = 0; j < n_keep; ++j) {
        const size_t koff = ((size_t)keep[j] * Hkv + h) * d;
        double acc = 0.0;
        for (int32_t c = 0; c < d; ++c) acc += qv[c] * load_elem(J->k, J->dtype, koff + c);
        sc[j] = acc * J->kq_scale;
        if (sc[j] > m) m = sc[j];
    }
    for (int32_t j = 0; j < n_pool; ++j) {
        const double* ks = J->psum + ((size_t)h * J->n_pages + pool[j]) * d;
        double acc = 0.0;
        for (int32_t c = 0; c < d; ++c) acc += qv[c] * epo_pool_elem(ks[c], P, J->dtype);
        sc[n_keep + j] = acc * J->kq_scale;
        if (sc[n_keep + j] > m) m = sc[n_keep + j];
    }
    double l = 0.0;
    double* o = J->out + qoff;
    for (int32_t c = 0; c < d; ++c) o[c] = 0.0;
    for (int32_t j = 0; j < n_keep; ++j) {
        const double e = exp(sc[j] - m);
        l += e;
        const size_t voff = ((size_t)keep[j] * Hkv + h) * d;
        for (int32_t c = 0; c < d; ++c) o[c] += e * load_elem(J->v, J->dtype, voff + c);
    }
    for (int32_t j = 0; j < n_pool; ++j) {
        const double e = exp(sc[n_keep + j] - m);
        l += e;
        const double* vs = J->vsum + ((size_t)h * J->n_pages + pool[j]) * d;
        for (int32_t c = 0; c < d; ++c) o[c] += e * epo_pool_elem(vs[c], P, J->dtype);
    }
    for (int32_t c = 0; c < d; ++c) o[c] /= l;
    free(sc);
    free(qv);
    free(keep);
}

int32_t epo_prefill_layer(const epo_params* p, const int32_t* k_budget,
                          const void* q, const void* k, const void* v, int32_t dtype,
                          uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                          double* out, const int32_t* rows, int32_t n_rows,
                          int32_t* sel_out, int32_t* sel_count, int32_t sel_cap,
                          int32_t n_threads) {
    return epo_prefill_layer_ex(p, k_budget, q, k, v, dtype, n_tokens, chunk_size, n_ubatch, out, rows, n_rows,
                                sel_out, sel_count, sel_cap, NULL, NULL, 0, n_threads);
}

int32_t epo_prefill_layer_ex(const epo_params* p, const int32_t* k_budget,
                             const void* q, const void* k, const void* v, int32_t dtype,
                             uint32_t n_tokens, uint32_t chunk_size, uint32_t n_ubatch,
                             double* out, const int32_t* rows, int32_t n_rows,
                             int32_t* sel_out, int32_t* sel_count, int32_t sel_cap,
                             int32_t* pool_out, int32_t* pool_count, int32_t pool_cap,
                             int32_t n_threads) {
    if (!p || p->n_head_kv <= 0 || p->n_head % p->n_head_kv || p->page_size <= 0) return -2;
    const int32_t Hkv = p->n_head_kv;
    const int32_t nb = epo_count_blocks(p, n_tokens, chunk_size, n_ubatch);
    if (nb <= 0) return nb < 0 ? nb : -2;
    int32_t* blocks = (int32_t*)malloc(sizeof(int32_t) * 2 * (size_t)nb);
    epo_list_blocks(p, n_tokens, chunk_size, n_ubatch, blocks, nb);

    layer_job J;
    memset(&J, 0, sizeof(J));
    J.p = p;
    J.k_budget = k_budget;
    J.q = q;
    J.k = k;
    J.v = v;
    J.dtype = dtype;
    J.blocks = blocks;
    J.nb = nb;
    J.plans = (epo_block_plan*)malloc(sizeof(epo_block_plan) * (size_t)nb * Hkv);
    int32_t max_sel = 1;
    for (int32_t b = 0; b < nb; ++b) {
        for (int32_t h = 0; h < Hkv; ++h) {
            const int32_t kb = k_budget ? k_budget[h] : p->sel_pages;
            epo_plan_block(p, blocks[2 * b], blocks[2 * b + 1], kb, &J.plans[(size_t)b * Hkv + h]);
            if (J.plans[(size_t)b * Hkv + h].k_sel > max_sel) max_sel = J.plans[(size_t)b * Hkv + h].k_sel;
            /* routing mode 2 may raise a head's budget up to the candidate count */
            if (p->route_mode == 2 && !p->shared && J.plans[(size_t)b * Hkv + h].lsp - 1 > max_sel)
                max_sel = J.plans[(size_t)b * Hkv + h].lsp - 1;
        }
    }
    if (sel_out && sel_cap < max_sel) {
        free(J.plans);
        free(blocks);
        return -2;
    }
    J.sel_cap = sel_out ? sel_cap : max_sel;
    J.sel = sel_out ? sel_out : (int32_t*)malloc(sizeof(int32_t) * (size_t)nb * Hkv * J.sel_cap);
    J.cnt = sel_count ? sel_count : (int32_t*)malloc(sizeof(int32_t) * (size_t)nb * Hkv);
    J.n_pages = (int32_t)(n_tokens / (uint32_t)p->page_size);
    double* psum = (double*)malloc(sizeof(double) * (size_t)(J.n_pages > 0 ? J.n_pages : 1) * Hkv * p->head_dim);
    epo_page_sums(k, dtype, (int32_t)n_tokens, Hkv, p->head_dim, p->page_size, psum);
    J.psum = psum;
    double* vsum = NULL;
    if (p->pool_pages > 0) {
        vsum = (double*)malloc(sizeof(double) * (size_t)(J.n_pages > 0 ? J.n_pages : 1) * Hkv * p->head_dim);
        epo_page_sums(v, dtype, (int32_t)n_tokens, Hkv, p->head_dim, p->page_size, vsum);
    }
    J.vsum = vsum;
    /* a block pools at most its lsp - 1 candidates */
    int32_t max_pool = 1;
    if (p->pool_pages > 0)
        for (int32_t b = 0; b < nb; ++b)
            for (int32_t h = 0; h < Hkv; ++h) {
                const int32_t c = J.plans[(size_t)b * Hkv + h].lsp - 1;
                if (c > max_pool) max_pool = c;
            }
    if (pool_out && pool_cap < (p->pool_pages < max_pool ? p->pool_pages : max_pool) && p->pool_pages > 0) {
        free(vsum);
        free(psum);
        if (!sel_out) free(J.sel);
        if (!sel_count) free(J.cnt);
        free(J.plans);
        free(blocks);
        return -2;
    }
    J.pool_cap = pool_out ? (pool_cap > 0 ? pool_cap : 1) : max_pool;
    J.pool = pool_out ? pool_out : (int32_t*)malloc(sizeof(int32_t) * (size_t)nb * Hkv * J.pool_cap);
    J.pool_cnt = pool_count ? pool_count : (int32_t*)calloc((size_t)nb * Hkv, sizeof(int32_t));
    if (pool_count) memset(pool_count, 0, sizeof(int32_t) * (size_t)nb * Hkv);
    J.kq_scale = p->kq_scale > 0 ? p->kq_scale : 1.0 / sqrt((double)p->head_dim);

    if (p->route_mode != 0 && !p->shared) {
        /* routing: effective per-head budgets of every block, before the selection */
        int32_t* kin = (int32_t*)malloc(sizeof(int32_t) * (size_t)Hkv);
        int32_t* kout = (int32_t*)malloc(sizeof(int32_t) * (size_t)Hkv);
        for (int32_t b = 0; b < nb; ++b) {
            const size_t esz = dtype == EPO_F32 ? 4 : 2;
            const void* q_last = (const char*)q + (size_t)(blocks[2 * b + 1] - 1) * p->n_head * p->head_dim * esz;
            for (int32_t h = 0; h < Hkv; ++h) kin[h] = J.plans[(size_t)b * Hkv + h].k_sel;
            epo_route_block(p, &J.plans[(size_t)b * Hkv], q_last, dtype, psum, J.n_pages, kin, kout, NULL);
            for (int32_t h = 0; h < Hkv; ++h) {
                epo_block_plan* pl = &J.plans[(size_t)b * Hkv + h];
                if (pl->gated) pl->k_sel = kout[h];
            }
        }
        free(kin);
        free(kout);
    }
    parallel_for((int64_t)nb * Hkv, n_threads, select_body, &J);

    if (out) {
        J.out = out;
        J.rows = rows;
        J.row_block = (int32_t*)malloc(sizeof(int32_t) * (size_t)n_tokens);
        for (int32_t b = 0; b < nb; ++b)
            for (int32_t t = blocks[2 * b]; t < blocks[2 * b + 1]; ++t) J.row_block[t] = b;
        const int64_t nr = rows ? n_rows : (int64_t)n_tokens;
        parallel_for(nr * p->n_head, n_threads, attend_body, &J);
        free(J.row_block);
    }

    free(psum);
    free(vsum);
    if (!pool_out) free(J.pool);
    if (!pool_count) free(J.pool_cnt);
    if (!sel_out) free(J.sel);
    if (!sel_count) free(J.cnt);
    free(J.plans);
    free(blocks);
    return nb;
}

/* ------------------------------------------------------------------------ */
/* FFN skip compaction / scatter (ffn patch :146-149, sparse_prefill :214-232) */
/* ------------------------------------------------------------------------ */

int32_t epo_ffn_compact(const void* x, int32_t elem_bytes, const uint8_t* keep,
                        int32_t n_rows, int32_t hidden, int32_t layer_skipped,
                        void* x_kept, int32_t* row_ids) {
    if (layer_skipped) return 0;
    int32_t n = 0;
    const size_t row_bytes = (size_t)hidden * (size_t)elem_bytes;
    for (int32_t r = 0; r < n_rows; ++r) {
        if (!keep[r]) continue;
        memcpy((char*)x_kept + (size_t)n * row_bytes, (const char*)x + (size_t)r * row_bytes, row_bytes);
        row_ids[n++] = r;
    }
    return n;
}

void epo_ffn_scatter(const void* ffn_out, void* residual, int32_t dtype,
                     const int32_t* row_ids, int32_t n_keep, int32_t hidden) {
    for (int32_t i = 0; i < n_keep; ++i) {
        const size_t src = (size_t)i * hidden;
        const size_t dst = (size_t)row_ids[i] * hidden;
        for (int32_t c = 0; c < hidden; ++c) {
            if (dtype == EPO_F32) {
                float* r = (float*)residual + dst + c;
                *r = *r + ((const float*)ffn_out)[src + c];
            } else if (dtype == EPO_F16) {
                uint16_t* r = (uint16_t*)residual + dst + c;
                const float s = epo_f16_to_f32(*r) + epo_f16_to_f32(((const uint16_t*)ffn_out)[src + c]);
                *r = epo_f32_to_f16(s);
            } else {
                uint16_t* r = (uint16_t*)residual + dst + c;
                const float s = epo_bf16_to_f32(*r) + epo_bf16_to_f32(((const uint16_t*)ffn_out)[src + c]);
                *r = epo_f32_to_bf16(s);
            }
        }
    }
}
