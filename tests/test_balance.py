"""Host-side splitting of a layer's attention grid (no GPU): the
ep_sp_balance_ctas cuts, the ep_sp_cta_work accounting and the CTA-grid
geometry, on the c4 shapes (65,536 tokens, 32 q / 8 kv heads, adaptive
per-head budgets)."""
from __future__ import annotations

import ctypes

import pytest

import epsp
import workloads as W

C4 = W.CONFIGS["c4"]


def ctx_for(w, k_matrix=None):
    c = epsp.Context(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim, dtype=w.dtype,
                     out_dtype=w.dtype, max_ctx=w.n_tokens, page_size=w.page_size, device=0)
    c.check(c.set_ext(1, w.n_ubatch, 0))
    if k_matrix is not None:
        c.check(c.set_k_matrix([x for row in k_matrix for x in row]))
    c.check(c.set_qg_bound(1, min(w.top_k, 128), w.local_pages, 0))
    c.set_prefill_mode(True)
    return c


def test_grid_geometry():
    c = ctx_for(C4, C4.k_matrix())
    # 16 blocks of 4096 rows, 32-token query tiles (G = 4), two per CTA
    assert c.attention_grid(65536) == 16 * 4096 // 64
    assert c.attention_grid(1000) == 1 * ((1000 + 63) // 64)


def test_cta_work_sums_to_layer_work():
    c = ctx_for(C4, C4.k_matrix())
    N = C4.n_tokens
    total = C4.n_head_kv * c.attention_grid(N)
    arr = (ctypes.c_double * 6)()
    for layer in (0, 9, 31):
        assert epsp.lib.ep_sp_layer_work(c.h, layer, N, N, arr) == 0
        whole = c.cta_work(layer, N, N, 0, total)
        assert whole[0] == arr[3] and whole[2] == arr[5]
        parts = [c.cta_work(layer, N, N, a, b) for a, b in ((0, 1000), (1000, 4321), (4321, total))]
        assert sum(p[0] for p in parts) == pytest.approx(whole[0], rel=1e-12)


@pytest.mark.parametrize("n_parts", [2, 4, 8])
def test_equal_budgets_give_the_head_parallel_split(n_parts):
    w = W.scaled(C4, adaptive_k=(), pyramid_every=0, top_k=64)
    c = ctx_for(w)
    N = w.n_tokens
    per_head = c.attention_grid(N)
    cuts = c.balance_ctas(0, N, N, n_parts)
    assert cuts == [r * per_head * w.n_head_kv // n_parts for r in range(n_parts + 1)]


def cta_costs(w, k_matrix, layer, n_parts):
    """The balancer's cost of every CTA of a whole-prompt c4-shaped call in
    head-major order: KV tiles walked (sink + selected pages + local window up
    to the CTA's last token, one page per tile) plus the fixed share per CTA
    (0.4 tiles, and the exchange epilogue to n_parts ranks)."""
    P, L, T = w.page_size, w.n_ubatch, 128 // (w.n_head // w.n_head_kv)
    W_ = w.local_pages * P
    fixed = 0.4 + (0.55 + 1.4 * (n_parts - 1) if n_parts > 1 else 0.0)
    out = []
    for h in range(w.n_head_kv):
        for b in range(w.n_tokens // L):
            b0, b1 = b * L, (b + 1) * L
            lsp = max(0, b0 - W_) // P
            gated = lsp > 0
            k_sel = min(k_matrix[layer][h], lsp - 1) if gated else 0
            L0 = lsp * P if gated else 0
            for c in range(L // (2 * T)):
                t_end = min(b0 + (c + 1) * 2 * T, b1)
                n_loc = (t_end - L0 + P - 1) // P
                out.append((1 + k_sel + n_loc if gated else n_loc) + fixed)
    return out


@pytest.mark.parametrize("n_parts", [2, 3, 8])
def test_uneven_budgets_balanced(n_parts):
    """Every part's estimated cost is within 2 % of the mean; the algorithmic
    flops follow within 3 % at 2-3 parts and 12 % at 8 (where the exchange
    epilogue makes many cheap CTAs cost more than their flops)."""
    km = C4.k_matrix()
    c = ctx_for(C4, km)
    N = C4.n_tokens
    per_head = c.attention_grid(N)
    total = C4.n_head_kv * per_head
    for layer in range(C4.n_layer):
        cuts = c.balance_ctas(layer, N, N, n_parts)
        assert cuts[0] == 0 and cuts[-1] == total and cuts == sorted(cuts)
        cost = cta_costs(C4, km, layer, n_parts)
        assert len(cost) == total
        parts = [sum(cost[a:b]) for a, b in zip(cuts[:-1], cuts[1:])]
        mean = sum(parts) / n_parts
        assert max(parts) <= 1.02 * mean and min(parts) >= 0.98 * mean, (layer, [p / mean for p in parts])
        flops = [c.cta_work(layer, N, N, a, b)[0] for a, b in zip(cuts[:-1], cuts[1:])]
        fmean = sum(flops) / n_parts
        assert max(flops) <= (1.03 if n_parts < 8 else 1.12) * fmean, (layer, [f / fmean for f in flops])
        # a range reaches into at most three KV heads at 8 parts of 8 heads
        if n_parts == 8:
            for a, b in zip(cuts[:-1], cuts[1:]):
                assert (b - 1) // per_head - a // per_head + 1 <= 3


def test_balance_argument_checks():
    c = ctx_for(C4, C4.k_matrix())
    cuts = (ctypes.c_int32 * 3)()
    assert epsp.lib.ep_sp_balance_ctas(c.h, 0, 100, 200, 2, cuts) == epsp.INVALID_ARGUMENT  # kv_len < n_tok
    assert epsp.lib.ep_sp_balance_ctas(c.h, 32, 100, 100, 2, cuts) == epsp.INVALID_ARGUMENT  # layer
    assert epsp.lib.ep_sp_balance_ctas(c.h, 0, 100, 100, 0, cuts) == epsp.INVALID_ARGUMENT   # parts
    out = (ctypes.c_double * 3)()
    assert epsp.lib.ep_sp_cta_work(c.h, 0, 100, 100, 0, 10 ** 6, out) == epsp.INVALID_ARGUMENT


def test_one_tile_per_cta_grid_and_work():
    """ep_sp_set_attn_tiles(1): twice the CTAs, the same total work, cuts still
    covering the grid; invalid values are rejected and leave the setting."""
    c = ctx_for(C4, C4.k_matrix())
    N = C4.n_tokens
    assert c.attn_tiles() == 2
    per2 = c.attention_grid(N)
    assert c.set_attn_tiles(3) == epsp.INVALID_ARGUMENT and c.attn_tiles() == 2
    c.check(c.set_attn_tiles(1))
    per1 = c.attention_grid(N)
    assert per1 == 2 * per2
    total = C4.n_head_kv * per1
    arr = (ctypes.c_double * 6)()
    for layer in (0, 17):
        assert epsp.lib.ep_sp_layer_work(c.h, layer, N, N, arr) == 0
        assert c.cta_work(layer, N, N, 0, total)[0] == arr[3]
        cuts = c.balance_ctas(layer, N, N, 8)
        assert cuts[0] == 0 and cuts[-1] == total and cuts == sorted(cuts)
        flops = [c.cta_work(layer, N, N, a, b)[0] for a, b in zip(cuts[:-1], cuts[1:])]
        assert max(flops) <= 1.12 * sum(flops) / 8
    c.check(c.set_attn_tiles(2))
    assert c.attention_grid(N) == per2
