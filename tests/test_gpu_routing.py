"""Per-KV-head routing by the live page-score spread (ep_sp_set_head_routing)
against the oracle.

Streaming heads (spread below the threshold) select no page; mode 2 re-splits
their pages over the block's retrieval heads.  The spread arithmetic is the
same fp64 sequence on both sides (scores bit-exact by the selection contract,
then max, an ascending sum, one division), so the routed counts and page lists
are compared bit for bit; attention within 2e-3 max-abs / 1e-3 mean-abs.
"""
import numpy as np
import pytest
import torch

import epsp
import oracle
import workloads as W
from gpu_util import assert_selection_equal, attn_errors, make_ctx, oracle_params, run_gpu, run_oracle, to_np

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3

# needle pages make some heads' score spread high and others' low
W_ROUTE = W.Workload("rg", 2048, 1, 16, 4, 64, W.BF16, 512, 32, 6, 64, per_kv_head=1, max_gather_rows=0,
                     seed=9, needle_frac=0.03)


def _median_spread(w, q, k):
    p = oracle_params(w, 0, w.top_k, 0)
    vals = []
    for b0, b1 in oracle.list_blocks(p, w.n_tokens, 0, w.n_ubatch):
        plan = oracle.plan_block(p, b0, b1, w.top_k)
        if not plan.gated or plan.lsp < 2:
            continue
        _, sp = oracle.route_block(oracle_params(w, 0, w.top_k, 0, route_mode=1), plan, to_np(q[b1 - 1]), w.dtype,
                                   oracle.page_sums(to_np(k[:b1]), w.dtype, w.page_size),
                                   [plan.k_sel] * w.n_head_kv)
        vals.extend(sp.tolist())
    return float(np.median(vals))


@pytest.mark.parametrize("mode,pool", [(1, 0), (2, 0), (2, 3)])
def test_routing_matches_oracle(mode, pool):
    w = W_ROUTE
    q, k, v = W.gen_layer(w, 0)
    thr = _median_spread(w, q, k)
    res = run_oracle(w, q, k, v, shared=0, route_mode=mode, route_threshold=thr, pool_pages=pool, return_pool=True)
    out_o, sel_o, cnt_o, _, pool_o, pcnt_o = res
    base = run_oracle(w, q, k, v, shared=0, attention=False)
    assert (cnt_o == 0).sum() > (base[2] == 0).sum(), "some heads must stream"
    if mode == 2:
        assert cnt_o.max() > base[2].max(), "mode 2 must raise some retrieval head's budget"
    ctx = make_ctx(w, shared=0)
    ctx.check(ctx.set_qg_bound(1, w.top_k, w.local_pages, pool))
    ctx.check(ctx.set_head_routing(mode, thr))
    assert ctx.head_routing() == (mode, thr)
    pooled = []
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v, pooled=pooled)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    if pool:
        pc = torch.cat([c for _, c in pooled]).cpu().numpy()
        pp = torch.cat([p for p, _ in pooled]).cpu().numpy()
        assert np.array_equal(pc, pcnt_o)
        for b in range(pc.shape[0]):
            for h in range(pc.shape[1]):
                assert np.array_equal(pp[b, h, :pc[b, h]], pool_o[b, h, :pc[b, h]]), (b, h)
    mx, mean = attn_errors(out_g, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_routing_argument_rules():
    w = W_ROUTE
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    N = w.n_tokens
    ctx = make_ctx(w, shared=0)
    assert ctx.set_head_routing(3, 1.0) == epsp.INVALID_ARGUMENT
    assert ctx.set_head_routing(1, float("nan")) == epsp.INVALID_ARGUMENT
    ctx.check(ctx.set_head_routing(2, 1.0))
    # mode 2 re-splits a block over all its heads: a head range is refused
    assert ctx.select_heads(0, q, k, v, N, N, 0, 2) == epsp.UNSUPPORTED
    ctx.check(ctx.set_head_routing(1, 1.0))
    ctx.check(ctx.select_heads(0, q, k, v, N, N, 0, 2))
    # the shared (reference) selection has no per-head lists to route
    shared = make_ctx(W.scaled(w, per_kv_head=0, max_gather_rows=4096), shared=1)
    shared.check(shared.set_head_routing(1, 1.0))
    out = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    assert shared.attend_layer(0, q[N - 512:], k, v, N, 512, out[N - 512:]) == epsp.UNSUPPORTED
    torch.cuda.synchronize()
