"""The pooled ("compressed") rows of qg_pool_pages against the oracle.

The reference reserves pool_pages (patch :578) and gives pooled rows their
meaning in its AR004 branch (patch :1595-1715): a page that is not gathered
adds one KV row, the mean of its K rows and of its V rows, causally gated by
the page's last position.  Armed here, each gating block (per KV head, or
shared) pools the pool_pages candidates ranked right after its selection.
Bars: the pooled page lists and counts bit-exact, attention within the usual
2e-3 max-abs / 1e-3 mean-abs of the fp64 oracle, CTA-range splits bit-equal
to the whole call.
"""
import numpy as np
import pytest
import torch

import epsp
import workloads as W
from gpu_util import assert_selection_equal, attn_errors, make_ctx, run_gpu, run_oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3

CASES = {
    # per-KV-head lists, page 128, d 128, bf16, ubatch 512 (gating block = ubatch)
    "per_head_p128_bf16": (W.Workload("pa", 2048, 1, 32, 8, 128, W.BF16, 512, 128, 2, 256, max_gather_rows=0),
                           0, 4, 0),
    # the reference's mode: page 32, one shared list (MAX over heads), 4096 guard, f16, d 64
    "shared_p32_f16": (W.Workload("pb", 2048, 1, 8, 2, 64, W.F16, 512, 32, 3, 64, per_kv_head=0,
                                  max_gather_rows=4096), 1, 6, 0),
    # sub-blocks of 128, page 64, GQA 7
    "sub128_p64_gqa7": (W.Workload("pc", 2048, 1, 28, 4, 128, W.BF16, 1024, 64, 2, 128, q_subblock=128,
                                   max_gather_rows=0), 0, 3, 0),
    # selection budget 0 in the shared mode: pooled rows only
    "shared_sel0_pool": (W.Workload("pd", 1024, 1, 8, 2, 64, W.BF16, 256, 32, 0, 64, per_kv_head=0,
                                    max_gather_rows=4096), 1, 5, 0),
    # f32 Q/K/V attended in fp32 (mode 0) and on f16 tensor cores (mode 1)
    "f32_mode0": (W.scaled(W.CONFIGS["c1"], n_tokens=2048, n_ubatch=2048, top_k=4), 0, 4, 0),
    "f32_mode1": (W.scaled(W.CONFIGS["c1"], n_tokens=2048, n_ubatch=2048, top_k=4), 0, 4, 1),
}


@pytest.mark.parametrize("name", list(CASES))
def test_pooled_rows_match_oracle(name):
    w, shared, pool, f32_mode = CASES[name]
    q, k, v = W.gen_layer(w, 0)
    out_o, sel_o, cnt_o, _, pool_o, pcnt_o = run_oracle(w, q, k, v, shared=shared, pool_pages=pool,
                                                        return_pool=True)
    assert pcnt_o.sum() > 0, "the case must pool pages"
    ctx = make_ctx(w, shared=shared)
    ctx.check(ctx.set_qg_bound(1, w.top_k, w.local_pages, pool))
    if w.dtype == W.F32:
        ctx.check(ctx.set_f32_attention(f32_mode))
    pooled = []
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v, pooled=pooled)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    pp = torch.cat([p for p, _ in pooled]).cpu().numpy()
    pc = torch.cat([c for _, c in pooled]).cpu().numpy()
    assert np.array_equal(pc, pcnt_o), (pc, pcnt_o)
    for b in range(pc.shape[0]):
        for h in range(pc.shape[1]):
            n = pc[b, h]
            assert np.array_equal(pp[b, h, :n], pool_o[b, h, :n]), (b, h, pp[b, h, :n], pool_o[b, h, :n])
            assert not set(pp[b, h, :n]) & set(sel_g[b, h, :cnt_g[b, h]])
    mx, mean = attn_errors(out_g, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_pooled_rows_change_the_output_and_disarm_restores():
    """The pooled rows enter the attention (the output differs from the
    unpooled one) and re-arming with pool_pages 0 gives the unpooled output
    back bit for bit."""
    w, shared, pool, _ = CASES["per_head_p128_bf16"]
    q, k, v = W.gen_layer(w, 0)
    ctx = make_ctx(w, shared=shared)
    base, _, _ = run_gpu(ctx, w, q, k, v)
    ctx.check(ctx.set_qg_bound(1, w.top_k, w.local_pages, pool))
    pooled, _, _ = run_gpu(ctx, w, q, k, v)
    assert not torch.equal(base, pooled)
    ctx.check(ctx.set_qg_bound(1, w.top_k, w.local_pages, 0))
    again, _, _ = run_gpu(ctx, w, q, k, v)
    assert torch.equal(base, again)


def test_pooled_rows_in_cta_ranges_equal_whole_call():
    w, shared, pool, _ = CASES["sub128_p64_gqa7"]
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    N = w.n_tokens
    ctx = make_ctx(w, shared=shared)
    ctx.check(ctx.set_ext(1, 128, 0))
    ctx.check(ctx.set_qg_bound(1, w.top_k, w.local_pages, pool))
    ref = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    ctx.check(ctx.attend_layer(0, q, k, v, N, N, ref))
    total = ctx.attention_grid(N) * w.n_head_kv
    cuts = ctx.balance_ctas(0, N, N, 3)
    per_head = ctx.attention_grid(N)
    out = torch.zeros_like(ref)
    for r in range(3):
        if cuts[r + 1] > cuts[r]:
            ctx.check(ctx.select_heads(0, q, k, v, N, N, cuts[r] // per_head, (cuts[r + 1] - 1) // per_head + 1))
            ctx.check(ctx.attend_ctas(0, N, N, cuts[r], cuts[r + 1], out))
    torch.cuda.synchronize()
    ctx.check(ctx.sync_status())
    assert cuts[-1] == total
    assert torch.equal(out, ref)
