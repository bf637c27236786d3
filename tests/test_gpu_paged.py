"""Paged KV cache (ep_sp_set_paged_kv): the KV-layout adapter.

The logical cache of a sequence is scattered over a pool of fixed-size blocks
in a shuffled order, through a device block table; every other block of the
pool, and the rows of the sequence's last block past kv_len, hold stale data
(NaN included).  The paged calls must give the same page lists and the same
attention output, bit for bit, as the contiguous layout on the logical cache,
and within the usual bars of the oracle; the fused append must write each new
row to its table row; a table entry outside the pool is reported, not used.
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
    # per-KV-head, page 128, blocks of 128 rows, bf16, ragged length (last block partial)
    "p128_b128_bf16": (W.Workload("pg1", 2000, 1, 32, 8, 128, W.BF16, 500, 128, 3, 256, max_gather_rows=0), 128),
    # the reference's mode (shared list, page 32), blocks of 64 rows, f16
    "p32_b64_f16_shared": (W.Workload("pg2", 1500, 1, 8, 2, 64, W.F16, 512, 32, 4, 64, per_kv_head=0,
                                      max_gather_rows=4096), 64),
    # f32 attended in f32, page 64, blocks of 64 rows
    "p64_b64_f32": (W.scaled(W.CONFIGS["c1"], n_tokens=1800, n_ubatch=600, top_k=3), 64),
}


def make_pool(k, v, block_rows, seed):
    """Scatter the logical cache into a shuffled pool with stale rows (NaN in
    every stale row).  Returns (k_pool, v_pool, table, pool_rows)."""
    n = k.shape[0]
    n_blk = (n + block_rows - 1) // block_rows
    pool_blocks = n_blk + 5
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(pool_blocks, generator=g)[:n_blk].to(torch.int32)
    rows = pool_blocks * block_rows
    kp = torch.full((rows,) + k.shape[1:], float("nan"), dtype=k.dtype)
    vp = torch.full((rows,) + v.shape[1:], float("nan"), dtype=v.dtype)
    for b in range(n_blk):
        lo, hi = b * block_rows, min(n, (b + 1) * block_rows)
        p = int(perm[b]) * block_rows
        kp[p:p + hi - lo] = k[lo:hi]
        vp[p:p + hi - lo] = v[lo:hi]
    return kp.cuda(), vp.cuda(), perm.cuda(), rows


@pytest.mark.parametrize("name", list(CASES))
def test_paged_equals_contiguous_and_oracle(name):
    w, B = CASES[name]
    shared = 0 if w.per_kv_head else 1
    q, k, v = W.gen_layer(w, 0)
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=shared)
    ctx_c = make_ctx(w, shared=shared)
    out_c, sel_c, cnt_c = run_gpu(ctx_c, w, q, k, v)
    kp, vp, table, rows = make_pool(k, v, B, seed=3)
    ctx_p = make_ctx(w, shared=shared)
    ctx_p.check(ctx_p.set_paged_kv(B, table, table.numel(), rows))
    out_p, sel_p, cnt_p = run_gpu(ctx_p, w, q, kp, vp)
    assert_selection_equal(sel_p, cnt_p, sel_c, cnt_c)
    assert_selection_equal(sel_p, cnt_p, sel_o, cnt_o)
    assert cnt_o.sum() > 0
    assert torch.isfinite(out_p).all()
    assert torch.equal(out_p, out_c)
    mx, mean = attn_errors(out_p, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_paged_append_writes_table_rows_and_matches_contiguous():
    w, B = CASES["p128_b128_bf16"]
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    n = w.n_tokens
    n_blk = (n + B - 1) // B
    g = torch.Generator().manual_seed(7)
    table = torch.randperm(n_blk + 3, generator=g)[:n_blk].to(torch.int32).cuda()
    rows = (n_blk + 3) * B
    kp = torch.full((rows, w.n_head_kv, w.head_dim), float("nan"), dtype=k.dtype, device="cuda")
    vp = torch.full_like(kp, float("nan"))
    kc, vc = torch.zeros_like(k), torch.zeros_like(v)
    a, c = make_ctx(w, shared=0), make_ctx(w, shared=0)
    a.check(a.set_paged_kv(B, table, n_blk, rows))
    cap = n // w.page_size + 1
    pos = 0
    for chunk in (700, 60, 1240):
        r = slice(pos, pos + chunk)
        outs, sels = [], []
        for ctx, kk, vv in ((a, kp, vp), (c, kc, vc)):
            ctx.check(ctx.append_kv(0, k[r].contiguous(), v[r].contiguous(), chunk, kk, vv, pos))
            _, nb = ctx.query_blocks(chunk)
            sel = torch.full((nb, w.n_head_kv, cap), -1, dtype=torch.int32, device="cuda")
            cnt = torch.zeros((nb, w.n_head_kv), dtype=torch.int32, device="cuda")
            out = torch.zeros((chunk, w.n_head, w.head_dim), dtype=torch.float32, device="cuda")
            ctx.check(ctx.attend_layer(0, q[r].contiguous(), kk, vv, pos + chunk, chunk, out, sel, cnt, cap))
            outs.append(out)
            sels.append((sel, cnt))
        torch.cuda.synchronize()
        a.check(a.sync_status())
        assert torch.equal(sels[0][1], sels[1][1])
        assert torch.equal(outs[0], outs[1])
        pos += chunk
    # every logical row sits at its table row
    phys = (table.long()[torch.arange(n, device="cuda") // B] * B + torch.arange(n, device="cuda") % B)
    assert torch.equal(kp[phys], k) and torch.equal(vp[phys], v)


def test_paged_bad_table_entry_reported():
    w, B = CASES["p32_b64_f16_shared"]
    q, k, v = W.gen_layer(w, 0)
    kp, vp, table, rows = make_pool(k, v, B, seed=5)
    table[3] = rows // B + 10  # outside the pool
    ctx = make_ctx(w, shared=0 if w.per_kv_head else 1)
    ctx.check(ctx.set_paged_kv(B, table, table.numel(), rows))
    out = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    qd = q.cuda()
    ctx.check(ctx.attend_layer(0, qd, kp, vp, w.n_tokens, w.n_tokens, out))
    assert ctx.sync_status() == epsp.PREFILL
    assert "block table" in ctx.last_error()
    # argument rules
    assert ctx.set_paged_kv(48, table, table.numel(), rows) == epsp.INVALID_ARGUMENT  # not a page multiple
    assert ctx.set_paged_kv(B, None, 4, rows) == epsp.INVALID_ARGUMENT
    ctx.check(ctx.set_paged_kv(B, table, 2, rows))                                   # covers 128 rows only
    assert ctx.attend_layer(0, qd, kp, vp, w.n_tokens, w.n_tokens, out) == epsp.INVALID_ARGUMENT
    ctx.check(ctx.set_paged_kv(0))
