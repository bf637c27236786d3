"""The no-allocation page selection (ep_sp_select_pages_noalloc) against the
regular path (ep_sp_attend_layer's selection outputs).

The entry point serves callers that cannot allocate device memory at the
point of use -- an operator inside a graph executor that pre-plans all of
its buffers, or a host with a fixed device-memory budget -- so it keeps its
scratch in a fixed-size array inside the library.  Its page lists must be
identical to the regular path's (page indices are compared exactly, the
tolerance every selection test here uses), call after call, although every
call reuses the same scratch array.

Kept in a file of its own, collected last, and self-contained: it passes in a
fresh process and after the rest of the suite.
"""
import numpy as np
import pytest
import torch

import epsp
import workloads as W

pytestmark = pytest.mark.gpu

CAP = 64


def _ctx(w, shared, k_matrix=None):
    ctx = epsp.Context(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                       dtype=w.dtype, out_dtype=epsp.F32, max_ctx=w.n_tokens, page_size=w.page_size)
    ctx.check(ctx.set_ext(0 if shared else 1, w.q_subblock, w.max_gather_rows))
    if k_matrix is not None:
        ctx.check(ctx.set_k_matrix([x for row in k_matrix for x in row]))
    ctx.check(ctx.set_qg_bound(1, min(w.top_k, 128), w.local_pages, 0))
    ctx.set_prefill_mode(True)
    return ctx


def _regular_selection(w, shared, k_matrix, q, k, v):
    """Selection lists of every ubatch through ep_sp_attend_layer."""
    ctx = _ctx(w, shared, k_matrix)
    out = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    rc, ranges = epsp.chunk_plan(w.n_tokens, 0, w.n_ubatch)
    assert rc == 0
    res = []
    for a, b in ranges:
        _, nb = ctx.query_blocks(b - a)
        sel = torch.full((nb, w.n_head_kv, CAP), -7, dtype=torch.int32, device="cuda")
        cnt = torch.full((nb, w.n_head_kv), -7, dtype=torch.int32, device="cuda")
        ctx.check(ctx.attend_layer(0, q[a:b], k, v, b, b - a, out[a:b], sel, cnt, CAP))
        res.append((a, b, sel, cnt))
    torch.cuda.synchronize()
    ctx.check(ctx.sync_status())
    return res


def _compare(sel_a, cnt_a, sel_b, cnt_b):
    ca, cb = cnt_a.cpu().numpy(), cnt_b.cpu().numpy()
    assert np.array_equal(ca, cb), (ca, cb)
    sa, sb = sel_a.cpu().numpy(), sel_b.cpu().numpy()
    for bl in range(ca.shape[0]):
        for h in range(ca.shape[1]):
            n = ca[bl, h]
            assert np.array_equal(sa[bl, h, :n], sb[bl, h, :n]), (bl, h)


CASES = {
    # per-KV-head lists, page 128, head_dim 128, a k-matrix with a dense head
    "per_head_p128": (W.Workload("na1", 8192, 1, 32, 8, 128, W.BF16, 2048, 128, 8, 1024, max_gather_rows=0),
                      0, [[8, 16, 4, -1, 8, 2, 12, 8]]),
    # the reference's mode: page 32, one shared list, 4096-row guard
    "shared_p32": (W.Workload("na2", 4096, 1, 8, 2, 64, W.F16, 512, 32, 8, 128, per_kv_head=0,
                              max_gather_rows=4096), 1, None),
}


@pytest.mark.parametrize("name", list(CASES))
def test_noalloc_matches_regular_path_on_consecutive_calls(name):
    w, shared, km = CASES[name]
    torch.cuda.set_device(0)
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    regular = _regular_selection(w, shared, km, q, k, v)
    ctx = _ctx(w, shared, km)  # never reserved: the entry point must not need it
    gated = [r for r in regular if int(r[3].clamp(min=0).sum()) > 0]
    assert len(gated) >= 2, "the case must gate at least two ubatches"
    # two calls in a row on different ubatches, then the first again: each must
    # match the regular path although they share one scratch array
    for a, b, sel_a, cnt_a in gated[-2:] + gated[-2:-1]:
        _, nb = ctx.query_blocks(b - a)
        sel = torch.full((nb, w.n_head_kv, CAP), -9, dtype=torch.int32, device="cuda")
        cnt = torch.full((nb, w.n_head_kv), -9, dtype=torch.int32, device="cuda")
        ctx.check(ctx.select_pages_noalloc(0, q[a:b], k, b, b - a, sel, cnt, CAP))
        torch.cuda.synchronize()
        _compare(sel_a, cnt_a, sel, cnt)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    # 8 KV heads x d 128 x 8 bytes = 8 KiB of page sums per scored page; a
    # ubatch ending at row 32768 with page 32 scores ~1000 pages (> 4 MiB).
    w = W.Workload("na3", 32768, 1, 32, 8, 128, W.BF16, 4096, 32, 8, 64, max_gather_rows=0)
    torch.cuda.set_device(0)
    ctx = _ctx(w, 0)
    q = torch.zeros(4096, 32, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(32768, 8, 128, dtype=torch.bfloat16, device="cuda")
    sel = torch.zeros((1, 8, CAP), dtype=torch.int32, device="cuda")
    cnt = torch.zeros((1, 8), dtype=torch.int32, device="cuda")
    rc = ctx.select_pages_noalloc(0, q, k, 32768, 4096, sel, cnt, CAP)
    assert rc == epsp.INVALID_ARGUMENT
    assert "exceed the no-allocation scratch" in ctx.last_error()
