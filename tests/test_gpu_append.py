"""ep_sp_append_kv: KV-cache writes with the page sums fused in.

A prompt is appended in ragged chunks (straddling pages, one chunk smaller
than a page), each chunk followed by ep_sp_attend_layer on it, the reference's
chunked-prefill order.  The cache must hold exactly the appended rows; the
selected pages, their counts and the attention output must equal, bit for bit,
a context whose cache is written with plain copies and pooled by K1; and each
chunk's page lists must equal the oracle's selection (epo_select_block) over
the page sums of the rows appended so far.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import epsp
import oracle
import workloads as W
from gpu_util import to_np

pytestmark = pytest.mark.gpu

CASES = {
    # 32 q / 8 kv heads, d 128, bf16, page 128, per-KV-head top-k 6, window 256
    "p128_bf16": (W.Workload("ap", 4096, 2, 32, 8, 128, W.BF16, 4096, 128, 6, 256, per_kv_head=1,
                             max_gather_rows=0), [700, 1000, 33, 1363, 1000]),
    # reference mode (shared list, MAX over heads), page 32, f16, d 64
    "p32_f16_shared": (W.Workload("as", 2048, 1, 8, 2, 64, W.F16, 2048, 32, 4, 64, per_kv_head=0,
                                  max_gather_rows=4096), [512, 20, 300, 1216]),
    # f32 cache (16-byte vectors of 4 elements; attention in f32), page 64
    "p64_f32": (W.Workload("af", 2048, 1, 14, 2, 64, W.F32, 2048, 64, 5, 128, per_kv_head=1,
                           max_gather_rows=0), [1000, 48, 1000]),
}


def make(w):
    c = epsp.Context(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                     dtype=w.dtype, out_dtype=epsp.F32, max_ctx=w.n_tokens, page_size=w.page_size, device=0)
    c.check(c.set_ext(w.per_kv_head, 0, w.max_gather_rows))
    c.check(c.set_qg_bound(1, w.top_k, w.local_pages, 0))
    c.set_prefill_mode(True)
    return c


@pytest.mark.parametrize("name", sorted(CASES))
def test_append_then_attend_equals_copy_then_attend(name):
    w, chunks = CASES[name]
    assert sum(chunks) == w.n_tokens
    N, dev = w.n_tokens, torch.device("cuda")
    a, b = make(w), make(w)
    cap = N // w.page_size + 1
    for l in range(w.n_layer):
        q, k, v = (t.to(dev) for t in W.gen_layer(w, l))
        ka, va = torch.zeros_like(k), torch.zeros_like(v)
        kb, vb = torch.zeros_like(k), torch.zeros_like(v)
        pos = 0
        for n in chunks:
            r = slice(pos, pos + n)
            outs, sels = [], []
            for ctx, kc, vc, append in ((a, ka, va, True), (b, kb, vb, False)):
                if append:
                    ctx.check(ctx.append_kv(l, k[r].contiguous(), v[r].contiguous(), n, kc, vc, pos))
                else:
                    kc[r].copy_(k[r])
                    vc[r].copy_(v[r])
                _, nb = ctx.query_blocks(n)
                sel = torch.full((nb, w.n_head_kv, cap), -1, dtype=torch.int32, device=dev)
                cnt = torch.zeros((nb, w.n_head_kv), dtype=torch.int32, device=dev)
                out = torch.zeros((n, w.n_head, w.head_dim), dtype=torch.float32, device=dev)
                ctx.check(ctx.attend_layer(l, q[r].contiguous(), kc, vc, pos + n, n, out, sel, cnt, cap))
                outs.append(out)
                sels.append((sel, cnt))
            torch.cuda.synchronize()
            a.check(a.sync_status())
            b.check(b.sync_status())
            assert torch.equal(sels[0][1], sels[1][1]), (l, pos)
            for bi in range(sels[0][1].shape[0]):
                for h in range(sels[0][1].shape[1]):
                    m = int(sels[0][1][bi, h])
                    assert torch.equal(sels[0][0][bi, h, :m], sels[1][0][bi, h, :m]), (l, pos, bi, h)
            assert torch.equal(outs[0], outs[1]), (l, pos)
            # the appended cache's selection against the oracle directly: page
            # sums of the rows written so far, the chunk's last query row
            p = oracle.params(n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                              page_size=w.page_size, sel_pages=w.top_k, local_pages=w.local_pages,
                              shared=0 if w.per_kv_head else 1, max_gather_rows=w.max_gather_rows)
            plan = oracle.plan_block(p, pos, pos + n, w.top_k)
            ps = oracle.page_sums(to_np(ka[:pos + n]), w.dtype, w.page_size)
            cnt_a = sels[0][1].cpu().numpy()
            sel_a = sels[0][0].cpu().numpy()
            for h in range(w.n_head_kv):
                want = oracle.select_block(p, plan, to_np(q[pos + n - 1]), w.dtype, ps, h if w.per_kv_head else -1)
                assert cnt_a[0, h] == len(want), (l, pos, h)
                assert np.array_equal(sel_a[0, h, :len(want)], want), (l, pos, h)
            pos += n
        assert torch.equal(ka, k) and torch.equal(va, v)


def test_append_argument_checks():
    w, _ = CASES["p128_bf16"]
    c = make(w)
    k = torch.zeros((16, w.n_head_kv, w.head_dim), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((w.n_tokens, w.n_head_kv, w.head_dim), dtype=torch.bfloat16, device="cuda")
    assert c.append_kv(2, k, k, 16, kc, kc, 0) == epsp.INVALID_ARGUMENT            # layer
    assert c.append_kv(0, k, k, 0, kc, kc, 0) == epsp.INVALID_ARGUMENT             # no rows
    assert c.append_kv(0, k, k, 16, kc, kc, w.n_tokens - 8) == epsp.INVALID_ARGUMENT  # past max_ctx
    assert c.append_kv(0, None, k, 16, kc, kc, 0) == epsp.INVALID_ARGUMENT         # null
