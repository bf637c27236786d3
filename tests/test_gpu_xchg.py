"""Head-parallel output exchange (ep_sp_attend_rows_xchg / ep_sp_xchg_wait)
on one GPU.

A 1-rank group must give exactly the bytes of ep_sp_attend_layer; two
head-slice contexts on the same GPU that exchange into each other's buffers
(the multi-GPU data path with local instead of peer memory: the K3 kernels
never wait on one another, so running them one after the other on one GPU is
sound) must both hold the full-width output of one context over all heads,
bit for bit; so must three whole-model contexts that each attend their
ep_sp_balance_ctas range of the head-major CTA grid.  Covers the staged-tile
epilogue (tiles inside their gating block) and the per-row store fallback
(tiles straddling a block end), slot rotation and counter accumulation over
several layers.
"""
from __future__ import annotations

import pytest
import torch

import epsp
import workloads as W
from gpu_util import attn_errors, run_oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3
# 32 q / 8 kv heads, d 128, bf16, page 128; gating blocks of 1024 rows (whole 32-token tiles)
BIG = W.Workload("xg", 4096, 3, 32, 8, 128, W.BF16, 4096, 128, 6, 256, per_kv_head=1, max_gather_rows=0,
                 q_subblock=1024)
# gating blocks of 100 rows: most query tiles straddle a block end (per-row store path)
ODD = W.Workload("xo", 1000, 2, 8, 2, 64, W.BF16, 1000, 32, 3, 64, per_kv_head=1, max_gather_rows=0,
                 q_subblock=100)


def ctx_for(w, kv0, kv1, n_layer):
    G = w.n_head // w.n_head_kv
    c = epsp.Context(n_layer=n_layer, n_head=(kv1 - kv0) * G, n_head_kv=kv1 - kv0, head_dim=w.head_dim,
                     dtype=w.dtype, out_dtype=w.dtype, max_ctx=w.n_tokens, page_size=w.page_size, device=0,
                     kv_head_offset=kv0, n_head_kv_total=w.n_head_kv)
    c.check(c.set_ext(1, w.q_subblock, w.max_gather_rows))
    c.check(c.set_qg_bound(1, w.top_k, w.local_pages, 0))
    c.set_prefill_mode(True)
    return c


def reference_outputs(w, layers):
    """ep_sp_attend_layer of one context over every head, per layer."""
    full = ctx_for(w, 0, w.n_head_kv, len(layers))
    outs = []
    for l, (q, k, v) in enumerate(layers):
        o = torch.empty_like(q)
        full.check(full.attend_layer(l, q, k, v, w.n_tokens, w.n_tokens, o))
        outs.append(o)
    torch.cuda.synchronize()
    full.check(full.sync_status())
    return outs


@pytest.mark.parametrize("w", [BIG, ODD], ids=["tma_tiles", "straddling_tiles"])
def test_single_rank_exchange_equals_attend_layer(w):
    N = w.n_tokens
    layers = [tuple(t.cuda() for t in W.gen_layer(w, l)) for l in range(w.n_layer)]
    ref = reference_outputs(w, layers)
    c = ctx_for(w, 0, w.n_head_kv, w.n_layer)
    base, _ = c.xchg_alloc(N, 2, ipc=False)
    c.check(c.xchg_attach(0, [base]))
    for l, (q, k, v) in enumerate(layers):
        c.check(c.select_layer(l, q, k, v, N, N))
        c.check(c.attend_rows_xchg(l, N, N, 0, N, l % 2))
        c.check(c.xchg_wait(l % 2, N))
        torch.cuda.synchronize()
        c.check(c.sync_status())
        got = epsp.device_view(c.xchg_slot(l % 2), (N, w.n_head, w.head_dim), w.dtype)
        assert torch.equal(got, ref[l]), f"layer {l}"


@pytest.mark.parametrize("w", [BIG, ODD], ids=["tma_tiles", "straddling_tiles"])
def test_two_head_slices_exchange_full_width_output(w):
    N, Hkv = w.n_tokens, w.n_head_kv
    half = Hkv // 2
    layers = [tuple(t.cuda() for t in W.gen_layer(w, l)) for l in range(w.n_layer)]
    ref = reference_outputs(w, layers)
    ranks = [ctx_for(w, 0, half, w.n_layer), ctx_for(w, half, Hkv, w.n_layer)]
    bases = [r.xchg_alloc(N, 2, ipc=False)[0] for r in ranks]
    for i, r in enumerate(ranks):
        r.check(r.xchg_attach(i, bases))
    G = w.n_head // Hkv
    slices = [W.gen_layer(w, l, head_slice=(0, half)) for l in range(w.n_layer)], \
        [W.gen_layer(w, l, head_slice=(half, Hkv)) for l in range(w.n_layer)]
    for l in range(w.n_layer):
        for i, r in enumerate(ranks):
            q, k, v = (t.cuda() for t in slices[i][l])
            r.check(r.select_layer(l, q, k, v, N, N))
            r.check(r.attend_rows_xchg(l, N, N, 0, N, l % 2))
        for r in ranks:
            r.check(r.xchg_wait(l % 2, N))
        torch.cuda.synchronize()
        for i, r in enumerate(ranks):
            r.check(r.sync_status())
            got = epsp.device_view(r.xchg_slot(l % 2), (N, w.n_head, w.head_dim), w.dtype)
            assert torch.equal(got, ref[l]), f"layer {l} rank {i}"
    # the exchanged output is the oracle's attention within tolerance
    q, k, v = layers[0]
    out_o, _, _, _ = run_oracle(w, q.cpu(), k.cpu(), v.cpu(), shared=0)
    mx, mean = attn_errors(ref[0].float(), out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean, G)


def test_exchange_wait_times_out_on_missing_peer():
    """A rank whose peer never writes: the bounded wait records the device
    error (rc 6 from ep_sp_sync_status), the context stays usable."""
    w = ODD
    N, Hkv = w.n_tokens, w.n_head_kv
    ranks = [ctx_for(w, 0, 1, 1), ctx_for(w, 1, 2, 1)]
    bases = [r.xchg_alloc(N, 2, ipc=False)[0] for r in ranks]
    for i, r in enumerate(ranks):
        r.check(r.xchg_attach(i, bases))
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0, head_slice=(0, 1)))
    r0 = ranks[0]
    r0.check(r0.select_layer(0, q, k, v, N, N))
    r0.check(r0.attend_rows_xchg(0, N, N, 0, N, 0))
    r0.check(r0.xchg_wait(0, N))       # rank 1 never attends: half the rows are missing
    torch.cuda.synchronize()
    assert r0.sync_status() == epsp.PREFILL
    assert "0x105" in r0.last_error()
    assert r0.sync_status() == epsp.OK  # the error word was cleared; the context still works


def test_exchange_argument_checks():
    w = ODD
    c = ctx_for(w, 0, w.n_head_kv, 1)
    assert c.xchg_attach(0, [0]) == epsp.INVALID_ARGUMENT            # no buffer yet
    base, _ = c.xchg_alloc(w.n_tokens, 2, ipc=False)
    assert c.xchg_attach(1, [base]) == epsp.INVALID_ARGUMENT         # rank out of range
    assert c.xchg_attach(0, [base + 4096]) == epsp.INVALID_ARGUMENT  # own base mismatch
    assert c.xchg_wait(0, 10) == epsp.INVALID_ARGUMENT               # not attached
    c.check(c.xchg_attach(0, [base]))
    assert c.xchg_attach(0, [base]) == epsp.INVALID_ARGUMENT         # attached once
    assert c.xchg_wait(2, 10) == epsp.INVALID_ARGUMENT               # slot out of range
    assert c.xchg_wait(0, w.n_tokens + 1) == epsp.INVALID_ARGUMENT   # more rows than a slot holds
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    assert c.attend_rows_xchg(0, w.n_tokens, w.n_tokens, 0, w.n_tokens, 0) == epsp.INVALID_ARGUMENT  # no select
    c.check(c.select_layer(0, q, k, v, w.n_tokens, w.n_tokens))
    assert c.attend_rows_xchg(0, w.n_tokens, w.n_tokens, 0, w.n_tokens, 5) == epsp.INVALID_ARGUMENT
    f32 = epsp.Context(n_layer=1, n_head=8, n_head_kv=2, head_dim=64, dtype=epsp.F32, out_dtype=epsp.F32,
                       max_ctx=1024, page_size=32, device=0)
    with pytest.raises(epsp.EpspError):
        f32.xchg_alloc(1024, 2, ipc=False)


@pytest.mark.parametrize("tiles", [2, 1], ids=["2_tiles_per_cta", "1_tile_per_cta"])
@pytest.mark.parametrize("w", [BIG, ODD], ids=["tma_tiles", "straddling_tiles"])
def test_balanced_cta_ranges_exchange_full_width_output(w, tiles):
    """Three 'ranks' with whole-model contexts, each attending its balanced
    CTA range (which cuts through KV heads and gating blocks), with either K3
    variant (the CTA grid differs, the output bits do not)."""
    N, n_parts = w.n_tokens, 3
    layers = [tuple(t.cuda() for t in W.gen_layer(w, l)) for l in range(w.n_layer)]
    ref = reference_outputs(w, layers)
    ranks = [ctx_for(w, 0, w.n_head_kv, w.n_layer) for _ in range(n_parts)]
    for r in ranks:
        r.check(r.set_attn_tiles(tiles))
    bases = [r.xchg_alloc(N, 2, ipc=False)[0] for r in ranks]
    for i, r in enumerate(ranks):
        r.check(r.xchg_attach(i, bases))
    per_head = ranks[0].attention_grid(N)
    for l, (q, k, v) in enumerate(layers):
        cuts = ranks[0].balance_ctas(l, N, N, n_parts)
        assert cuts[0] == 0 and cuts[-1] == per_head * w.n_head_kv and cuts == sorted(cuts)
        assert all(x.balance_ctas(l, N, N, n_parts) == cuts for x in ranks)
        for i, r in enumerate(ranks):
            c0, c1 = cuts[i], cuts[i + 1]
            if c1 > c0:
                r.check(r.select_heads(l, q, k, v, N, N, c0 // per_head, (c1 - 1) // per_head + 1))
                r.check(r.attend_ctas_xchg(l, N, N, c0, c1, l % 2))
        for r in ranks:
            r.check(r.xchg_wait(l % 2, N))
        torch.cuda.synchronize()
        for i, r in enumerate(ranks):
            r.check(r.sync_status())
            got = epsp.device_view(r.xchg_slot(l % 2), (N, w.n_head, w.head_dim), w.dtype)
            assert torch.equal(got, ref[l]), f"layer {l} rank {i}"


def test_cta_ranges_without_exchange_equal_attend_layer():
    """ep_sp_select_heads + ep_sp_attend_ctas over uneven CTA pieces write the
    same output as one ep_sp_attend_layer; a CTA range outside the selected
    heads is rejected."""
    w = BIG
    N = w.n_tokens
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    ref = reference_outputs(w, [(q, k, v)])[0]
    c = ctx_for(w, 0, w.n_head_kv, 1)
    per_head = c.attention_grid(N)
    out = torch.zeros_like(ref)
    edges = [0, 5, per_head - 3, per_head + 17, 3 * per_head, 3 * per_head + 1, w.n_head_kv * per_head]
    for a, b in zip(edges[:-1], edges[1:]):
        c.check(c.select_heads(0, q, k, v, N, N, a // per_head, (b - 1) // per_head + 1))
        c.check(c.attend_ctas(0, N, N, a, b, out))
    torch.cuda.synchronize()
    c.check(c.sync_status())
    assert torch.equal(out, ref)
    c.check(c.select_heads(0, q, k, v, N, N, 2, 4))
    assert c.attend_ctas(0, N, N, per_head, 3 * per_head, out) == epsp.INVALID_ARGUMENT   # head 1 not selected
    assert c.attend_ctas(0, N, N, 2 * per_head, 5 * per_head, out) == epsp.INVALID_ARGUMENT  # head 4 not selected
    assert c.attend_rows(0, N, N, 0, N, out) == epsp.INVALID_ARGUMENT  # rows need every head selected
    assert c.select_heads(0, q, k, v, N, N, 3, 3) == epsp.INVALID_ARGUMENT


@pytest.mark.parametrize("w", [BIG, ODD], ids=["tma_tiles", "straddling_tiles"])
def test_one_tile_per_cta_bit_identical(w):
    """The one-tile-per-CTA K3 variant (two CTAs per SM) writes exactly the
    bytes of the default two-tile variant, f32 and 16-bit outputs."""
    N = w.n_tokens
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    for out_dtype, tdt in ((epsp.F32, torch.float32), (w.dtype, torch.bfloat16)):
        outs = []
        for tiles in (2, 1):
            G = w.n_head // w.n_head_kv
            c = epsp.Context(n_layer=1, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                             dtype=w.dtype, out_dtype=out_dtype, max_ctx=N, page_size=w.page_size, device=0)
            c.check(c.set_ext(1, w.q_subblock, 0))
            c.check(c.set_qg_bound(1, w.top_k, w.local_pages, 0))
            c.set_prefill_mode(True)
            c.check(c.set_attn_tiles(tiles))
            assert c.attn_tiles() == tiles
            o = torch.zeros(q.shape, dtype=tdt, device="cuda")
            c.check(c.attend_layer(0, q, k, v, N, N, o))
            torch.cuda.synchronize()
            c.check(c.sync_status())
            outs.append(o)
            assert c.set_attn_tiles(3) == epsp.INVALID_ARGUMENT
        assert torch.equal(outs[0], outs[1])
