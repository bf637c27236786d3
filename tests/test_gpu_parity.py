"""GPU parity of the page-gated path through the C ABI against the CPU oracle.

Bars:
  * selected page indices and per-block counts: bit-exact;
  * attention output: max-abs <= 2e-3 and mean-abs <= 1e-3 against the fp64
    oracle (f32 output).  With a 16-bit output the stored value also carries
    its own rounding (2^-8 relative for bf16), so the max-abs bar there is
    2e-3 + 2^-8 * |ref|.
Cases cover the reference mode (P = 32, one shared list, MAX over KV heads,
k_sel = min(sel, lsp) with its off-by-one page 0, the 4096-row guard) and the
extended modes (P = 64 / 128, per-KV-head lists, sub-blocks, k-matrix with a
dense head, GQA groups of 4 and 7, head_dim 64 / 128, f32 / f16 / bf16), ragged
lengths, ties, disarm/restore and determinism.
"""
import numpy as np
import pytest
import torch

import epsp
import workloads as W
from gpu_util import (assert_selection_equal, attn_errors, make_ctx, run_gpu, run_oracle, to_np,
                      torch_dense_reference)

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-3, 1e-3

BASE = W.Workload("t", 1024, 1, 8, 2, 64, W.BF16, 256, 32, 4, 64, per_kv_head=0, max_gather_rows=4096)

CASES = {
    # reference mode: P=32, shared list, 4096 guard
    "ref_p32": (W.scaled(BASE), 1, None),
    # reference off-by-one: sel >= lsp selects page 0 (sink duplicated)
    "ref_p32_offbyone": (W.scaled(BASE, top_k=8), 1, None),
    # reference mode, ragged length and ubatch
    "ref_ragged": (W.scaled(BASE, n_tokens=777, n_ubatch=200, dtype=W.F16), 1, None),
    # extended: per-KV-head, P=64, sub-blocks of 128, f16
    "ext_p64_sub128_f16": (W.scaled(BASE, page_size=64, local_rows=128, top_k=3, n_ubatch=1024, q_subblock=128,
                                    dtype=W.F16, max_gather_rows=0), 0, None),
    # extended: P=128, d=128, k-matrix with a dense head
    "ext_p128_kmatrix": (W.scaled(BASE, n_tokens=2048, n_ubatch=512, page_size=128, local_rows=256, head_dim=128,
                                  top_k=2, max_gather_rows=0), 0, [[-1, 3]]),
    # GQA group of 7 (T = 18 tokens per tile), P=64, sub-blocks of 64
    "gqa7_p64": (W.scaled(BASE, n_head=28, n_head_kv=4, head_dim=128, page_size=64, local_rows=128, top_k=4,
                          n_ubatch=512, q_subblock=64, max_gather_rows=0), 0, None),
    # f32 inputs (c1-like shapes), P=64, sub-blocks of 128
    "c1_like_f32": (W.scaled(W.CONFIGS["c1"], n_tokens=2048, n_ubatch=2048, top_k=4), 0, None),
    # needle data (c2-like), f16, ubatch 512
    "c2_like_needles": (W.scaled(W.CONFIGS["c2"], n_tokens=2048, n_layer=1, top_k=4, local_rows=128), 0, None),
}


@pytest.mark.parametrize("name", list(CASES))
def test_parity(name):
    w, shared, kmat = CASES[name]
    q, k, v = W.gen_layer(w, 0)
    kb = None if kmat is None else np.array(kmat[0], np.int32)
    out_o, sel_o, cnt_o, blocks = run_oracle(w, q, k, v, shared=shared, k_budget=kb)
    ctx = make_ctx(w, shared=shared, k_matrix=kmat)
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    assert cnt_o.sum() > 0 or name == "ref_ragged", "case must exercise selection"
    mx, mean = attn_errors(out_g, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_offbyone_includes_sink():
    w, shared, _ = CASES["ref_p32_offbyone"]
    q, k, v = W.gen_layer(w, 0)
    _, sel_o, cnt_o, blocks = run_oracle(w, q, k, v, shared=shared, attention=False)
    hit = [(b, sel_o[b, 0, :cnt_o[b, 0]]) for b in range(len(blocks)) if cnt_o[b, 0] and sel_o[b, 0, 0] == 0]
    assert hit, "the reference off-by-one (page 0 selected) must occur in this case"


def test_bf16_output_tolerance():
    w, shared, _ = CASES["ext_p128_kmatrix"]
    w = W.scaled(w, top_k=3)
    q, k, v = W.gen_layer(w, 0)
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=0)
    ctx = make_ctx(w, shared=0, out_dtype=epsp.BF16)
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v, out_dtype=torch.bfloat16)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    o = out_g.float().cpu().numpy()
    bound = MAX_ABS + np.abs(out_o) * 2.0 ** -8
    assert np.all(np.abs(o - out_o) <= bound)
    assert np.abs(o - out_o).mean() <= MEAN_ABS


def test_ties_break_to_lower_page():
    w = W.scaled(BASE, n_tokens=1024, n_ubatch=512, per_kv_head=1, max_gather_rows=0, local_rows=64, top_k=3)
    q, k, v = W.gen_layer(w, 0)
    P = w.page_size
    k = k.clone()
    page = k[P:2 * P].clone()
    for p in range(1, w.n_tokens // P):  # every page but the sink identical -> all scores tie
        k[p * P:(p + 1) * P] = page
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=0)
    ctx = make_ctx(w, shared=0)
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    b = cnt_o.shape[0] - 1
    assert list(sel_o[b, 0, :cnt_o[b, 0]]) == list(range(1, 1 + cnt_o[b, 0]))
    mx, mean = attn_errors(out_g, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS


def test_reference_guard_zeroes_selection_at_4096_ubatch():
    # Reference mode at ubatch 4096: n_local > 4096 so k_sel = 0 (patch :993);
    # gating still engages (local-only gather).
    w = W.scaled(BASE, n_tokens=8192, n_ubatch=4096, local_rows=0, top_k=8, head_dim=64)
    q, k, v = W.gen_layer(w, 0)
    rows = np.arange(4096, 8192, 37, dtype=np.int32)
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=1, rows=rows)
    assert cnt_o.sum() == 0
    ctx = make_ctx(w, shared=1)
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    mx, mean = attn_errors(out_g, out_o, rows)
    assert mx <= MAX_ABS and mean <= MEAN_ABS


@pytest.mark.parametrize("d,dtype", [(64, W.BF16), (128, W.F16), (128, W.BF16)])
def test_dense_matches_torch_fp32(d, dtype):
    """Disarmed: the same kernel runs dense causal attention; compare with a
    plain torch fp32 reference of the same op."""
    w = W.scaled(BASE, n_tokens=1000, n_ubatch=300, head_dim=d, dtype=dtype)
    q, k, v = W.gen_layer(w, 0)
    ctx = make_ctx(w, shared=1, armed=False)
    out_g, _, cnt = run_gpu(ctx, w, q, k, v)
    assert cnt.sum() == 0
    ref = torch_dense_reference(q.cuda(), k.cuda(), v.cuda())
    err = (out_g - ref).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS


def test_disarm_restores_dense_bit_identical_and_deterministic():
    """bound_gating_execution_and_restore (tests/test_sparse_attn_exec.cpp
    :1596-1662): gated outputs are finite and deterministic; after disarming,
    the dense path is bit-identical to the untouched run."""
    w = W.scaled(BASE, n_tokens=1024, n_ubatch=256, top_k=4, local_rows=32)
    q, k, v = W.gen_layer(w, 0)
    ctx = make_ctx(w, shared=1, armed=False)
    dense1, _, _ = run_gpu(ctx, w, q, k, v)
    ctx.check(ctx.set_qg_bound(1, 4, 1, 0))
    g1, s1, c1 = run_gpu(ctx, w, q, k, v)
    g2, s2, c2 = run_gpu(ctx, w, q, k, v)
    assert torch.isfinite(g1).all()
    assert torch.equal(g1, g2) and np.array_equal(s1, s2) and np.array_equal(c1, c2)
    assert c1.sum() > 0
    assert not torch.equal(g1, dense1)
    ctx.check(ctx.set_qg_bound(0, 0, 0, 0))
    dense2, _, _ = run_gpu(ctx, w, q, k, v)
    assert torch.equal(dense1, dense2)


def test_prefill_loop_matches_per_layer_calls():
    """ep_sp_prefill (native chunk loop, arms/disarms itself) gives the same
    result as the per-layer calls and always leaves gating disarmed."""
    w = W.scaled(BASE, n_tokens=1024, n_ubatch=256, top_k=4, local_rows=64)
    layers = [W.gen_layer(w, l) for l in range(2)]
    ctx = epsp.Context(n_layer=2, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim, dtype=w.dtype,
                       out_dtype=epsp.F32, max_ctx=w.n_tokens, page_size=w.page_size)
    opts = epsp.PrefillOptions(0, 1, 1, 4, w.local_pages, 0)
    qs = [t[0].cuda() for t in layers]
    ks = [t[1].cuda() for t in layers]
    vs = [t[2].cuda() for t in layers]
    outs = [torch.zeros(q.shape, dtype=torch.float32, device="cuda") for q in qs]
    rc, stats = ctx.prefill(opts, qs, ks, vs, outs, w.n_tokens, w.n_ubatch)
    ctx.check(rc)
    ctx.check(ctx.sync_status())
    assert stats.query_gating == 1 and stats.attn_fallback == 0 and stats.chunks == 4
    assert ctx.qg_bound() == 0 and ctx.prefill_mode() == 0
    for l in range(2):
        out_o, _, _, _ = run_oracle(w, layers[l][0], layers[l][1], layers[l][2], shared=1)
        mx, mean = attn_errors(outs[l], out_o)
        assert mx <= MAX_ABS and mean <= MEAN_ABS
    # a rejected arming degrades to dense, never fails
    bad = epsp.PrefillOptions(0, 1, 1, 129, 0, 0)
    rc, stats = ctx.prefill(bad, qs, ks, vs, outs, w.n_tokens, w.n_ubatch)
    ctx.check(rc)
    assert stats.attn_fallback == 1 and stats.query_gating == 0
    ref = torch_dense_reference(qs[0], ks[0], vs[0])
    torch.cuda.synchronize()
    assert (outs[0] - ref).abs().max().item() <= MAX_ABS


def test_bad_sizes_rejected():
    w = W.scaled(BASE)
    q, k, v = W.gen_layer(w, 0)
    ctx = make_ctx(w, shared=1)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    out = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    assert ctx.attend_layer(1, qd, kd, vd, 256, 256, out) == epsp.INVALID_ARGUMENT   # layer
    assert ctx.attend_layer(0, qd, kd, vd, 100, 256, out) == epsp.INVALID_ARGUMENT   # kv_len < n_tok
    assert ctx.attend_layer(0, qd, kd, vd, 2048, 256, out) == epsp.INVALID_ARGUMENT  # > max_ctx
    assert ctx.attend_layer(0, qd, kd, vd, 256, 0, out) == epsp.INVALID_ARGUMENT     # empty
    sel = torch.zeros((1, 2, 1), dtype=torch.int32, device="cuda")
    cnt = torch.zeros((1, 2), dtype=torch.int32, device="cuda")
    # sel_cap 1 is smaller than this block's k_sel
    assert ctx.attend_layer(0, qd[768:], kd, vd, 1024, 256, out[768:], sel, cnt, 1) == epsp.INVALID_ARGUMENT


def test_select_then_attend_rows_in_chunks_equals_attend_layer():
    """A whole-prompt call gated per 256-row block, attended in 4 chunks of
    gating blocks (the overlap schedule), equals the single ep_sp_attend_layer
    call bit for bit, and the row ranges are validated."""
    w = W.scaled(BASE, n_tokens=2048, n_ubatch=2048, q_subblock=256, per_kv_head=1, max_gather_rows=0, top_k=3)
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    ctx = make_ctx(w, shared=0)
    ref = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    ctx.check(ctx.attend_layer(0, q, k, v, 2048, 2048, ref))
    out = torch.zeros_like(ref)
    ctx.check(ctx.select_layer(0, q, k, v, 2048, 2048))
    for r0 in range(0, 2048, 512):
        ctx.check(ctx.attend_rows(0, 2048, 2048, r0, r0 + 512, out))
    torch.cuda.synchronize()
    ctx.check(ctx.sync_status())
    assert torch.equal(out, ref)
    assert ctx.attend_rows(0, 2048, 2048, 100, 512, out) == epsp.INVALID_ARGUMENT   # not block aligned
    assert ctx.attend_rows(0, 2048, 1024, 0, 512, out) == epsp.INVALID_ARGUMENT     # no matching selection
    ctx.check(ctx.set_qg_bound(1, 2, 2, 0))                                         # settings changed
    assert ctx.attend_rows(0, 2048, 2048, 0, 512, out) == epsp.INVALID_ARGUMENT
    out_o, _, _, _ = run_oracle(w, q.cpu(), k.cpu(), v.cpu(), shared=0)
    mx, mean = attn_errors(ref, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS


# ------------------------------------------------------------ f32 inputs
def _c1_small():
    return W.scaled(W.CONFIGS["c1"], n_tokens=2048, n_ubatch=2048, top_k=4)


@pytest.mark.parametrize("mode", [0, 1])
def test_f32_modes_match_oracle(mode):
    """c1 shapes (f32 Q/K/V, GQA 7, d 64): mode 0 attends in fp32 on the CUDA
    cores, mode 1 on f16 shadows with the tensor cores; both within the bar,
    and mode 0 far inside it."""
    w = _c1_small()
    q, k, v = W.gen_layer(w, 0)
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=0)
    ctx = make_ctx(w, shared=0)
    ctx.check(ctx.set_f32_attention(mode))
    assert ctx.f32_attention() == mode
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    assert cnt_o.sum() > 0
    mx, mean = attn_errors(out_g, out_o)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    if mode == 0:
        assert mx <= 1e-5, mx  # fp32 arithmetic, no 16-bit rounding anywhere


def _beyond_f16(w):
    """c1 data with a few K and V entries at +-1e5, outside the f16 range."""
    q, k, v = W.gen_layer(w, 0)
    g = torch.Generator().manual_seed(11)
    for t in (k, v):
        flat = t.view(-1)
        idx = torch.randperm(flat.numel(), generator=g)[:40]
        flat[idx] = torch.where(torch.rand(40, generator=g) < 0.5, -1e5, 1e5)
    return q, k, v


def test_f32_beyond_f16_range_attended_in_f32():
    w = _c1_small()
    q, k, v = _beyond_f16(w)
    assert k.abs().max().item() > 65504 and v.abs().max().item() > 65504
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=0)
    ctx = make_ctx(w, shared=0)  # mode 0 (default)
    out_g, sel_g, cnt_g = run_gpu(ctx, w, q, k, v)
    assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o)
    o = out_g.cpu().numpy().astype(np.float64)
    assert np.isfinite(o).all()
    err = np.abs(o - out_o)
    assert np.all(err <= MAX_ABS + 1e-5 * np.abs(out_o)), float((err - 1e-5 * np.abs(out_o)).max())


def test_f32_beyond_f16_range_rejected_by_tensor_core_mode():
    w = _c1_small()
    q, k, v = _beyond_f16(w)
    ctx = make_ctx(w, shared=0)
    ctx.check(ctx.set_f32_attention(1))
    dev = torch.device("cuda")
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.zeros(q.shape, dtype=torch.float32, device=dev)
    ctx.check(ctx.attend_layer(0, qd, kd, vd, w.n_tokens, w.n_tokens, out))
    assert ctx.sync_status() == epsp.UNSUPPORTED
    assert "f16 range" in ctx.last_error()
    assert ctx.sync_status() == epsp.OK  # the word is cleared once reported
    assert ctx.set_f32_attention(2) == epsp.INVALID_ARGUMENT


def test_f32_cta_ranges_cover_the_call():
    """The f32 kernel keeps K3's CTA grid: attending two halves of the grid
    through ep_sp_attend_ctas equals one whole call, bit for bit."""
    w = W.scaled(_c1_small(), q_subblock=256)
    q, k, v = (t.cuda() for t in W.gen_layer(w, 0))
    N = w.n_tokens
    ctx = make_ctx(w, shared=0)
    ref = torch.zeros(q.shape, dtype=torch.float32, device="cuda")
    ctx.check(ctx.attend_layer(0, q, k, v, N, N, ref))
    per_head = ctx.attention_grid(N)
    total = per_head * w.n_head_kv
    out = torch.zeros_like(ref)
    ctx.check(ctx.select_layer(0, q, k, v, N, N))
    ctx.check(ctx.attend_ctas(0, N, N, 0, total // 3, out))
    ctx.check(ctx.attend_ctas(0, N, N, total // 3, total, out))
    torch.cuda.synchronize()
    ctx.check(ctx.sync_status())
    assert torch.equal(out, ref)
