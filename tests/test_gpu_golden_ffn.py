"""GPU checks against the committed known-answer fixtures, the K4 FFN-skip
compaction/scatter against the oracle (bit-exact), and full-size selection
parity at the benchmark sizes (64K and 128K tokens)."""
import glob
import os
import sys

import numpy as np
import pytest
import torch

import epsp
import oracle
import workloads as W
from gpu_util import assert_selection_equal, make_ctx, run_gpu, run_oracle, to_np

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_gpu_matches_golden(path):
    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_golden

    name = os.path.basename(path)[:-4]
    ref = np.load(path)
    w, shared, kb, _ = make_golden.CASES[name]
    q, k, v = W.gen_layer(w, 0)
    assert make_golden.digest(to_np(q), to_np(k), to_np(v)) == str(ref["input_sha256"])
    ctx = make_ctx(w, shared=shared, k_matrix=None if kb is None else [kb])
    out, sel, cnt = run_gpu(ctx, w, q, k, v)
    assert np.array_equal(cnt, ref["cnt"])
    for b in range(cnt.shape[0]):
        for h in range(cnt.shape[1]):
            n = cnt[b, h]
            assert np.array_equal(sel[b, h, :n], ref["sel"][b, h, :n])
    o = out.float().cpu().numpy()[ref["rows"]]
    err = np.abs(o - ref["out_rows"].astype(np.float64))
    assert err.max() <= 2e-3 and err.mean() <= 1e-3, (err.max(), err.mean())


# ------------------------------------------------------------------ FFN skip
@pytest.mark.parametrize("dtype", [W.BF16, W.F16, W.F32])
@pytest.mark.parametrize("frac", [0.0, 0.15, 1.0])
def test_ffn_compact_scatter_bit_exact(dtype, frac):
    n_rows, hidden = 1000, 256
    tdt = W.TORCH_DTYPE[dtype]
    g = torch.Generator().manual_seed(7)
    x = torch.randn(n_rows, hidden, generator=g).to(tdt)
    res = torch.randn(n_rows, hidden, generator=g).to(tdt)
    keep = (torch.rand(n_rows, generator=g) < frac).to(torch.uint8)
    ctx = epsp.Context(n_layer=4, n_head=8, n_head_kv=2, head_dim=64, dtype=dtype, max_ctx=1024)
    xd, rd, kd = x.cuda(), res.cuda(), keep.cuda()
    x_kept = torch.zeros_like(xd)
    ids = torch.full((n_rows,), -1, dtype=torch.int32, device="cuda")
    n_keep = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.check(ctx.ffn_compact(1, xd, kd, n_rows, hidden, x_kept, ids, n_keep))
    ffn_out = (x_kept.float() * 0.5 + 0.25).to(tdt)  # stand-in FFN output of the kept rows
    ctx.check(ctx.ffn_scatter(1, ffn_out, rd, ids, n_keep, n_rows, hidden))
    torch.cuda.synchronize()
    xk_o, ids_o = oracle.ffn_compact(to_np(x), to_np(keep))
    n = int(n_keep.item())
    assert n == len(ids_o)
    assert np.array_equal(ids[:n].cpu().numpy(), ids_o)
    assert np.array_equal(to_np(x_kept[:n]), xk_o)
    res_o = oracle.ffn_scatter(to_np(ffn_out[:n]), to_np(res), dtype, ids_o)
    assert np.array_equal(to_np(rd), res_o)


def test_ffn_layer_skip_mask_keeps_residual():
    """ffn patch :146-149: a skipped layer's FFN contributes zero; in prefill
    mode a layer in the FFN skip mask compacts no row."""
    n_rows, hidden = 512, 128
    ctx = epsp.Context(n_layer=4, n_head=8, n_head_kv=2, head_dim=64, dtype=epsp.BF16, max_ctx=1024)
    ctx.set_ffn_skip(0b0100)
    x = torch.randn(n_rows, hidden, device="cuda").to(torch.bfloat16)
    keep = torch.ones(n_rows, dtype=torch.uint8, device="cuda")
    x_kept = torch.zeros_like(x)
    ids = torch.zeros(n_rows, dtype=torch.int32, device="cuda")
    n_keep = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    ctx.set_prefill_mode(True)
    ctx.check(ctx.ffn_compact(2, x, keep, n_rows, hidden, x_kept, ids, n_keep))
    torch.cuda.synchronize()
    assert n_keep.item() == 0
    res = torch.randn(n_rows, hidden, device="cuda").to(torch.bfloat16)
    before = res.clone()
    ctx.check(ctx.ffn_scatter(2, x_kept, res, ids, n_keep, n_rows, hidden))
    torch.cuda.synchronize()
    assert torch.equal(res, before)
    ctx.check(ctx.ffn_compact(1, x, keep, n_rows, hidden, x_kept, ids, n_keep))  # layer 1 not skipped
    ctx.set_prefill_mode(False)
    ctx.check(ctx.ffn_compact(2, x, keep, n_rows, hidden, x_kept, ids, n_keep))  # not in prefill mode
    torch.cuda.synchronize()
    assert n_keep.item() == n_rows


# ------------------------------------------------------ full-size selection
@pytest.mark.parametrize("name,layer", [("c4", 0), ("c4", 20), ("c3", 5), ("c5", 3)])
def test_fullsize_selection_bit_exact(name, layer):
    """Selection of every gating block of one layer at the benchmark size,
    against the oracle; attention on a sample of rows."""
    w = W.CONFIGS[name]
    km = w.k_matrix()
    if km is None and w.top_k > 128:
        km = [[w.top_k] * w.n_head_kv for _ in range(w.n_layer)]
    q, k, v = W.gen_layer(w, layer, device="cuda")
    rows = np.sort(np.random.default_rng(layer).choice(w.n_tokens, 24, replace=False)).astype(np.int32)
    out_o, sel_o, cnt_o, _ = run_oracle(w, q, k, v, shared=0, k_budget=None if km is None else np.array(km[layer]),
                                        rows=rows)
    ctx = make_ctx(w, shared=0, n_layer=w.n_layer, k_matrix=km)
    out, sel, cnt = run_gpu(ctx, w, q, k, v, layer=layer)
    assert_selection_equal(sel, cnt, sel_o, cnt_o)
    assert cnt_o.sum() > 0
    o = out.float().cpu().numpy()[rows]
    err = np.abs(o - out_o[rows])
    assert err.max() <= 2e-3 and err.mean() <= 1e-3, (err.max(), err.mean())
