"""Shared helpers of the GPU parity tests: run one layer through the C ABI
chunk by chunk, and the same layer through the CPU oracle."""
from __future__ import annotations

import numpy as np
import torch

import epsp
import oracle
import workloads as W


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def oracle_params(w: W.Workload, shared: int, sel_pages: int, max_gather_rows: int, pool_pages: int = 0,
                  route_mode: int = 0, route_threshold: float = 0.0):
    return oracle.params(n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim, page_size=w.page_size,
                         sel_pages=sel_pages, local_pages=w.local_pages, shared=shared, q_subblock=w.q_subblock,
                         max_gather_rows=max_gather_rows, pool_pages=pool_pages, route_mode=route_mode,
                         route_threshold=route_threshold)


def run_oracle(w: W.Workload, q, k, v, *, shared, k_budget=None, rows=None, attention=True, pool_pages=0,
               return_pool=False, route_mode=0, route_threshold=0.0):
    p = oracle_params(w, shared, w.top_k, w.max_gather_rows, pool_pages, route_mode, route_threshold)
    return oracle.prefill_layer(p, to_np(q), to_np(k), to_np(v), w.dtype, n_ubatch=w.n_ubatch,
                                k_budget=k_budget, rows=rows, attention=attention,
                                sel_cap=max(1, q.shape[0] // w.page_size + 1), return_pool=return_pool)


def make_ctx(w: W.Workload, *, shared, out_dtype=epsp.F32, n_layer=1, k_matrix=None, armed=True, device=0):
    ctx = epsp.Context(n_layer=n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                       dtype=w.dtype, out_dtype=out_dtype, max_ctx=w.n_tokens, page_size=w.page_size,
                       device=device)
    ctx.check(ctx.set_ext(0 if shared else 1, w.q_subblock, w.max_gather_rows))
    if k_matrix is not None:
        ctx.check(ctx.set_k_matrix([x for row in k_matrix for x in row]))
    if armed:
        ctx.check(ctx.set_qg_bound(1, min(w.top_k, 128), w.local_pages, 0))
    ctx.set_prefill_mode(True)
    return ctx


def run_gpu(ctx: epsp.Context, w: W.Workload, q, k, v, *, layer=0, out_dtype=torch.float32, sel_cap=None,
            pooled=None):
    """Chunk loop through ep_sp_attend_layer; returns out (torch, cuda), and
    per-chunk (sel, cnt) numpy arrays concatenated over blocks.  With a list
    `pooled`, each chunk's (pooled pages, counts) are appended to it."""
    N = q.shape[0]
    dev = torch.device("cuda")
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.zeros(q.shape, dtype=out_dtype, device=dev)
    cap = sel_cap or max(1, N // w.page_size + 1)
    rc, ranges = epsp.chunk_plan(N, 0, w.n_ubatch)
    assert rc == 0
    sels, cnts = [], []
    for a, b in ranges:
        _, nb = ctx.query_blocks(b - a)
        sel = torch.full((nb, w.n_head_kv, cap), -1, dtype=torch.int32, device=dev)
        cnt = torch.zeros((nb, w.n_head_kv), dtype=torch.int32, device=dev)
        ctx.check(ctx.attend_layer(layer, qd[a:b], kd, vd, b, b - a, out[a:b], sel, cnt, cap))
        sels.append(sel)
        cnts.append(cnt)
        if pooled is not None:
            pp = torch.full((nb, w.n_head_kv, cap), -1, dtype=torch.int32, device=dev)
            pc = torch.full((nb, w.n_head_kv), -1, dtype=torch.int32, device=dev)
            ctx.check(ctx.pooled_pages(pp, pc, cap))
            pooled.append((pp, pc))
    torch.cuda.synchronize()
    ctx.check(ctx.sync_status())
    sel = torch.cat(sels).cpu().numpy()
    cnt = torch.cat(cnts).cpu().numpy()
    return out, sel, cnt


def assert_selection_equal(sel_g, cnt_g, sel_o, cnt_o):
    assert cnt_g.shape == cnt_o.shape, (cnt_g.shape, cnt_o.shape)
    assert np.array_equal(cnt_g, cnt_o), f"counts differ:\n{cnt_g}\n{cnt_o}"
    for b in range(cnt_o.shape[0]):
        for h in range(cnt_o.shape[1]):
            n = cnt_o[b, h]
            assert np.array_equal(sel_g[b, h, :n], sel_o[b, h, :n]), (b, h, sel_g[b, h, :n], sel_o[b, h, :n])


def attn_errors(out_gpu: torch.Tensor, out_ref: np.ndarray, rows=None):
    o = out_gpu.float().cpu().numpy().astype(np.float64)
    if rows is not None:
        o = o[rows]
        out_ref = out_ref[rows]
    err = np.abs(o - out_ref)
    return float(err.max()), float(err.mean())


def torch_dense_reference(q, k, v, kq_scale=None):
    """Plain fp32 causal GQA attention (torch), the dense-path reference."""
    qf, kf, vf = q.float(), k.float(), v.float()
    N, Hq, d = qf.shape
    Hkv = kf.shape[1]
    G = Hq // Hkv
    scale = kq_scale or 1.0 / np.sqrt(d)
    kf = kf.repeat_interleave(G, dim=1)
    vf = vf.repeat_interleave(G, dim=1)
    s = torch.einsum("thd,shd->hts", qf, kf) * scale
    mask = torch.ones(N, N, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hts,shd->thd", p, vf)
