"""Head-parallel partition over 2 ranks (gloo, CPU): every rank gates and
attends only its KV-head slice (with its rows of the global k-matrix), the
outputs are all-gathered, and the result must equal the single-process
computation over all heads -- selection lists bit-exact, attention identical.
The ranks compute with the oracle (there is no GPU here); the GPU path takes
the same slices through ep_sp_config.kv_head_offset / n_head_kv_total."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import workloads as W

W_CASE = W.Workload("mr", 1024, 2, 16, 4, 64, W.BF16, 256, 64, 3, 128, q_subblock=128, seed=21)
K_MATRIX = [[2, 3, -1, 4], [1, 4, 2, 3]]
ROWS = np.arange(5, 1024, 41, dtype=np.int32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_slice(layer, kv0, kv1):
    import oracle
    from gpu_util import to_np

    w = W_CASE
    q, k, v = W.gen_layer(w, layer, head_slice=(kv0, kv1))
    G = w.n_head // w.n_head_kv
    p = oracle.params(n_head=(kv1 - kv0) * G, n_head_kv=kv1 - kv0, head_dim=w.head_dim, page_size=w.page_size,
                      sel_pages=w.top_k, local_pages=w.local_pages, shared=0, q_subblock=w.q_subblock,
                      max_gather_rows=0)
    out, sel, cnt, _ = oracle.prefill_layer(p, to_np(q), to_np(k), to_np(v), w.dtype, n_ubatch=w.n_ubatch,
                                            k_budget=np.array(K_MATRIX[layer][kv0:kv1], np.int32), rows=ROWS,
                                            sel_cap=w.n_tokens // w.page_size + 1)
    return out[ROWS], sel, cnt


def _worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.join(os.path.dirname(here), "edge-prefill_b200"),
              os.path.join(os.path.dirname(here), "oracle")):
        sys.path.insert(0, p)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kv0, kv1 = W.shard_kv_heads(W_CASE.n_head_kv, world, rank)
        res = []
        for layer in range(W_CASE.n_layer):
            out, sel, cnt = _oracle_slice(layer, kv0, kv1)
            gathered = [torch.zeros_like(torch.from_numpy(out)) for _ in range(world)]
            dist.all_gather(gathered, torch.from_numpy(out))
            full = torch.cat(gathered, dim=1).numpy()  # [rows][Hq][d], heads rank-major
            sels = [torch.zeros_like(torch.from_numpy(sel)) for _ in range(world)]
            dist.all_gather(sels, torch.from_numpy(sel))
            cnts = [torch.zeros_like(torch.from_numpy(cnt)) for _ in range(world)]
            dist.all_gather(cnts, torch.from_numpy(cnt))
            res.append((full, torch.cat(sels, 1).numpy(), torch.cat(cnts, 1).numpy()))
        if rank == 0:
            q_out.put(res)
    finally:
        dist.destroy_process_group()


def test_head_parallel_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for layer in range(W_CASE.n_layer):
        full, sel, cnt = res[layer]
        ref_out, ref_sel, ref_cnt = _oracle_slice(layer, 0, W_CASE.n_head_kv)
        assert np.array_equal(cnt, ref_cnt)
        for b in range(cnt.shape[0]):
            for h in range(cnt.shape[1]):
                assert np.array_equal(sel[b, h, :cnt[b, h]], ref_sel[b, h, :cnt[b, h]])
        assert np.array_equal(full, ref_out)
        assert cnt.sum() > 0


def test_shard_kv_heads():
    assert [W.shard_kv_heads(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        W.shard_kv_heads(4, 8, 0)


# --------------------------------------------------- balanced split (gloo, CPU)
def _balanced_worker(rank, world, port, q_out):
    """Each rank takes its ep_sp_balance_ctas range of every layer's head-major
    CTA grid (a whole-prompt call gated per q_subblock), computes the oracle
    output of the (row, query head) pairs its CTAs own over the KV heads its
    range touches, and the ranks' full-width buffers are summed: every pair
    must be owned exactly once and the sum must equal the single-process
    oracle over all heads."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.join(os.path.dirname(here), "edge-prefill_b200"),
              os.path.join(os.path.dirname(here), "oracle")):
        sys.path.insert(0, p)
    import epsp

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = W_CASE
        G, T, N = w.n_head // w.n_head_kv, 128 // (w.n_head // w.n_head_kv), w.n_tokens
        c = epsp.Context(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                         dtype=w.dtype, out_dtype=w.dtype, max_ctx=N, page_size=w.page_size, device=0)
        c.check(c.set_ext(1, w.q_subblock, 0))
        c.check(c.set_k_matrix([x for row in K_MATRIX for x in row]))
        c.check(c.set_qg_bound(1, w.top_k, w.local_pages, 0))
        c.set_prefill_mode(True)
        per_head = c.attention_grid(N)
        tpb = per_head // (N // w.q_subblock)
        res = []
        for layer in range(w.n_layer):
            cuts = c.balance_ctas(layer, N, N, world)
            all_cuts = [None] * world
            dist.all_gather_object(all_cuts, cuts)
            c0, c1 = cuts[rank], cuts[rank + 1]
            h0, h1 = c0 // per_head, (c1 - 1) // per_head + 1
            out, _, _ = _oracle_slice(layer, h0, h1)  # [ROWS][(h1-h0)*G][d] for this rank's KV heads
            mine = np.zeros((len(ROWS), w.n_head, w.head_dim), np.float64)
            owned = np.zeros((len(ROWS), w.n_head), np.int64)
            for i, r in enumerate(ROWS):
                blk, rem = divmod(int(r), w.q_subblock)
                for h in range(h0, h1):
                    cid = h * per_head + blk * tpb + rem // (2 * T)
                    if c0 <= cid < c1:
                        mine[i, h * G:(h + 1) * G] = out[i, (h - h0) * G:(h - h0 + 1) * G]
                        owned[i, h * G:(h + 1) * G] = 1
            tm, to = torch.from_numpy(mine), torch.from_numpy(owned)
            dist.all_reduce(tm)
            dist.all_reduce(to)
            res.append((all_cuts, tm.numpy(), to.numpy()))
        if rank == 0:
            q_out.put(res)
    finally:
        dist.destroy_process_group()


def test_balanced_split_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_balanced_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for layer in range(W_CASE.n_layer):
        all_cuts, full, owned = res[layer]
        assert all_cuts[0] == all_cuts[1]            # every rank computes the same cuts
        assert all_cuts[0][0] == 0 and all_cuts[0] == sorted(all_cuts[0])
        assert np.all(owned == 1)                    # every (row, head) owned exactly once
        ref_out, _, _ = _oracle_slice(layer, 0, W_CASE.n_head_kv)
        assert np.array_equal(full, ref_out.astype(np.float64))
