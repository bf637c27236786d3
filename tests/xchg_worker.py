"""One rank of the multi-GPU exchange test (run by tests/test_gpu_xchg_multi.py
under torch.distributed.run, one process per GPU).

Each rank owns a slice of the KV heads, maps every rank's exchange buffer over
CUDA IPC, and for three layers runs ep_sp_select_layer +
ep_sp_attend_rows_xchg (slots rotating) + ep_sp_xchg_wait -- or, with the
argument `balanced`, a whole-model context per rank attending its
ep_sp_balance_ctas range through ep_sp_select_heads + ep_sp_attend_ctas_xchg;
its slot must then equal, bit for bit, ep_sp_attend_layer of one context over
all heads run on the same GPU.  With `multicast` the balanced run's exchange
buffers are one symmetric-memory allocation per rank, attached with
ep_sp_xchg_attach_buffers together with its NVLink multicast address, so the
attention epilogue stores each tile once through the switch (the run prints
`multicast unsupported` and exits 0 when the GPUs offer no multicast object).
Exit code 0 when every rank matched.
"""
from __future__ import annotations

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "edge-prefill_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import epsp  # noqa: E402
import workloads as W  # noqa: E402

W_X = W.Workload("xm", 8192, 3, 32, 8, 128, W.BF16, 8192, 128, 8, 512, per_kv_head=1, max_gather_rows=0,
                 q_subblock=2048)


def make(w, kv0, kv1, dev):
    G = w.n_head // w.n_head_kv
    c = epsp.Context(n_layer=w.n_layer, n_head=(kv1 - kv0) * G, n_head_kv=kv1 - kv0, head_dim=w.head_dim,
                     dtype=w.dtype, out_dtype=w.dtype, max_ctx=w.n_tokens, page_size=w.page_size, device=dev,
                     kv_head_offset=kv0, n_head_kv_total=w.n_head_kv)
    c.check(c.set_ext(1, w.q_subblock, 0))
    c.check(c.set_qg_bound(1, w.top_k, w.local_pages, 0))
    c.set_prefill_mode(True)
    return c


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    mode = sys.argv[1] if len(sys.argv) > 1 else "heads"
    balanced = mode in ("balanced", "multicast")
    w, N = W_X, W_X.n_tokens
    kv0, kv1 = (0, w.n_head_kv) if balanced else W.shard_kv_heads(w.n_head_kv, world, rank)
    ctx = make(w, kv0, kv1, local)
    full = make(w, 0, w.n_head_kv, local)
    symm_buf = None
    attach_rc = epsp.OK
    if mode == "multicast":
        import torch.distributed._symmetric_memory as symm

        from torch._C._autograd import DeviceType

        buf = symm.empty(ctx.xchg_bytes(N, 2), dtype=torch.uint8, device="cuda")
        handle = symm.rendezvous(buf, dist.group.WORLD)
        if not (handle.has_multicast_support(DeviceType.CUDA, local) and handle.multicast_ptr):
            torch.cuda.synchronize()
            dist.barrier()
            del handle, buf
            ctx.close()
            full.close()
            dist.barrier()
            if rank == 0:
                print("multicast unsupported", flush=True)
            dist.destroy_process_group()
            sys.exit(0)
        symm_buf = (buf, handle)
        try:
            # the tensor sits at handle.offset in every rank's allocation and in the multicast range
            bases = [p + handle.offset for p in handle.buffer_ptrs]
            if bases[rank] != buf.data_ptr():
                raise RuntimeError("symmetric buffer address mismatch")
            attach_rc = ctx.xchg_attach_buffers(N, 2, rank, bases, handle.multicast_ptr + handle.offset)
        except Exception as e:
            print(f"rank {rank}: {e}", flush=True)
            attach_rc = epsp.INVALID_ARGUMENT
    else:
        base, handle = ctx.xchg_alloc(N, 2)
        handles = [None] * world
        dist.all_gather_object(handles, handle)
        bases = [base if r == rank else ctx.xchg_open(handles[r]) for r in range(world)]
        ctx.check(ctx.xchg_attach(rank, bases))
    torch.cuda.synchronize()
    dist.barrier()
    # every rank learns whether every rank attached before any kernel stores through the mappings
    att = torch.tensor([1 if attach_rc == epsp.OK else 0], device="cuda")
    dist.all_reduce(att, op=dist.ReduceOp.MIN)
    ok = bool(att.item())
    if not ok:
        print(f"rank {rank}: attach rc {attach_rc} ({ctx.last_error()})", flush=True)
    try:
        if ok:
            ok = run_layers(ctx, full, w, N, rank, world, kv0, kv1, balanced)
    except Exception as e:  # keep every rank alive until the collective teardown below
        print(f"rank {rank}: {e}", flush=True)
        ok = False
    torch.cuda.synchronize()
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"exchange over {world} GPUs ({mode}): {'match' if flag.item() else 'MISMATCH'}", flush=True)
    dist.barrier()
    ctx.close()
    full.close()
    if symm_buf is not None:
        # every rank's stores through the multicast address are complete before any rank unmaps
        torch.cuda.synchronize()
        dist.barrier()
        del symm_buf
        torch.cuda.synchronize()
        dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flag.item() else 1)


def run_layers(ctx, full, w, N, rank, world, kv0, kv1, balanced):
    ok = True
    for l in range(w.n_layer):
        q, k, v = (t.cuda() for t in W.gen_layer(w, l))
        ref = torch.empty_like(q)
        full.check(full.attend_layer(l, q, k, v, N, N, ref))
        if balanced:
            per_head = ctx.attention_grid(N)
            cuts = ctx.balance_ctas(l, N, N, world)
            c0, c1 = cuts[rank], cuts[rank + 1]
            if c1 > c0:
                ctx.check(ctx.select_heads(l, q, k, v, N, N, c0 // per_head, (c1 - 1) // per_head + 1))
                ctx.check(ctx.attend_ctas_xchg(l, N, N, c0, c1, l % 2))
        else:
            qs, ks, vs = (t.cuda() for t in W.gen_layer(w, l, head_slice=(kv0, kv1)))
            ctx.check(ctx.select_layer(l, qs, ks, vs, N, N))
            ctx.check(ctx.attend_rows_xchg(l, N, N, 0, N, l % 2))
        ctx.check(ctx.xchg_wait(l % 2, N))
        torch.cuda.synchronize()
        rc = ctx.sync_status()
        got = epsp.device_view(ctx.xchg_slot(l % 2), (N, w.n_head, w.head_dim), w.dtype)
        same = rc == epsp.OK and torch.equal(got, ref)
        if not same:
            bad = (got != ref).reshape(N, w.n_head, -1).any(-1).nonzero()[:8].tolist()
            print(f"rank {rank} layer {l}: rc {rc} ({ctx.last_error()}), first differing (row, head): {bad}",
                  flush=True)
        ok = ok and same
    return ok


if __name__ == "__main__":
    main()
