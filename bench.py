#!/usr/bin/env python
"""Benchmark of the page-gated sparse prefill attention path.

Metric: sparse-prefill attention tokens/s at 64K context (workload c4:
65536 tokens, 32 layers of Llama-3-8B attention -- 32 query / 8 KV heads,
head_dim 128, bf16 -- ubatch 4096, page 128, per-(layer, KV head) top-k from
{32, 64, 128} halved every 8 layers, sink page + 1024-row local window, and
FFN-skip compaction of 85% of the rows with hidden 4096), plus the fraction of
the roofline of the dominant kernel (K3, tensor-bound).

One step = the whole prefill, layer by layer: K1 page sums and K2 score + top-k
for every gating block of the ubatch length (ep_sp_select_layer), K3 sparse
attention of all 65536 query rows (ep_sp_attend_rows, one launch), then the
FFN-skip compaction and the scatter-add of the FFN output (the FFN GEMMs
themselves are outside the path; the compacted rows stand in for their output).
The selections, kept sets and arithmetic are those of the reference's
per-ubatch order, which is also timed and reported (`ubatch_schedule`).
With --gpus N > 1 (torchrun, one process per GPU) each rank attends its
cost-balanced range of the layer's head-major K3 grid (--partition balanced,
the default) or its KV-head slice (--partition heads), and K3's epilogue stores
every output tile into all ranks' full-width buffers over NVLink (the fused
exchange; --exchange nccl all-gathers per chunk instead); each rank compacts its
1/N share of the FFN rows.

  value  device-resident inputs, CUDA events on the compute stream, max over ranks
  e2e    through the same C ABI with host buffers: pinned H2D copies of the step's
         inputs and D2H of its outputs inside the timed region, overlapped with
         compute on separate streams
--impl reference times the CPU oracle (the restatement of the reference's
algorithm; the reference's own ggml path cannot be built: llama.cpp is not
vendored) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "edge-prefill_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import workloads as W  # noqa: E402

METRIC = "sparse-prefill attention tokens/s per GPU at 64K ctx; % of roofline at 1/2/4/8 B200"
UNIT = "tokens/s"


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out = ""
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                mx.append(float(row[2]))
            except ValueError:
                continue
            for n, v in zip(names, row[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------------- our arm
class Runner:
    def __init__(self, w: W.Workload, world: int, rank: int, local: int, exchange: str = "peer",
                 partition: str = "balanced", multicast: str = "off"):
        import epsp

        self.epsp = epsp
        self.multicast = multicast if world > 1 else "off"
        self.symm = []        # symmetric-memory exchange buffers (kept alive until close())
        self.mc_used = False  # an exchange stores through an NVLink multicast address
        self.w, self.world, self.rank = w, world, rank
        self.dev = torch.device("cuda", local)
        # a KV-head slice per rank exists only when the heads split evenly; the
        # balanced partition needs none (c5: 4 KV heads over 8 GPUs)
        self.sliceable = w.n_head_kv % world == 0
        self.kv0, self.kv1 = W.shard_kv_heads(w.n_head_kv, world, rank) if self.sliceable else (0, w.n_head_kv)
        self.hkv = self.kv1 - self.kv0
        self.G = w.n_head // w.n_head_kv
        self.hq = self.hkv * self.G
        self.U = w.n_ubatch
        self.n_ub = (w.n_tokens + self.U - 1) // self.U
        self.tdt = W.TORCH_DTYPE[w.dtype]
        km = w.k_matrix()
        if km is None and w.top_k > 128:
            km = [[w.top_k] * w.n_head_kv for _ in range(w.n_layer)]
        self.k_matrix = km
        self.ctx = None
        if self.sliceable:
            self.ctx = epsp.Context(n_layer=w.n_layer, n_head=self.hq, n_head_kv=self.hkv, head_dim=w.head_dim,
                                    dtype=w.dtype, out_dtype=w.dtype, max_ctx=w.n_tokens, page_size=w.page_size,
                                    device=local, kv_head_offset=self.kv0, n_head_kv_total=w.n_head_kv)
            c = self.ctx
            c.check(c.reserve())
            c.check(c.set_qg_bound(1, min(w.top_k, 128), w.local_pages, 0))
            c.set_prefill_mode(True)
        # FFN rows this rank compacts within each ubatch
        self.ffn = w.ffn_hidden > 0
        self.rows_per_rank = self.U // world
        # layer schedule: one K3 launch per layer on one GPU; with NCCL, 4 chunks
        # whose all-gathers overlap the next chunk
        self.chunks = 4 if world > 1 else 1
        self.exchange = exchange if world > 1 else None
        # balanced: the layer schedule runs on a context over every KV head, each
        # rank attending its cost-balanced range of the head-major CTA grid
        self.partition = "balanced" if (partition == "balanced" and self.exchange == "peer") else "heads"
        if not self.sliceable and self.partition != "balanced":
            raise SystemExit(f"{w.n_head_kv} KV heads do not split over {world} ranks: use the balanced partition")
        self.ctxs = [self.ctx] if self.ctx is not None else []
        self.bctx = None
        if self.partition == "balanced":
            b = epsp.Context(n_layer=w.n_layer, n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim,
                             dtype=w.dtype, out_dtype=w.dtype, max_ctx=w.n_tokens, page_size=w.page_size,
                             device=local)
            b.check(b.reserve())
            b.check(b.set_qg_bound(1, min(w.top_k, 128), w.local_pages, 0))
            b.set_prefill_mode(True)
            b.check(b.set_ext(w.per_kv_head, w.q_subblock or self.U, w.max_gather_rows))
            if km is not None:
                b.check(b.set_k_matrix([x for row in km for x in row]))
            self.bctx = b
            self.ctxs.append(b)
            N = w.n_tokens
            self.per_head = b.attention_grid(N)
            self.cuts = [b.balance_ctas(l, N, N, world) for l in range(w.n_layer)]
        self.fctx = self.ctx if self.ctx is not None else self.bctx  # the FFN calls' context
        self.schedule = None
        self.set_schedule("layer")

    def set_schedule(self, mode):
        """ubatch: one call per (ubatch, layer), gating block = ubatch (the
        reference's chunked prefill order).  layer: one call per layer over the
        whole prompt with gating blocks of the ubatch length (q_subblock), i.e.
        the same blocks, kept sets and arithmetic, 16x fewer launches."""
        w = self.w
        if self.ctx is None:  # balanced partition without head slices: the layer schedule only
            self.schedule = "layer"
            return
        qsb = w.q_subblock if (mode == "ubatch" or w.q_subblock) else self.U
        self.ctx.check(self.ctx.set_ext(w.per_kv_head, qsb, w.max_gather_rows))
        if self.k_matrix is not None:
            self.ctx.check(self.ctx.set_k_matrix([x for row in self.k_matrix for x in row]))
        self.schedule = mode

    def alloc_resident(self):
        w = self.w
        self.Q, self.K, self.V, self.O = [], [], [], []
        self.Qf, self.Kf, self.Vf = [], [], []
        for l in range(w.n_layer):
            if self.ctx is not None:
                q, k, v = W.gen_layer(w, l, device=self.dev, head_slice=(self.kv0, self.kv1))
                self.Q.append(q)
                self.K.append(k)
                self.V.append(v)
                self.O.append(torch.empty_like(q))
            if self.partition == "balanced":
                # every head resident on every rank: each rank's CTA range may reach into any head
                q, k, v = W.gen_layer(w, l, device=self.dev)
                self.Qf.append(q)
                self.Kf.append(k)
                self.Vf.append(v)
        if self.exchange == "peer":
            # exchange buffers of full-width rows, mapped on every rank over CUDA IPC,
            # 3 rotating slots (the e2e arm overlaps a slot's host copy with the next
            # layers' exchanges)
            if self.ctx is not None and self.partition != "balanced":
                self.attach_exchange(self.ctx, 3)
            if self.bctx is not None:
                self.attach_exchange(self.bctx, 3)
        if self.world > 1 and self.ctx is not None:
            self.gathered = torch.empty((self.world, self.U, self.hq, w.head_dim), dtype=self.tdt, device=self.dev)
            self.chunk_rows = self.U * ((self.n_ub + self.chunks - 1) // self.chunks)
            self.gbuf = [torch.empty((self.world, self.chunk_rows, self.hq, w.head_dim), dtype=self.tdt,
                                     device=self.dev) for _ in range(self.chunks)]
            self.comm = torch.cuda.Stream()
            self.chunk_ev = [torch.cuda.Event() for _ in range(self.chunks)]
        if self.ffn:
            g = torch.Generator(device=self.dev).manual_seed(w.seed + 5)
            n_rows = self.n_ub * self.rows_per_rank
            self.X = [torch.randn(n_rows, w.ffn_hidden, generator=g, device=self.dev).to(self.tdt)
                      for _ in range(w.n_layer)]
            self.R = [torch.randn(n_rows, w.ffn_hidden, generator=g, device=self.dev).to(self.tdt)
                      for _ in range(w.n_layer)]
            keep = W.ffn_keep_mask(w, device=self.dev)
            # this rank's share of each ubatch's rows, laid out ubatch by ubatch
            idx = torch.cat([torch.arange(u * self.U + self.rank * self.rows_per_rank,
                                          u * self.U + (self.rank + 1) * self.rows_per_rank, device=self.dev)
                             for u in range(self.n_ub)])
            self.keep = keep[idx].contiguous()
            n_all = self.n_ub * self.rows_per_rank  # this rank's rows of the whole prompt
            self.x_kept = torch.empty(n_all, w.ffn_hidden, dtype=self.tdt, device=self.dev)
            self.row_ids = torch.empty(n_all, dtype=torch.int32, device=self.dev)
            self.n_keep = torch.empty(1, dtype=torch.int32, device=self.dev)

    def attach_exchange(self, c, n_slots):
        import torch.distributed as dist

        if self.multicast != "off":
            # one symmetric-memory allocation per rank; with a multicast object
            # over them the attention epilogue stores each tile once
            import torch.distributed._symmetric_memory as symm

            from torch._C._autograd import DeviceType

            buf = symm.empty(c.xchg_bytes(self.w.n_tokens, n_slots), dtype=torch.uint8, device=self.dev)
            h = symm.rendezvous(buf, dist.group.WORLD)
            self.symm.append((buf, h))
            try:
                mc_ok = h.has_multicast_support(DeviceType.CUDA, self.dev.index) and h.multicast_ptr != 0
                if not mc_ok and self.multicast == "on":
                    raise RuntimeError("--multicast on: the GPUs offer no NVLink multicast object")
                # the tensor sits at h.offset in every rank's allocation and in the multicast range
                bases = [p + h.offset for p in h.buffer_ptrs]
                if bases[self.rank] != buf.data_ptr():
                    raise RuntimeError("symmetric buffer address mismatch")
                mc = h.multicast_ptr + h.offset if mc_ok else 0
                rc = c.xchg_attach_buffers(self.w.n_tokens, n_slots, self.rank, bases, mc or None)
            except Exception as e:
                print(f"rank {self.rank}: {e}", file=sys.stderr, flush=True)
                rc, mc = self.epsp.INVALID_ARGUMENT, 0
            # all ranks fail together (and tear down in step) if any rank could not attach
            ok = torch.tensor([1 if rc == self.epsp.OK else 0], device=self.dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if not ok.item():
                raise RuntimeError(f"exchange attach failed on some rank (here rc {rc}: {c.last_error()})")
            self.mc_used = self.mc_used or bool(mc)
            torch.cuda.synchronize()
            dist.barrier()
            return
        base, handle = c.xchg_alloc(self.w.n_tokens, n_slots)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle)
        bases = [base if r == self.rank else c.xchg_open(handles[r]) for r in range(self.world)]
        c.check(c.xchg_attach(self.rank, bases))
        torch.cuda.synchronize()
        dist.barrier()

    def close(self):
        """Every rank's work (and every store into a peer's buffer) completes
        before any rank frees its contexts or unmaps an exchange buffer."""
        torch.cuda.synchronize()
        barrier(self.world)
        for x in self.ctxs:
            x.close()
        self.ctxs = []
        if self.symm:
            torch.cuda.synchronize()
            barrier(self.world)
            self.symm.clear()
            torch.cuda.synchronize()
            barrier(self.world)

    def layer_call(self, l, u, q, out):
        """Attention (+ all-gather) (+ FFN compaction/scatter) of one (ubatch, layer)."""
        c, U = self.ctx, self.U
        a, b = u * U, min((u + 1) * U, self.w.n_tokens)
        rc = c.attend_layer(l, q, self.K[l], self.V[l], b, b - a, out)
        if rc:
            c.check(rc)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.gathered.view(-1), out.reshape(-1))

    def ffn_call(self, l, x_rows, keep_rows, r_rows, n=None):
        c = self.fctx
        n, hid = n or self.rows_per_rank, self.w.ffn_hidden
        rc = c.ffn_compact(l, x_rows, keep_rows, n, hid, self.x_kept, self.row_ids, self.n_keep)
        if rc:
            c.check(rc)
        rc = c.ffn_scatter(l, self.x_kept, r_rows, self.row_ids, self.n_keep, n, hid)
        if rc:
            c.check(rc)

    def step(self):
        if self.schedule == "layer":
            return self.step_layer()
        return self.step_ubatch()

    def step_layer(self):
        """Per layer: K1 + K2 for the whole prompt (gating blocks of the ubatch
        length), then K3.  One GPU: K3 in chunks of gating blocks.  N > 1 with
        the peer exchange: one K3 launch per rank whose epilogue stores the
        output tiles into every rank's full-width buffer, then the bounded
        wait for the other ranks' tiles -- over this rank's cost-balanced CTA
        range of a whole-model context (balanced) or over its KV-head slice
        (heads).  N > 1 with NCCL: each chunk's output is all-gathered on a
        comm stream while the next chunk is attended.  The layer completes
        before its FFN rows are compacted and the next layer starts."""
        c, N = self.ctx, self.w.n_tokens
        for x in self.ctxs:
            x.reset()
        comp = torch.cuda.current_stream()
        chunk_rows = self.U * ((self.n_ub + self.chunks - 1) // self.chunks)
        n_all = self.n_ub * self.rows_per_rank
        for l in range(self.w.n_layer):
            if self.partition == "balanced":
                b = self.bctx
                r0, r1 = self.cuts[l][self.rank], self.cuts[l][self.rank + 1]
                if r1 > r0:
                    rc = b.select_heads(l, self.Qf[l], self.Kf[l], self.Vf[l], N, N, r0 // self.per_head,
                                        (r1 - 1) // self.per_head + 1)
                    if rc:
                        b.check(rc)
                    rc = b.attend_ctas_xchg(l, N, N, r0, r1, l % 3)
                    if rc:
                        b.check(rc)
                rc = b.xchg_wait(l % 3, N)
                if rc:
                    b.check(rc)
            else:
                rc = c.select_layer(l, self.Q[l], self.K[l], self.V[l], N, N)
                if rc:
                    c.check(rc)
                if self.exchange == "peer":
                    rc = c.attend_rows_xchg(l, N, N, 0, N, l % 2)
                    if rc:
                        c.check(rc)
                    rc = c.xchg_wait(l % 2, N)
                    if rc:
                        c.check(rc)
                else:
                    for ci, r0 in enumerate(range(0, N, chunk_rows)):
                        r1 = min(N, r0 + chunk_rows)
                        rc = c.attend_rows(l, N, N, r0, r1, self.O[l])
                        if rc:
                            c.check(rc)
                        if self.world > 1:
                            import torch.distributed as dist

                            self.chunk_ev[ci].record(comp)
                            with torch.cuda.stream(self.comm):
                                self.comm.wait_event(self.chunk_ev[ci])
                                src = self.O[l][r0:r1].reshape(-1)
                                dist.all_gather_into_tensor(self.gbuf[ci].view(-1)[: self.world * src.numel()],
                                                            src)
                    if self.world > 1:
                        comp.wait_stream(self.comm)
            if self.ffn:
                self.ffn_call(l, self.X[l], self.keep, self.R[l], n=n_all)

    def step_ubatch(self):
        self.ctx.reset()
        U, n = self.U, self.rows_per_rank
        for u in range(self.n_ub):
            a, b = u * U, min((u + 1) * U, self.w.n_tokens)
            for l in range(self.w.n_layer):
                self.layer_call(l, u, self.Q[l][a:b], self.O[l][a:b])
                if self.ffn:
                    self.ffn_call(l, self.X[l][u * n:(u + 1) * n], self.keep[u * n:(u + 1) * n],
                                  self.R[l][u * n:(u + 1) * n])

    def work(self):
        """Algorithmic K1/K2/K3/K4 work of one step (this rank)."""
        tot = np.zeros(6)
        import ctypes

        arr = (ctypes.c_double * 6)()
        calls = ([(self.w.n_tokens, self.w.n_tokens)] if self.schedule == "layer" else
                 [(min((u + 1) * self.U, self.w.n_tokens), min((u + 1) * self.U, self.w.n_tokens) - u * self.U)
                  for u in range(self.n_ub)])
        if self.schedule == "layer" and self.partition == "balanced":
            # this rank's CTA range; K1/K2 over the KV heads the range touches
            N, b = self.w.n_tokens, self.bctx
            for l in range(self.w.n_layer):
                r0, r1 = self.cuts[l][self.rank], self.cuts[l][self.rank + 1]
                rc = self.epsp.lib.ep_sp_layer_work(b.h, l, N, N, arr)
                assert rc == 0
                full = np.frombuffer(arr, dtype=np.float64).copy()
                heads = ((r1 - 1) // self.per_head + 1 - r0 // self.per_head) if r1 > r0 else 0
                frac = heads / self.w.n_head_kv
                k3 = b.cta_work(l, N, N, r0, r1)
                tot += np.array([full[0] * frac, full[1] * frac, full[2] * frac, k3[0], k3[1], k3[2]])
        else:
            for kv_len, n_tok in calls:
                for l in range(self.w.n_layer):
                    rc = self.epsp.lib.ep_sp_layer_work(self.ctx.h, l, kv_len, n_tok, arr)
                    assert rc == 0
                    tot += np.frombuffer(arr, dtype=np.float64)
        k4 = 0.0
        if self.ffn:
            esz = torch.finfo(self.tdt).bits // 8
            keep_rows = float(self.keep.sum().item())
            # compaction: read + write kept rows, read mask; scatter: read ffn rows,
            # read + write residual rows; row ids written and read twice
            k4 = (2 * keep_rows * self.w.ffn_hidden * esz + self.keep.numel()
                  + 3 * keep_rows * self.w.ffn_hidden * esz + 12 * keep_rows) * self.w.n_layer
        return {"k1_bytes": tot[0], "k2_bytes": tot[1], "k2_flops": tot[2], "k3_flops": tot[3], "k3_bytes": tot[4],
                "k3_keys": tot[5], "k4_bytes": k4}


def run_ours(args, w, world, rank, local):
    import epsp

    r = Runner(w, world, rank, local, exchange=args.exchange, partition=args.partition, multicast=args.multicast)
    try:
        run_runner(r, args, w, world, rank, local)
    finally:
        r.close()


def run_runner(r, args, w, world, rank, local):
    import epsp

    tiles = args.attn_tiles or 2
    for x in r.ctxs:
        x.check(x.set_attn_tiles(tiles))
    r.alloc_resident()
    if r.bctx is not None:
        # after the exchange is attached: the cuts' cost model depends on how the epilogue stores
        r.cuts = [r.bctx.balance_ctas(l, w.n_tokens, w.n_tokens, world) for l in range(w.n_layer)]
        r.per_head = r.bctx.attention_grid(w.n_tokens)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        r.step()
    torch.cuda.synchronize()
    for x in r.ctxs:
        x.check(x.sync_status())

    sampler = ClockSampler(local)
    for x in r.ctxs:
        x.check(epsp.lib.ep_sp_profile_enable(x.h, 1))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    # NVTX range over the timed steps: `ncu --nvtx --nvtx-include ep_sp_timed/`
    # captures exactly these launches
    torch.cuda.nvtx.range_push("ep_sp_timed")
    ev0.record(stream)
    for _ in range(args.steps):
        r.step()
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    ms_local = ev0.elapsed_time(ev1)
    import ctypes

    kms, kl = [0.0] * epsp.NUM_KERNELS, [0] * epsp.NUM_KERNELS
    for x in r.ctxs:
        xm = (ctypes.c_double * epsp.NUM_KERNELS)()
        xl = (ctypes.c_int64 * epsp.NUM_KERNELS)()
        x.check(epsp.lib.ep_sp_profile_read(x.h, xm, xl))
        x.check(epsp.lib.ep_sp_profile_enable(x.h, 0))
        x.check(x.sync_status())
        kms = [a + b for a, b in zip(kms, xm)]
        kl = [a + b for a, b in zip(kl, xl)]
    ms = max_over_ranks(ms_local, world)
    ms_step = ms / args.steps
    value = w.n_tokens * args.steps / (ms / 1e3)
    per_rank = None
    if world > 1:
        import torch.distributed as dist

        mine = torch.tensor([ms_local / args.steps, kms[2] / args.steps, kms[5] / args.steps],
                            dtype=torch.float64, device="cuda")
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        allr = [x.tolist() for x in allr]
        per_rank = {"step_ms": [round(x[0], 3) for x in allr], "k3_ms": [round(x[1], 3) for x in allr],
                    "exchange_ms": [round(x[2], 3) for x in allr]}

    work = r.work()
    peaks = load_peaks()
    k3_ms = kms[2] / args.steps
    k3_launches = kl[2] / args.steps
    k3_flops_launch = work["k3_flops"] / k3_launches
    achieved_tf = k3_flops_launch / (k3_ms / k3_launches / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(achieved_tf, 1), "peak": peaks["bf16_tflops_sustained"],
                "unit": "TFLOP/s", "frac": round(achieved_tf / peaks["bf16_tflops_sustained"], 4),
                "traffic": load_traffic(w.name), "kernel": "k3_sparse_attention",
                "peak_kind": f"bf16 sustained ({peaks['source']})",
                "algorithmic_flops_per_launch": k3_flops_launch}
    kernels = {}
    names = epsp.KERNEL_NAMES
    total_kms = sum(kms) or 1.0
    for i, n in enumerate(names):
        kernels[n] = {"ms_per_step": round(kms[i] / args.steps, 3), "launches_per_step": kl[i] / args.steps,
                      "share": round(kms[i] / total_kms, 4)}
    if kms[0] > 0:
        kernels["k1_pool_pages"]["hbm_gbs"] = round(work["k1_bytes"] / (kms[0] / args.steps / 1e3) / 1e9, 1)
    if kms[1] > 0:
        kernels["k2_select_pages"]["hbm_gbs"] = round(work["k2_bytes"] / (kms[1] / args.steps / 1e3) / 1e9, 1)
        kernels["k2_select_pages"]["note"] = ("algorithmic bytes (page sums of every scored page, the gating "
                                              "query, the lists) over event time; the page sums are read from L2 "
                                              "when K1 has just written them")
    if kms[3] + kms[4] > 0:
        kernels["k4_compact"]["hbm_gbs_k4"] = round(work["k4_bytes"] / ((kms[3] + kms[4]) / args.steps / 1e3) / 1e9, 1)
    launches = int(round(sum(kl) / args.steps)) * args.steps

    # ------------------------------------------- reference (ubatch) order
    if r.ctx is not None:
        r.set_schedule("ubatch")
        for _ in range(2):
            r.step()
        barrier(world)
        torch.cuda.synchronize()
        u0e, u1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        u0e.record(stream)
        for _ in range(args.steps):
            r.step()
        u1e.record(stream)
        torch.cuda.synchronize()
        ub_ms = max_over_ranks(u0e.elapsed_time(u1e), world) / args.steps
        ubatch_schedule = {"value": round(w.n_tokens / (ub_ms / 1e3), 1), "ms_per_step": round(ub_ms, 3),
                           "order": "one ep_sp_attend_layer call per (ubatch, layer), gating block = ubatch, "
                                    "serialized all-gather per call (the reference's chunked-prefill order)"}
        r.ctx.check(r.ctx.sync_status())
    else:
        ubatch_schedule = {"skipped": f"{w.n_head_kv} KV heads do not split over {world} ranks; the per-ubatch "
                                      "order runs on KV-head slices"}

    # ------------------------------------------------------------ e2e arm
    if r.partition == "balanced":
        e2e = run_e2e_balanced(r, args, world)
    elif r.exchange == "peer":
        e2e = run_e2e_layers(r, args, world)
    else:
        e2e = run_e2e(r, args, world)

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": {W.BF16: "bf16", W.F16: "f16", W.F32: "f32"}[w.dtype],
        "data": "synthetic (seeded; no dataset or checkpoint)",
        "config": config_of(w, world, r.partition == "balanced"),
        "per_gpu_value": round(value / world, 1),
        "schedule": schedule_text(r, world),
        "ubatch_schedule": ubatch_schedule,
        "roofline": roofline, "kernels": kernels, "gpu_launches": launches, "clocks": clocks, "e2e": e2e,
        "attn_tiles_per_cta": tiles,
    }
    if world > 1 and r.exchange == "peer":
        line["exchange_stores"] = ("NVLink multicast (multimem.st through symmetric memory)" if r.mc_used
                                   else "one peer store per rank (CUDA IPC mappings)")
    if per_rank:
        line["per_rank"] = per_rank
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, r, budget_s=args.cpu_seconds)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)


def config_of(w: W.Workload, world: int, balanced: bool) -> dict:
    """The workload description both arms print (identical dicts)."""
    return {"workload": f"{w.name}: {w.n_tokens} tokens x {w.n_layer} layers, {w.n_head}q/{w.n_head_kv}kv "
                        f"heads d{w.head_dim}, ubatch {w.n_ubatch}, page {w.page_size}, "
                        f"top-k {'{32,64,128}>>l/8' if w.adaptive_k else w.top_k}, window {w.local_rows}"
                        + (f", sub-block {w.q_subblock}" if w.q_subblock else "")
                        + (f", FFN compaction keep {w.ffn_keep_frac:.0%} hidden {w.ffn_hidden}" if w.ffn_hidden else ""),
            "tokens": w.n_tokens, "layers": w.n_layer,
            "parallelism": (f"head-parallel x{world}" + (" (cost-balanced CTA ranges)" if balanced else ""))
            if world > 1 else "1 GPU",
            "l2": "inputs larger than L2 (each step streams GBs of Q/K/V/O)"}


def schedule_text(r: Runner, world: int) -> str:
    if world == 1:
        return ("layer: per layer one ep_sp_select_layer (K1+K2, gating blocks of the 4096-row ubatch) and one "
                "ep_sp_attend_rows over the whole prompt (K3)")
    if r.partition == "balanced":
        return ("layer, balanced head-parallel: every rank takes its ep_sp_balance_ctas range of the layer's "
                "head-major K3 grid (equal estimated cost; at most 3 KV heads); per layer ep_sp_select_heads "
                "(K1+K2 of those heads) + one ep_sp_attend_ctas_xchg (K3 whose epilogue stores each output "
                "tile into every rank's full-width buffer over NVLink and counts it there) + ep_sp_xchg_wait "
                "(bounded wait until all rows x heads landed); no separate collective")
    if r.exchange == "peer":
        return ("layer, head-parallel (one KV-head slice per rank): per layer ep_sp_select_layer + one "
                "ep_sp_attend_rows_xchg (K3 storing every tile into all ranks' buffers over NVLink) + "
                "ep_sp_xchg_wait; no separate collective")
    return ("layer, head-parallel (one KV-head slice per rank): per layer ep_sp_select_layer and "
            f"{r.chunks} ep_sp_attend_rows chunks (K3), each all-gathered over NCCL while the next is attended")


def _cudart():
    import ctypes
    import ctypes.util

    for name in ("libcudart.so.12", ctypes.util.find_library("cudart"), "/usr/local/cuda/lib64/libcudart.so"):
        if not name:
            continue
        try:
            lib = ctypes.CDLL(name)
        except OSError:
            continue
        lib.cudaMemcpy2DAsync.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        lib.cudaMemcpy2DAsync.restype = ctypes.c_int
        return lib
    raise RuntimeError("libcudart not found")


def run_e2e_balanced(r: Runner, args, world):
    """N > 1 host-buffer variant of the balanced layer schedule through the
    same C ABI calls: per layer, H2D from pinned memory of only the KV heads
    this rank's CTA range touches (strided 2-D copies of those heads' columns
    of Q, K and V) and of its FFN rows, ep_sp_select_heads +
    ep_sp_attend_ctas_xchg + ep_sp_xchg_wait, the FFN compaction / scatter,
    then D2H of this rank's 1/N of the exchanged full-width output rows and
    of its residual rows.  Two pinned input slots (layers cycled) and three
    exchange slots let the copies overlap the compute."""
    rt = _cudart()
    b, w, N = r.bctx, r.w, r.w.n_tokens
    G, d, Hkv = r.G, w.head_dim, w.n_head_kv
    n_all = r.n_ub * r.rows_per_rank
    hid = w.ffn_hidden
    rows0, rows1 = r.rank * N // world, (r.rank + 1) * N // world
    pin = lambda *sh: torch.empty(*sh, dtype=r.tdt, pin_memory=True)  # noqa: E731
    hq = [pin(*r.Qf[0].shape) for _ in range(2)]
    hk = [pin(*r.Kf[0].shape) for _ in range(2)]
    hv = [pin(*r.Vf[0].shape) for _ in range(2)]
    for i in range(2):
        hq[i].copy_(r.Qf[i % w.n_layer])
        hk[i].copy_(r.Kf[i % w.n_layer])
        hv[i].copy_(r.Vf[i % w.n_layer])
    dq = [torch.empty_like(r.Qf[0]) for _ in range(2)]
    dk = [torch.empty_like(r.Kf[0]) for _ in range(2)]
    dv = [torch.empty_like(r.Vf[0]) for _ in range(2)]
    h_out = [pin(rows1 - rows0, w.n_head, d) for _ in range(3)]
    if r.ffn:
        hx = [pin(n_all, hid) for _ in range(2)]
        hr = [pin(n_all, hid) for _ in range(2)]
        for i in range(2):
            hx[i].copy_(r.X[i % w.n_layer])
            hr[i].copy_(r.R[i % w.n_layer])
        dx = [torch.empty(n_all, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
        dres = [torch.empty(n_all, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
        h_res = [pin(n_all, hid) for _ in range(2)]
    slots = [r.epsp.device_view(b.xchg_slot(i), (N, w.n_head, d), w.dtype) for i in range(3)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(3)]
    ev_out = [torch.cuda.Event() for _ in range(3)]
    esz = dq[0].element_size()
    bytes_in = bytes_out = 0

    def heads_of(l):
        r0, r1 = r.cuts[l][r.rank], r.cuts[l][r.rank + 1]
        if r1 <= r0:
            return r0, r1, 0, 0
        return r0, r1, r0 // r.per_head, (r1 - 1) // r.per_head + 1

    def copy_heads(dst, src, h0, h1, per_head_cols):
        """rows of src's head columns [h0, h1) -> the same columns of dst (pinned -> device)."""
        nonlocal bytes_in
        pitch = src.shape[1] * d * esz
        off = h0 * per_head_cols * d * esz
        width = (h1 - h0) * per_head_cols * d * esz
        rc = rt.cudaMemcpy2DAsync(dst.data_ptr() + off, pitch, src.data_ptr() + off, pitch, width, src.shape[0], 1,
                                  h2d.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"cudaMemcpy2DAsync rc {rc}")
        bytes_in += width * src.shape[0]

    def one_step():
        nonlocal bytes_in, bytes_out
        bytes_in = bytes_out = 0
        b.reset()
        for l in range(w.n_layer):
            bi, sl = l % 2, l % 3
            r0, r1, h0, h1 = heads_of(l)
            with torch.cuda.stream(h2d):
                if l >= 2:
                    h2d.wait_event(ev_used[bi])
                if h1 > h0:
                    copy_heads(dq[bi], hq[bi], h0, h1, G)
                    copy_heads(dk[bi], hk[bi], h0, h1, 1)
                    copy_heads(dv[bi], hv[bi], h0, h1, 1)
                if r.ffn:
                    dx[bi].copy_(hx[bi], non_blocking=True)
                    dres[bi].copy_(hr[bi], non_blocking=True)
                    bytes_in += 2 * dx[bi].numel() * esz
                ev_in[bi].record(h2d)
            comp.wait_event(ev_in[bi])
            if l >= 2:
                comp.wait_event(ev_out[(l + 1) % 3])  # the slot written next is read out
            if r1 > r0:
                b.check(b.select_heads(l, dq[bi], dk[bi], dv[bi], N, N, h0, h1))
                b.check(b.attend_ctas_xchg(l, N, N, r0, r1, sl))
            b.check(b.xchg_wait(sl, N))
            if r.ffn:
                r.ffn_call(l, dx[bi], r.keep, dres[bi], n=n_all)
            ev_used[bi].record(comp)
            ev_done[sl].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_done[sl])
                h_out[sl].copy_(slots[sl][rows0:rows1], non_blocking=True)
                bytes_out += h_out[sl].numel() * esz
                if r.ffn:
                    h_res[bi].copy_(dres[bi], non_blocking=True)
                    bytes_out += dres[bi].numel() * esz
                ev_out[sl].record(d2h)
        comp.wait_stream(d2h)

    steps = max(1, min(args.steps, args.e2e_steps))
    one_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for _ in range(steps):
        one_step()
    e1.record(comp)
    torch.cuda.synchronize()
    b.check(b.sync_status())
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    return {"value": round(w.n_tokens / (ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": int(bytes_in),
            "d2h_bytes_per_step": int(bytes_out), "ms_per_step": round(ms, 3), "steps": steps,
            "path": "C ABI ep_sp_select_heads / ep_sp_attend_ctas_xchg / ep_sp_xchg_wait / ep_sp_ffn_* per layer "
                    "on this rank's cost-balanced CTA range (the same partition as `value`); only the KV heads "
                    "the range touches are copied from pinned host memory (2 input slots cycled); this rank's "
                    "1/N of the exchanged output rows copied back"}


def run_e2e_layers(r: Runner, args, world):
    """N > 1 host-buffer variant of the layer schedule through the same C ABI
    calls: per layer, H2D of this rank's KV-head slice of Q/K/V and of its FFN
    rows from pinned memory, ep_sp_select_layer + ep_sp_attend_rows_xchg (the
    attention stores every tile into all ranks' slot) + ep_sp_xchg_wait, the
    FFN compaction/scatter, then D2H of this rank's 1/N of the full-width
    output rows and of its residual rows.  Two pinned input slots (layers
    cycled) and three exchange slots let the copies overlap the compute."""
    r.set_schedule("layer")
    w, c, N = r.w, r.ctx, r.w.n_tokens
    n_all = r.n_ub * r.rows_per_rank
    hid = w.ffn_hidden
    rows0, rows1 = r.rank * N // world, (r.rank + 1) * N // world
    pin = lambda *sh: torch.empty(*sh, dtype=r.tdt, pin_memory=True)  # noqa: E731
    hq = [pin(*r.Q[0].shape) for _ in range(2)]
    hk = [pin(*r.K[0].shape) for _ in range(2)]
    hv = [pin(*r.V[0].shape) for _ in range(2)]
    for i in range(2):
        hq[i].copy_(r.Q[i % w.n_layer])
        hk[i].copy_(r.K[i % w.n_layer])
        hv[i].copy_(r.V[i % w.n_layer])
    dq = [torch.empty_like(r.Q[0]) for _ in range(2)]
    dk = [torch.empty_like(r.K[0]) for _ in range(2)]
    dv = [torch.empty_like(r.V[0]) for _ in range(2)]
    h_out = [pin(rows1 - rows0, w.n_head, w.head_dim) for _ in range(3)]
    if r.ffn:
        hx = [pin(n_all, hid) for _ in range(2)]
        hr = [pin(n_all, hid) for _ in range(2)]
        for i in range(2):
            hx[i].copy_(r.X[i % w.n_layer])
            hr[i].copy_(r.R[i % w.n_layer])
        dx = [torch.empty(n_all, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
        dres = [torch.empty(n_all, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
        h_res = [pin(n_all, hid) for _ in range(2)]
    slots = [r.epsp.device_view(c.xchg_slot(i), (N, w.n_head, w.head_dim), w.dtype) for i in range(3)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]   # compute done with input buffer i
    ev_done = [torch.cuda.Event() for _ in range(3)]
    ev_out = [torch.cuda.Event() for _ in range(3)]    # D2H done with slot i
    esz = dq[0].element_size()
    bytes_in = bytes_out = 0

    def one_step():
        nonlocal bytes_in, bytes_out
        bytes_in = bytes_out = 0
        c.reset()
        for l in range(w.n_layer):
            b, sl = l % 2, l % 3
            with torch.cuda.stream(h2d):
                if l >= 2:
                    h2d.wait_event(ev_used[b])
                for d_, h_ in ((dq, hq), (dk, hk), (dv, hv)):
                    d_[b].copy_(h_[b], non_blocking=True)
                    bytes_in += d_[b].numel() * esz
                if r.ffn:
                    dx[b].copy_(hx[b], non_blocking=True)
                    dres[b].copy_(hr[b], non_blocking=True)
                    bytes_in += 2 * dx[b].numel() * esz
                ev_in[b].record(h2d)
            comp.wait_event(ev_in[b])
            if l >= 2:
                # readers of the slot written two exchange calls from now are done
                comp.wait_event(ev_out[(l + 1) % 3])
            c.check(c.select_layer(l, dq[b], dk[b], dv[b], N, N))
            c.check(c.attend_rows_xchg(l, N, N, 0, N, sl))
            c.check(c.xchg_wait(sl, N))
            if r.ffn:
                r.ffn_call(l, dx[b], r.keep, dres[b], n=n_all)
            ev_used[b].record(comp)
            ev_done[sl].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_done[sl])
                h_out[sl].copy_(slots[sl][rows0:rows1], non_blocking=True)
                bytes_out += h_out[sl].numel() * esz
                if r.ffn:
                    h_res[b].copy_(dres[b], non_blocking=True)
                    bytes_out += dres[b].numel() * esz
                ev_out[sl].record(d2h)
        comp.wait_stream(d2h)

    steps = max(1, min(args.steps, args.e2e_steps))
    one_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for _ in range(steps):
        one_step()
    e1.record(comp)
    torch.cuda.synchronize()
    c.check(c.sync_status())
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    return {"value": round(w.n_tokens / (ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": int(bytes_in),
            "d2h_bytes_per_step": int(bytes_out), "ms_per_step": round(ms, 3), "steps": steps,
            "path": "C ABI ep_sp_select_layer / ep_sp_attend_rows_xchg / ep_sp_xchg_wait / ep_sp_ffn_* per layer "
                    "(head-parallel slices), pinned host buffers (2 input slots cycled), this rank's 1/N of the "
                    "exchanged output rows copied back"}


def run_e2e(r: Runner, args, world):
    """Host-buffer variant through the same C ABI calls: per (ubatch, layer)
    H2D of Q/K/V rows (+ FFN x / residual rows) from pinned memory, compute,
    D2H of the attention output (+ residual rows); a 2-deep ring overlaps the
    copies of the next call with the compute of this one."""
    w, U = r.w, r.U
    d, hq, hkv = w.head_dim, r.hq, r.hkv
    n = r.rows_per_rank
    hid = w.ffn_hidden
    slots = 4  # pinned host slots of distinct (ubatch, layer) inputs, cycled
    pin = lambda *s: torch.empty(*s, dtype=r.tdt, pin_memory=True)  # noqa: E731
    hq_in = [pin(U, hq, d) for _ in range(slots)]
    hk_in = [pin(U, hkv, d) for _ in range(slots)]
    hv_in = [pin(U, hkv, d) for _ in range(slots)]
    for s in range(slots):
        l, u = s % w.n_layer, s // w.n_layer
        hq_in[s].copy_(r.Q[l][u * U:(u + 1) * U])
        hk_in[s].copy_(r.K[l][u * U:(u + 1) * U])
        hv_in[s].copy_(r.V[l][u * U:(u + 1) * U])
    h_out = [pin(U, hq, d) for _ in range(2)]
    if r.ffn:
        hx_in = [pin(n, hid) for _ in range(slots)]
        hr_in = [pin(n, hid) for _ in range(slots)]
        for s in range(slots):
            l, u = s % w.n_layer, (s // w.n_layer) % r.n_ub
            hx_in[s].copy_(r.X[l][u * n:(u + 1) * n])
            hr_in[s].copy_(r.R[l][u * n:(u + 1) * n])
        h_res = [pin(n, hid) for _ in range(2)]
        dx = [torch.empty(n, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
        dres = [torch.empty(n, hid, dtype=r.tdt, device=r.dev) for _ in range(2)]
    dq = [torch.empty(U, hq, d, dtype=r.tdt, device=r.dev) for _ in range(2)]
    dk = [torch.empty(U, hkv, d, dtype=r.tdt, device=r.dev) for _ in range(2)]
    dv = [torch.empty(U, hkv, d, dtype=r.tdt, device=r.dev) for _ in range(2)]
    do = [torch.empty(U, hq, d, dtype=r.tdt, device=r.dev) for _ in range(2)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    bytes_in = bytes_out = 0

    def one_step():
        nonlocal bytes_in, bytes_out
        bytes_in = bytes_out = 0
        r.ctx.reset()
        i = 0
        for u in range(r.n_ub):
            a, b = u * U, min((u + 1) * U, w.n_tokens)
            for l in range(w.n_layer):
                s, hs = i % 2, i % slots
                with torch.cuda.stream(h2d):
                    if i >= 2:
                        h2d.wait_event(ev_free[s])
                    dq[s][:b - a].copy_(hq_in[hs][:b - a], non_blocking=True)
                    dk[s][:b - a].copy_(hk_in[hs][:b - a], non_blocking=True)
                    dv[s][:b - a].copy_(hv_in[hs][:b - a], non_blocking=True)
                    bytes_in += (dq[s][:b - a].numel() + 2 * dk[s][:b - a].numel()) * dq[s].element_size()
                    if r.ffn:
                        dx[s].copy_(hx_in[hs], non_blocking=True)
                        dres[s].copy_(hr_in[hs], non_blocking=True)
                        bytes_in += 2 * dx[s].numel() * dx[s].element_size()
                    ev_in[s].record(h2d)
                comp.wait_event(ev_in[s])
                # the ubatch's new K/V rows enter the cache through the library's
                # fused append (page sums built in the same pass), as a KV write would
                r.ctx.check(r.ctx.append_kv(l, dk[s], dv[s], b - a, r.K[l], r.V[l], a))
                r.layer_call(l, u, dq[s][:b - a], do[s][:b - a])
                if r.ffn:
                    r.ffn_call(l, dx[s], r.keep[u * n:(u + 1) * n], dres[s])
                ev_done[s].record(comp)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_done[s])
                    h_out[s][:b - a].copy_(do[s][:b - a], non_blocking=True)
                    bytes_out += do[s][:b - a].numel() * do[s].element_size()
                    if r.ffn:
                        h_res[s].copy_(dres[s], non_blocking=True)
                        bytes_out += dres[s].numel() * dres[s].element_size()
                    ev_free[s].record(d2h)
                i += 1
        comp.wait_stream(d2h)

    steps = max(1, min(args.steps, args.e2e_steps))
    one_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for _ in range(steps):
        one_step()
    e1.record(comp)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    return {"value": round(w.n_tokens / (ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": int(bytes_in),
            "d2h_bytes_per_step": int(bytes_out), "ms_per_step": round(ms, 3), "steps": steps,
            "path": "C ABI ep_sp_append_kv (new K/V rows into the cache, page sums fused) / ep_sp_attend_layer / "
                    "ep_sp_ffn_* per (ubatch, layer), pinned host buffers; the host holds 4 distinct input slots "
                    "that are cycled over the (ubatch, layer) calls, so the copied bytes and the work are those of "
                    "the workload but the selections run on reused rows (results are checked by the tests, not "
                    "here)"}


def load_traffic(workload):
    """DRAM bytes per K3 launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", f"traffic_{workload}.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get("k3_dram_bytes_per_launch")
    return None


# ------------------------------------------------------------ CPU baseline
def cpu_sample(w: W.Workload, layer: int, qkv, n_rows: int, seed: int, n_threads: int, k_matrix):
    """Time the oracle on one layer: page sums + selection of every block, and
    attention of n_rows sampled query rows.  Returns the extrapolated seconds
    for the whole layer."""
    import oracle as O

    q, k, v = qkv
    p = O.params(n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim, page_size=w.page_size,
                 sel_pages=w.top_k, local_pages=w.local_pages, shared=0 if w.per_kv_head else 1,
                 q_subblock=w.q_subblock, max_gather_rows=w.max_gather_rows)
    kb = None if k_matrix is None else np.array(k_matrix[layer], np.int32)
    rng = np.random.default_rng(seed)
    rows = np.sort(rng.choice(w.n_tokens, size=n_rows, replace=False)).astype(np.int32)
    t0 = time.perf_counter()
    O.prefill_layer(p, q, k, v, w.dtype, n_ubatch=w.n_ubatch, k_budget=kb, attention=False, n_threads=n_threads)
    t1 = time.perf_counter()
    O.prefill_layer(p, q, k, v, w.dtype, n_ubatch=w.n_ubatch, k_budget=kb, attention=True, rows=rows,
                    n_threads=n_threads)
    t2 = time.perf_counter()
    t_sel = t1 - t0
    t_attn = (t2 - t1) - t_sel
    return t_sel + max(t_attn, 0.0) * (w.n_tokens / n_rows), (t2 - t0)


def layer_np(w, layer, device):
    q, k, v = W.gen_layer(w, layer, device=device)

    def cv(t):
        t = t.cpu().contiguous()
        return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()

    return cv(q), cv(k), cv(v)


def cpu_baseline(w: W.Workload, r=None, budget_s=20.0, levels=None):
    n_threads = os.cpu_count() or 1
    km = w.k_matrix()
    if km is None and w.top_k > 128:
        km = [[w.top_k] * w.n_head_kv for _ in range(w.n_layer)]
    levels = levels or sorted({min(w.n_layer - 1, i * max(1, w.pyramid_every or w.n_layer // 4)) for i in range(4)})
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    n_rows = 256
    est, spent = [], 0.0
    for i, l in enumerate(levels):
        qkv = layer_np(w, l, dev)
        e, s = cpu_sample(w, l, qkv, n_rows, seed=1000 + l, n_threads=n_threads, k_matrix=km)
        est.append(e)
        spent += s
        if spent > budget_s and i >= 0:
            break
    per_layer = sum(est) / len(est)
    total = per_layer * w.n_layer
    return {"value": round(w.n_tokens / total, 2), "unit": UNIT, "cores": n_threads, "kind": "port",
            "sample": f"oracle (C, fp64) on layers {levels[:len(est)]}: page sums + selection of all "
                      f"{w.n_tokens // w.n_ubatch} ubatches and attention of {n_rows} sampled query rows per "
                      f"layer, extrapolated to {w.n_tokens} rows x {w.n_layer} layers; {spent:.1f} s of CPU work",
            "seconds": round(spent, 1)}


def run_reference(args, w, world, rank):
    """--impl reference: the oracle port on the host cores (rank 0 only)."""
    if rank != 0:
        return
    n_threads = os.cpu_count() or 1
    km = w.k_matrix()
    if km is None and w.top_k > 128:
        km = [[w.top_k] * w.n_head_kv for _ in range(w.n_layer)]
    levels = sorted({min(w.n_layer - 1, i * max(1, w.pyramid_every or w.n_layer // 4)) for i in range(4)})
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cache = {}
    n_rows = 48
    ests, walls = [], []
    for i in range(args.warmup + args.steps):
        l = levels[i % len(levels)]
        if l not in cache:
            cache[l] = layer_np(w, l, dev)
        e, s = cpu_sample(w, l, cache[l], n_rows, seed=2000 + i, n_threads=n_threads, k_matrix=km)
        if i >= args.warmup:
            ests.append(e)
            walls.append(s)
    per_layer = statistics.mean(ests)
    value = w.n_tokens / (per_layer * w.n_layer)
    wall_ms = statistics.mean(walls) * 1e3
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(wall_ms, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": f"f64 (oracle arithmetic on {({W.BF16: 'bf16', W.F16: 'f16', W.F32: 'f32'})[w.dtype]} inputs)",
        "data": "synthetic (seeded)", "impl": "reference",
        "config": config_of(w, world, world > 1),
        "step": f"one sampled step = one layer's page sums + selection of every ubatch and the attention of "
                f"{n_rows} sampled query rows; ms_per_step is its measured wall time",
        "extrapolated": {"extrapolated": True, "ms_per_prefill": round(per_layer * w.n_layer * 1e3, 1),
                         "value": round(value, 2), "unit": UNIT,
                         "how": f"attention time scaled by {w.n_tokens}/{n_rows} rows, plus the selection, "
                                f"times {w.n_layer} layers; `value` is this whole-prefill throughput"},
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": n_threads, "kind": "port",
                         "sample": f"per step: one layer of {levels} (cycled): page sums + selection of every "
                                   f"ubatch + attention of {n_rows} sampled query rows, extrapolated to the "
                                   f"whole prefill; mean wall {statistics.mean(walls):.1f} s per step",
                         "reference_ggml_path": "unavailable: llama.cpp @3bb63cbc is not vendored and there is "
                                                "no network; the timed CPU arm is the oracle port"},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c4", choices=sorted(W.CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=0, help="profiling only: shorten the workload (not a bench value)")
    ap.add_argument("--layers", type=int, default=0, help="profiling only: fewer layers (not a bench value)")
    ap.add_argument("--partition", choices=["balanced", "heads"], default="balanced",
                    help="N > 1 with the peer exchange: cost-balanced ranges of the head-major attention grid "
                         "(balanced) or one KV-head slice per rank (heads)")
    ap.add_argument("--attn-tiles", type=int, choices=[1, 2], default=0,
                    help="query tiles per attention CTA (2: one CTA per SM, the default; 1: two CTAs per SM)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="N > 1: head outputs exchanged by the attention kernel over peer memory (peer) or by "
                         "chunked NCCL all-gathers (nccl)")
    ap.add_argument("--multicast", choices=["off", "auto", "on"], default=None,
                    help="N > 1 with the peer exchange: exchange buffers in symmetric memory, the attention "
                         "epilogue storing each tile once through their NVLink multicast address (auto: when the "
                         "GPUs offer one).  Default: auto from 4 GPUs up (one multicast store replaces N peer "
                         "stores), off below (at 2 GPUs one multicast store costs more than a local plus a "
                         "remote store)")
    args = ap.parse_args()
    if args.multicast is None:
        args.multicast = "auto" if args.gpus >= 4 else "off"
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    w = W.CONFIGS[args.workload]
    if args.tokens or args.layers:
        w = W.scaled(w, name=w.name + "-reduced", n_tokens=args.tokens or w.n_tokens, n_layer=args.layers or w.n_layer)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, w, world, rank)
        return
    if args.gpus > 1 and w.n_head_kv % args.gpus and (args.partition != "balanced" or args.exchange != "peer"):
        raise SystemExit(f"--workload {w.name} has {w.n_head_kv} KV heads: the {args.partition} partition needs a "
                         "number of GPUs that divides them (the balanced partition with the peer exchange does not)")
    world, rank, local = dist_setup(args.gpus)
    try:
        run_ours(args, w, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
