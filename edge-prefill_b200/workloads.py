"""Synthetic workloads of the page-gated sparse prefill path (seeded).

No public dataset is involved; these stand in for real prompts with the
shapes, sizes and value distributions of the five benchmark configurations:

  c1  Qwen2-0.5B-like attention (14 q heads, 2 KV heads, d 64), 1 layer,
      4096 tokens as one ubatch, f32 Q/K/V ~ N(0,1)/sqrt(64), page 64,
      top-k 16 + sink + 256-row window (sub-blocks of 128 rows in the
      per-KV-head mode; the reference's shared mode bypasses to dense here).
  c2  same heads, 8192 tokens in ubatches of 512, 24 layers, f16,
      Q/K ~ N(0,1) with 2% of pages carrying a rank-1 "needle" direction
      (4*u added to every row of the page, +u added to every query row),
      page 64, top-k 32 + sink + 512-row window.
  c3  Llama-3-8B attention (32 q heads, 8 KV heads, d 128), 32768 tokens,
      bf16, ubatch 2048, page 128, top-k 64 + sink + 1024-row window;
      K channels scaled per (layer, head, channel) by lognormal(0, 0.5).
  c4  65536 tokens, Llama-3-8B shapes, bf16, ubatch 4096, page 128,
      top-k per (layer, KV head) uniform from {32, 64, 128} then halved every
      8 layers, 1024-row window, 32 layers; FFN-skip compaction keeping
      round(0.15 * N) rows (hidden 4096) chosen by a seeded permutation.
  c5  Qwen2-7B-like (28 q heads, 4 KV heads, d 128), 131072 tokens, bf16,
      ubatch 8192, page 64, top-k 256 + sink + 2048-row window, gating per
      512-row sub-block, 28 layers.

V rows are drawn N(0,1)/sqrt(d) everywhere (unit-RMS rows; the
configurations do not specify V), and Q/K of c3-c5 N(0,1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

F32, F16, BF16 = 0, 1, 2
TORCH_DTYPE = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}


@dataclass
class Workload:
    name: str
    n_tokens: int
    n_layer: int
    n_head: int
    n_head_kv: int
    head_dim: int
    dtype: int
    n_ubatch: int
    page_size: int
    top_k: int
    local_rows: int
    q_subblock: int = 0
    per_kv_head: int = 1
    max_gather_rows: int = 0
    adaptive_k: tuple = ()          # choices for per-(layer, head) budgets
    pyramid_every: int = 0          # halve budgets every N layers
    k_outlier_sigma: float = 0.0    # lognormal per-channel K scale
    needle_frac: float = 0.0
    qk_std: float = 1.0
    ffn_hidden: int = 0
    ffn_keep_frac: float = 0.0
    seed: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def local_pages(self) -> int:
        return self.local_rows // self.page_size

    def k_matrix(self):
        """[n_layer][n_head_kv] budgets, or None for a uniform top_k."""
        if not self.adaptive_k and not self.pyramid_every:
            return None
        g = torch.Generator().manual_seed(self.seed + 7)
        out = []
        for l in range(self.n_layer):
            row = []
            for _ in range(self.n_head_kv):
                if self.adaptive_k:
                    k = self.adaptive_k[int(torch.randint(len(self.adaptive_k), (1,), generator=g))]
                else:
                    k = self.top_k
                if self.pyramid_every:
                    k = max(1, k >> (l // self.pyramid_every))
                row.append(k)
            out.append(row)
        return out


CONFIGS = {
    "c1": Workload("c1", 4096, 1, 14, 2, 64, F32, 4096, 64, 16, 256, q_subblock=128,
                   qk_std=1.0 / 8.0),
    "c2": Workload("c2", 8192, 24, 14, 2, 64, F16, 512, 64, 32, 512, needle_frac=0.02),
    "c3": Workload("c3", 32768, 32, 32, 8, 128, BF16, 2048, 128, 64, 1024, k_outlier_sigma=0.5),
    "c4": Workload("c4", 65536, 32, 32, 8, 128, BF16, 4096, 128, 64, 1024, adaptive_k=(32, 64, 128),
                   pyramid_every=8, k_outlier_sigma=0.5, ffn_hidden=4096, ffn_keep_frac=0.15),
    "c5": Workload("c5", 131072, 28, 28, 4, 128, BF16, 8192, 64, 256, 2048, q_subblock=512),
}


def scaled(w: Workload, **over) -> Workload:
    """A copy with some fields replaced (small parity cases of a config)."""
    d = dict(w.__dict__)
    d.update(over)
    return Workload(**d)


def gen_layer(w: Workload, layer: int, device="cpu", n_tokens=None, head_slice=None):
    """Q [N][Hq][d], K, V [N][Hkv][d] of one layer in the workload dtype.
    head_slice=(kv0, kv1) returns only those KV heads and their query heads
    (the same values the full tensors hold there)."""
    N = n_tokens or w.n_tokens
    Hq, Hkv, d = w.n_head, w.n_head_kv, w.head_dim
    G = Hq // Hkv
    g = torch.Generator(device=device).manual_seed(w.seed * 1000003 + layer * 7919 + 1)
    q = torch.randn(N, Hq, d, generator=g, device=device) * w.qk_std
    k = torch.randn(N, Hkv, d, generator=g, device=device) * w.qk_std
    v = torch.randn(N, Hkv, d, generator=g, device=device) / math.sqrt(d)
    if w.k_outlier_sigma > 0:
        s = torch.exp(torch.randn(1, Hkv, d, generator=g, device=device) * w.k_outlier_sigma)
        k = k * s
    if w.needle_frac > 0:
        P = w.page_size
        n_pages = N // P
        u = torch.randn(Hkv, d, generator=g, device=device)
        u = u / u.norm(dim=-1, keepdim=True)
        n_needle = max(1, int(round(w.needle_frac * n_pages)))
        for h in range(Hkv):
            pages = torch.randperm(n_pages, generator=g, device=device)[:n_needle]
            rows = (pages[:, None] * P + torch.arange(P, device=device)[None, :]).reshape(-1)
            k[rows, h, :] += 4.0 * u[h]
            q[:, h * G:(h + 1) * G, :] += u[h]
    dt = TORCH_DTYPE[w.dtype]
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    if head_slice is not None:
        a, b = head_slice
        q = q[:, a * G:b * G].contiguous()
        k = k[:, a:b].contiguous()
        v = v[:, a:b].contiguous()
    return q, k, v


def ffn_keep_mask(w: Workload, n_tokens=None, device="cpu"):
    N = n_tokens or w.n_tokens
    g = torch.Generator().manual_seed(w.seed + 99)
    keep = torch.zeros(N, dtype=torch.uint8)
    n_keep = int(round(w.ffn_keep_frac * N))
    keep[torch.randperm(N, generator=g)[:n_keep]] = 1
    return keep.to(device)


def shard_kv_heads(n_head_kv: int, world: int, rank: int):
    """Head-parallel partition: rank r owns KV heads [r*Hkv/W, (r+1)*Hkv/W)."""
    if n_head_kv % world:
        raise ValueError(f"{n_head_kv} KV heads do not split over {world} ranks")
    per = n_head_kv // world
    return rank * per, (rank + 1) * per
