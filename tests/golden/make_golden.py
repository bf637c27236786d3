"""Generates the known-answer fixtures of tests/golden/*.npz from the oracle.

The reference holds no golden vectors for this path (its hot-path tests need
a GGUF model and pin no values), so these fixtures are produced by the CPU
oracle (oracle/ep_oracle.c) on seeded synthetic inputs.  They pin the oracle
and the CUDA path to the same answers across changes.  Inputs are not stored:
they are regenerated from the workload seed (edge-prefill_b200/workloads.py),
and the fixture keeps their SHA-256 so a generator change is detected.

Each fixture holds, for one layer: the selected pages and counts of every
gating block and KV head, and the fp64 attention output of a seeded sample of
query rows (stored as float32).

    python tests/golden/make_golden.py        # rewrites the .npz files
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "edge-prefill_b200"), os.path.join(ROOT, "oracle"), os.path.dirname(HERE)):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402

import oracle  # noqa: E402
import workloads as W  # noqa: E402
from gpu_util import to_np  # noqa: E402

# name: (workload, shared, k_budget per KV head or None, sampled rows)
CASES = {
    "ref_p32_bf16": (W.Workload("g1", 1024, 1, 8, 2, 64, W.BF16, 256, 32, 4, 64, per_kv_head=0,
                                max_gather_rows=4096), 1, None, 48),
    "ref_p32_offbyone_f16": (W.Workload("g2", 1024, 1, 8, 2, 64, W.F16, 256, 32, 8, 64, per_kv_head=0,
                                        max_gather_rows=4096, seed=1), 1, None, 48),
    "ext_p64_sub128_f16": (W.Workload("g3", 1024, 1, 8, 2, 64, W.F16, 1024, 64, 3, 128, q_subblock=128,
                                      seed=2), 0, None, 48),
    "ext_p128_kmatrix_bf16": (W.Workload("g4", 2048, 1, 8, 2, 128, W.BF16, 512, 128, 2, 256, seed=3), 0,
                              [-1, 3], 24),
    "gqa7_p64_bf16": (W.Workload("g5", 1024, 1, 28, 4, 128, W.BF16, 512, 64, 4, 128, q_subblock=64, seed=4), 0,
                      None, 12),
    "c1_f32": (W.CONFIGS["c1"], 0, None, 32),
    "c1_ref_mode_f32": (W.scaled(W.CONFIGS["c1"], per_kv_head=0, q_subblock=0, max_gather_rows=4096), 1, None, 16),
}


def inputs(w):
    q, k, v = W.gen_layer(w, 0)
    return to_np(q), to_np(k), to_np(v)


def digest(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def compute(name):
    w, shared, kb, n_rows = CASES[name]
    q, k, v = inputs(w)
    rng = np.random.default_rng(12345)
    rows = np.sort(rng.choice(w.n_tokens, size=n_rows, replace=False)).astype(np.int32)
    p = oracle.params(n_head=w.n_head, n_head_kv=w.n_head_kv, head_dim=w.head_dim, page_size=w.page_size,
                      sel_pages=w.top_k, local_pages=w.local_pages, shared=shared, q_subblock=w.q_subblock,
                      max_gather_rows=w.max_gather_rows)
    out, sel, cnt, blocks = oracle.prefill_layer(p, q, k, v, w.dtype, n_ubatch=w.n_ubatch,
                                                 k_budget=None if kb is None else np.array(kb, np.int32),
                                                 rows=rows, sel_cap=w.n_tokens // w.page_size + 1)
    width = max(1, int(cnt.max()))
    return {
        "sel": sel[:, :, :width].copy(), "cnt": cnt, "rows": rows, "out_rows": out[rows].astype(np.float32),
        "blocks": np.array(blocks, np.int32), "input_sha256": digest(q, k, v),
        "meta": json.dumps({"workload": w.__dict__, "shared": shared, "k_budget": kb}, default=str),
    }


def main():
    for name in CASES:
        d = compute(name)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print(name, "blocks", d["cnt"].shape[0], "selected", int(d["cnt"].sum()))


if __name__ == "__main__":
    main()
