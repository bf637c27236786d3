"""ctypes wrapper of the CPU oracle (libep_oracle.so) and of the reference's
own host code compiled into _ref/ (libep_ref_host.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference leg, always as the checker or the
timed CPU baseline, never as a product path.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_int32, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "libep_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libep_ref_host.so")

F32, F16, BF16 = 0, 1, 2


class Params(ctypes.Structure):
    _fields_ = [
        ("n_head", c_int32), ("n_head_kv", c_int32), ("head_dim", c_int32), ("page_size", c_int32),
        ("sel_pages", c_int32), ("local_pages", c_int32), ("shared", c_int32), ("q_subblock", c_int32),
        ("max_gather_rows", c_int32), ("kq_scale", c_double), ("pool_pages", c_int32), ("route_mode", c_int32),
        ("route_threshold", c_double),
    ]


class BlockPlan(ctypes.Structure):
    _fields_ = [("b0", c_int32), ("b1", c_int32), ("lsp", c_int32), ("gated", c_int32), ("k_sel", c_int32),
                ("n_local", c_int32)]


def _load():
    if not os.path.exists(ORACLE_LIB):
        raise ImportError(f"{ORACLE_LIB} not built (make -C oracle)")
    lib = ctypes.CDLL(ORACLE_LIB)
    P = c_void_p
    lib.epo_plan_block.argtypes = [POINTER(Params), c_int32, c_int32, c_int32, POINTER(BlockPlan)]
    lib.epo_plan_block.restype = None
    lib.epo_chunk_plan.argtypes = [c_uint32, c_uint32, c_uint32, POINTER(c_uint32), c_int32]
    lib.epo_chunk_plan.restype = c_int32
    lib.epo_count_blocks.argtypes = [POINTER(Params), c_uint32, c_uint32, c_uint32]
    lib.epo_count_blocks.restype = c_int32
    lib.epo_list_blocks.argtypes = [POINTER(Params), c_uint32, c_uint32, c_uint32, POINTER(c_int32), c_int32]
    lib.epo_list_blocks.restype = c_int32
    lib.epo_page_sums.argtypes = [P, c_int32, c_int32, c_int32, c_int32, c_int32, P]
    lib.epo_page_sums.restype = None
    lib.epo_select_block.argtypes = [POINTER(Params), POINTER(BlockPlan), P, c_int32, P, c_int32, c_int32, P, P]
    lib.epo_select_block.restype = c_int32
    lib.epo_prefill_layer.argtypes = [POINTER(Params), P, P, P, P, c_int32, c_uint32, c_uint32, c_uint32, P, P,
                                      c_int32, P, P, c_int32, c_int32]
    lib.epo_prefill_layer.restype = c_int32
    lib.epo_prefill_layer_ex.argtypes = [POINTER(Params), P, P, P, P, c_int32, c_uint32, c_uint32, c_uint32, P, P,
                                         c_int32, P, P, c_int32, P, P, c_int32, c_int32]
    lib.epo_prefill_layer_ex.restype = c_int32
    lib.epo_pool_block.argtypes = [POINTER(Params), POINTER(BlockPlan), P, c_int32, P, c_int32, c_int32, P]
    lib.epo_pool_block.restype = c_int32
    lib.epo_pool_elem.argtypes = [c_double, c_int32, c_int32]
    lib.epo_pool_elem.restype = c_double
    lib.epo_route_block.argtypes = [POINTER(Params), POINTER(BlockPlan), P, c_int32, P, c_int32, P, P, P]
    lib.epo_route_block.restype = None
    lib.epo_ffn_compact.argtypes = [P, c_int32, P, c_int32, c_int32, c_int32, P, P]
    lib.epo_ffn_compact.restype = c_int32
    lib.epo_ffn_scatter.argtypes = [P, P, c_int32, P, c_int32, c_int32]
    lib.epo_ffn_scatter.restype = None
    for n in ("epo_f16_to_f32", "epo_bf16_to_f32"):
        getattr(lib, n).argtypes = [ctypes.c_uint16]
        getattr(lib, n).restype = ctypes.c_float
    for n in ("epo_f32_to_f16", "epo_f32_to_bf16"):
        getattr(lib, n).argtypes = [ctypes.c_float]
        getattr(lib, n).restype = ctypes.c_uint16
    return lib


lib = _load()


def _p(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def params(*, n_head, n_head_kv, head_dim, page_size=32, sel_pages=8, local_pages=0, shared=1, q_subblock=0,
           max_gather_rows=4096, kq_scale=0.0, pool_pages=0, route_mode=0, route_threshold=0.0) -> Params:
    return Params(n_head, n_head_kv, head_dim, page_size, sel_pages, local_pages, shared, q_subblock,
                  max_gather_rows, kq_scale, pool_pages, route_mode, route_threshold)


def plan_block(p: Params, b0, b1, k_budget) -> BlockPlan:
    out = BlockPlan()
    lib.epo_plan_block(ctypes.byref(p), b0, b1, k_budget, ctypes.byref(out))
    return out


def chunk_plan(n_tokens, chunk_size, n_ubatch, cap=1 << 16):
    buf = (c_uint32 * (2 * cap))()
    n = lib.epo_chunk_plan(n_tokens, chunk_size, n_ubatch, buf, cap)
    if n < 0:
        return n, []
    return 0, [(buf[2 * i], buf[2 * i + 1]) for i in range(n)]


def list_blocks(p: Params, n_tokens, chunk_size, n_ubatch):
    nb = lib.epo_count_blocks(ctypes.byref(p), n_tokens, chunk_size, n_ubatch)
    buf = (c_int32 * (2 * nb))()
    lib.epo_list_blocks(ctypes.byref(p), n_tokens, chunk_size, n_ubatch, buf, nb)
    return [(buf[2 * i], buf[2 * i + 1]) for i in range(nb)]


def dtype_code(arr: np.ndarray, hint=None) -> int:
    """numpy arrays: float32 -> F32; uint16 carries f16/bf16 bits (hint)."""
    if arr.dtype == np.float32:
        return F32
    if arr.dtype == np.float16:
        return F16
    if hint is None:
        raise ValueError("uint16 input needs a dtype hint (F16 or BF16)")
    return hint


def _raw(arr):
    if arr.dtype == np.float16:
        return np.ascontiguousarray(arr).view(np.uint16)
    return np.ascontiguousarray(arr)


def page_sums(k, dtype, page_size):
    n_rows, hkv, d = k.shape
    n_pages = n_rows // page_size
    out = np.zeros((hkv, max(n_pages, 1), d), np.float64)
    kk = _raw(k)
    lib.epo_page_sums(_p(kk), dtype, n_rows, hkv, d, page_size, _p(out))
    return out[:, :n_pages]


def select_block(p: Params, plan: BlockPlan, q_last, dtype, psum, head):
    """Selection of one gating block (epo_select_block): q_last = the block's
    last query row [Hq][d]; psum = page_sums(...) [Hkv][n_pages][d]; head >= 0
    per-KV-head, -1 shared.  Returns the page list (ascending)."""
    ps = np.ascontiguousarray(psum, np.float64)
    out = np.zeros(max(1, plan.k_sel), np.int32)
    qq = _raw(np.ascontiguousarray(q_last))
    n = lib.epo_select_block(ctypes.byref(p), ctypes.byref(plan), _p(qq), dtype, _p(ps), ps.shape[1], head,
                             _p(out), None)
    return out[:n]


def pool_block(p: Params, plan: BlockPlan, q_last, dtype, psum, head):
    """Pooled pages of one gating block (epo_pool_block), ascending."""
    ps = np.ascontiguousarray(psum, np.float64)
    out = np.zeros(max(1, p.pool_pages, plan.lsp), np.int32)
    qq = _raw(np.ascontiguousarray(q_last))
    n = lib.epo_pool_block(ctypes.byref(p), ctypes.byref(plan), _p(qq), dtype, _p(ps), ps.shape[1], head, _p(out))
    return out[:n]


def route_block(p: Params, plan: BlockPlan, q_last, dtype, psum, k_in):
    """Routing of one block (epo_route_block): (effective budgets [Hkv], spreads [Hkv])."""
    ps = np.ascontiguousarray(psum, np.float64)
    kin = np.ascontiguousarray(k_in, np.int32)
    kout = np.zeros(p.n_head_kv, np.int32)
    spread = np.full(p.n_head_kv, np.nan)
    qq = _raw(np.ascontiguousarray(q_last))
    lib.epo_route_block(ctypes.byref(p), ctypes.byref(plan), _p(qq), dtype, _p(ps), ps.shape[1], _p(kin), _p(kout),
                        _p(spread))
    return kout, spread


def prefill_layer(p: Params, q, k, v, dtype, *, n_ubatch, chunk_size=0, k_budget=None, attention=True,
                  rows=None, sel_cap=None, n_threads=None, return_pool=False):
    """Returns (out fp64 [n_tok][Hq][d] or None, sel [nb][Hkv][cap], cnt [nb][Hkv], blocks), plus
    (pool [nb][Hkv][pool_cap], pool_cnt [nb][Hkv]) with return_pool."""
    n_tok = q.shape[0]
    blocks = list_blocks(p, n_tok, chunk_size, n_ubatch)
    nb = len(blocks)
    hkv = p.n_head_kv
    if sel_cap is None:
        sel_cap = max(1, n_tok // p.page_size + 1)
    sel = np.full((nb, hkv, sel_cap), -1, np.int32)
    cnt = np.zeros((nb, hkv), np.int32)
    out = np.zeros(q.shape, np.float64) if attention else None
    kb = None if k_budget is None else np.ascontiguousarray(k_budget, np.int32)
    rr = None if rows is None else np.ascontiguousarray(rows, np.int32)
    qq, kk, vv = _raw(q), _raw(k), _raw(v)
    pool_cap = max(1, n_tok // p.page_size)
    pool = np.full((nb, hkv, pool_cap), -1, np.int32)
    pcnt = np.zeros((nb, hkv), np.int32)
    rc = lib.epo_prefill_layer_ex(ctypes.byref(p), _p(kb), _p(qq), _p(kk), _p(vv), dtype, n_tok, chunk_size,
                                  n_ubatch, _p(out), _p(rr), 0 if rr is None else len(rr), _p(sel), _p(cnt), sel_cap,
                                  _p(pool), _p(pcnt), pool_cap, n_threads or os.cpu_count() or 1)
    if rc < 0:
        raise RuntimeError(f"epo_prefill_layer rc {rc}")
    if return_pool:
        return out, sel, cnt, blocks, pool, pcnt
    return out, sel, cnt, blocks


def ffn_compact(x, keep, layer_skipped=False):
    n_rows, hidden = x.shape
    xk = np.zeros_like(x)
    ids = np.zeros(n_rows, np.int32)
    xr = np.ascontiguousarray(x)
    kp = np.ascontiguousarray(keep, np.uint8)
    n = lib.epo_ffn_compact(_p(xr), xr.dtype.itemsize, _p(kp), n_rows, hidden, 1 if layer_skipped else 0, _p(xk),
                            _p(ids))
    return xk[:n], ids[:n]


def ffn_scatter(ffn_out, residual, dtype, row_ids):
    res = np.ascontiguousarray(residual).copy()
    fo = np.ascontiguousarray(ffn_out)
    ids = np.ascontiguousarray(row_ids, np.int32)
    lib.epo_ffn_scatter(_p(fo), _p(res), dtype, _p(ids), len(ids), res.shape[1])
    return res


# ---------------------------------------------------------------- reference
def load_ref():
    """The reference's own ChunkScheduler / FfnSkipController built from its
    sources (oracle/Makefile `ref`), or None when not built."""
    if not os.path.exists(REF_LIB):
        return None
    r = ctypes.CDLL(REF_LIB)
    r.ref_chunk_plan.argtypes = [c_uint32, c_uint32, c_uint32, POINTER(c_uint32), c_int32, POINTER(c_int32)]
    r.ref_chunk_plan.restype = c_int32
    r.ref_ffn_auto_mask.argtypes = [c_int32, c_double, POINTER(c_uint64)]
    r.ref_ffn_auto_mask.restype = c_int32
    r.ref_ffn_parse.argtypes = [ctypes.c_char_p, c_int32, POINTER(c_uint64), ctypes.c_char_p, c_int32]
    r.ref_ffn_parse.restype = c_int32
    r.ref_error_code_name.argtypes = [c_int32]
    r.ref_error_code_name.restype = ctypes.c_char_p
    return r
