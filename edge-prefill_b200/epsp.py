"""ctypes binding of libepsp.so (include/epsp.h) for the Python test and bench
harness.  Every call goes through the C ABI; torch tensors are only used as
device allocations (their data_ptr() is passed as a plain pointer).

The native library is mandatory: importing this module raises when
libepsp.so is missing or does not export the ABI.  There is no fallback.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int32, c_size_t, c_uint32, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
# EPSP_LIB names another build of the same library (for example a tuning
# variant); by default the in-tree build next to this file is loaded.
LIB_PATH = os.environ.get("EPSP_LIB") or os.path.join(HERE, "libepsp.so")

OK, INVALID_ARGUMENT, PREFILL, UNSUPPORTED, OUT_OF_MEMORY, IO, INTERNAL, UNAVAILABLE = 0, 2, 6, 9, 10, 11, 12, 13
F32, F16, BF16 = 0, 1, 2

# Every symbol include/epsp.h declares.
EXPORTS = [
    "ep_sp_create", "ep_sp_reserve", "ep_sp_destroy", "ep_sp_set_qg_bound", "ep_sp_get_qg_bound",
    "ep_sp_set_ext", "ep_sp_set_k_matrix", "ep_sp_get_k_matrix_size", "ep_sp_set_prefill_mode",
    "ep_sp_get_prefill_mode", "ep_sp_set_ffn_skip", "ep_sp_get_ffn_skip", "ep_sp_reset",
    "ep_sp_query_blocks", "ep_sp_attend_layer", "ep_sp_prefill", "ep_sp_ffn_compact", "ep_sp_ffn_scatter",
    "ep_sp_sync_status", "ep_sp_last_error", "ep_sp_error_name", "ep_sp_chunk_plan", "ep_sp_ffn_auto_mask",
    "ep_sp_ffn_parse", "ep_sp_parse_config", "ep_sp_profile_enable", "ep_sp_profile_read", "ep_sp_layer_work",
    "ep_sp_select_pages_noalloc", "ep_sp_select_layer", "ep_sp_attend_rows", "ep_sp_xchg_alloc",
    "ep_sp_xchg_open", "ep_sp_xchg_attach", "ep_sp_xchg_slot", "ep_sp_attend_rows_xchg", "ep_sp_xchg_wait",
    "ep_sp_select_heads", "ep_sp_attend_ctas", "ep_sp_attend_ctas_xchg", "ep_sp_attention_grid", "ep_sp_balance_ctas",
    "ep_sp_cta_work", "ep_sp_set_attn_tiles", "ep_sp_get_attn_tiles", "ep_sp_append_kv",
    "ep_sp_set_f32_attention", "ep_sp_get_f32_attention", "ep_sp_get_pooled_pages", "ep_sp_set_head_routing",
    "ep_sp_get_head_routing", "ep_sp_set_paged_kv", "ep_sp_xchg_attach_buffers", "ep_sp_xchg_bytes",
]
NUM_KERNELS = 6  # EP_SP_NUM_KERNELS
KERNEL_NAMES = ["k1_pool_pages", "k2_select_pages", "k3_sparse_attention", "k4_compact", "k4_scatter",
                "k5_exchange_wait"]
XCHG_HANDLE_BYTES = 64


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layer", c_int32), ("n_head", c_int32), ("n_head_kv", c_int32), ("head_dim", c_int32),
        ("dtype", c_int32), ("out_dtype", c_int32), ("max_ctx", c_int32), ("page_size", c_int32),
        ("device", c_int32), ("kv_head_offset", c_int32), ("n_head_kv_total", c_int32), ("kq_scale", c_float),
    ]


class PrefillOptions(ctypes.Structure):
    _fields_ = [
        ("chunk_size", c_uint32), ("enable_chunking", c_int32), ("enable_qg_bound", c_int32),
        ("qg_sel_pages", c_uint32), ("qg_local_rows", c_uint32), ("qg_pool_pages", c_uint32),
    ]


class PrefillStats(ctypes.Structure):
    _fields_ = [
        ("chunks", c_uint32), ("query_gating", c_int32), ("attn_fallback", c_int32), ("qg_groups", c_uint32),
        ("chunk_attn_rows", c_uint32),
    ]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libepsp.so not built ({LIB_PATH}); run __graft_entry__.build()")
    lib = ctypes.CDLL(LIB_PATH)
    missing = [s for s in EXPORTS if not hasattr(lib, s)]
    if missing:
        raise ImportError(f"libepsp.so lacks {missing}")
    P = c_void_p
    sig = {
        "ep_sp_create": (c_int32, [POINTER(Config), POINTER(P)]),
        "ep_sp_reserve": (c_int32, [P]),
        "ep_sp_destroy": (None, [P]),
        "ep_sp_set_qg_bound": (c_int32, [P, c_int32, c_int32, c_int32, c_int32]),
        "ep_sp_get_qg_bound": (c_int32, [P]),
        "ep_sp_set_ext": (c_int32, [P, c_int32, c_int32, c_int32]),
        "ep_sp_set_k_matrix": (c_int32, [P, POINTER(c_int32), c_size_t]),
        "ep_sp_get_k_matrix_size": (c_int32, [P]),
        "ep_sp_set_prefill_mode": (None, [P, c_int32]),
        "ep_sp_get_prefill_mode": (c_int32, [P]),
        "ep_sp_set_ffn_skip": (None, [P, c_uint64]),
        "ep_sp_get_ffn_skip": (c_uint64, [P]),
        "ep_sp_reset": (c_int32, [P]),
        "ep_sp_query_blocks": (c_int32, [P, c_int32, POINTER(c_int32)]),
        "ep_sp_attend_layer": (c_int32, [P, c_int32, P, P, P, c_int32, c_int32, P, P, P, c_int32, P]),
        "ep_sp_prefill": (c_int32, [P, POINTER(PrefillOptions), c_int32, POINTER(P), POINTER(P), POINTER(P),
                                    POINTER(P), c_int32, c_int32, POINTER(PrefillStats), P]),
        "ep_sp_ffn_compact": (c_int32, [P, c_int32, P, P, c_int32, c_int32, P, P, P, P]),
        "ep_sp_ffn_scatter": (c_int32, [P, c_int32, P, P, P, P, c_int32, c_int32, P]),
        "ep_sp_sync_status": (c_int32, [P, P]),
        "ep_sp_last_error": (c_char_p, [P]),
        "ep_sp_error_name": (c_char_p, [c_int32]),
        "ep_sp_chunk_plan": (c_int32, [c_uint32, c_uint32, c_uint32, POINTER(c_uint32), c_int32, POINTER(c_int32)]),
        "ep_sp_ffn_auto_mask": (c_int32, [c_int32, c_double, POINTER(c_uint64)]),
        "ep_sp_ffn_parse": (c_int32, [c_char_p, c_int32, POINTER(c_uint64), ctypes.c_char_p, c_int32]),
        "ep_sp_parse_config": (c_int32, [c_char_p, POINTER(PrefillOptions)]),
        "ep_sp_profile_enable": (c_int32, [P, c_int32]),
        "ep_sp_profile_read": (c_int32, [P, POINTER(c_double), POINTER(ctypes.c_int64)]),
        "ep_sp_layer_work": (c_int32, [P, c_int32, c_int32, c_int32, POINTER(c_double)]),
        "ep_sp_select_pages_noalloc": (c_int32, [P, c_int32, P, P, c_int32, c_int32, P, P, c_int32, P]),
        "ep_sp_select_layer": (c_int32, [P, c_int32, P, P, P, c_int32, c_int32, P, P, c_int32, P]),
        "ep_sp_attend_rows": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32, P, P]),
        "ep_sp_xchg_alloc": (c_int32, [P, c_int32, c_int32, POINTER(P), P]),
        "ep_sp_xchg_open": (c_int32, [P, P, POINTER(P)]),
        "ep_sp_xchg_attach": (c_int32, [P, c_int32, c_int32, POINTER(P)]),
        "ep_sp_xchg_slot": (c_int32, [P, c_int32, POINTER(P)]),
        "ep_sp_attend_rows_xchg": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, P]),
        "ep_sp_xchg_wait": (c_int32, [P, c_int32, c_int32, P]),
        "ep_sp_select_heads": (c_int32, [P, c_int32, P, P, P, c_int32, c_int32, c_int32, c_int32, P]),
        "ep_sp_attend_ctas": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32, P, P]),
        "ep_sp_attend_ctas_xchg": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, P]),
        "ep_sp_attention_grid": (c_int32, [P, c_int32, POINTER(c_int32)]),
        "ep_sp_balance_ctas": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, POINTER(c_int32)]),
        "ep_sp_cta_work": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32, POINTER(c_double)]),
        "ep_sp_set_attn_tiles": (c_int32, [P, c_int32]),
        "ep_sp_get_attn_tiles": (c_int32, [P]),
        "ep_sp_append_kv": (c_int32, [P, c_int32, P, P, c_int32, P, P, c_int32, P]),
        "ep_sp_set_f32_attention": (c_int32, [P, c_int32]),
        "ep_sp_get_f32_attention": (c_int32, [P]),
        "ep_sp_get_pooled_pages": (c_int32, [P, P, P, c_int32, P]),
        "ep_sp_set_head_routing": (c_int32, [P, c_int32, c_double]),
        "ep_sp_get_head_routing": (c_int32, [P, POINTER(c_int32), POINTER(c_double)]),
        "ep_sp_set_paged_kv": (c_int32, [P, c_int32, P, c_int32, c_int32]),
        "ep_sp_xchg_attach_buffers": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, POINTER(P), P]),
        "ep_sp_xchg_bytes": (c_int32, [P, c_int32, c_int32, POINTER(c_size_t)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class EpspError(RuntimeError):
    def __init__(self, rc: int, msg: str):
        super().__init__(f"{error_name(rc)} ({rc}): {msg}")
        self.rc = rc


def error_name(rc: int) -> str:
    return lib.ep_sp_error_name(rc).decode()


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype: int):
    """torch tensor aliasing `shape` elements of device memory at ptr (no copy),
    e.g. an exchange slot: device_view(ctx.xchg_slot(s), (n_tok, heads, d), BF16)."""
    import torch

    typestr = {F32: "<f4", F16: "<f2", BF16: "<i2"}[dtype]
    t = torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")
    return t.view(torch.bfloat16) if dtype == BF16 else t


class Context:
    """One ep_sp_ctx.  Methods return the C status code; `check()` raises."""

    def __init__(self, *, n_layer, n_head, n_head_kv, head_dim, dtype=BF16, out_dtype=None, max_ctx,
                 page_size=32, device=0, kv_head_offset=0, n_head_kv_total=0, kq_scale=0.0):
        self.cfg = Config(n_layer, n_head, n_head_kv, head_dim, dtype, dtype if out_dtype is None else out_dtype,
                          max_ctx, page_size, device, kv_head_offset, n_head_kv_total, kq_scale)
        self.h = c_void_p()
        rc = lib.ep_sp_create(ctypes.byref(self.cfg), ctypes.byref(self.h))
        if rc != OK:
            raise EpspError(rc, "ep_sp_create")

    def close(self):
        if self.h:
            lib.ep_sp_destroy(self.h)
            self.h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc: int) -> int:
        if rc != OK:
            raise EpspError(rc, self.last_error())
        return rc

    def last_error(self) -> str:
        return lib.ep_sp_last_error(self.h).decode()

    # controls -----------------------------------------------------------
    def reserve(self):
        return lib.ep_sp_reserve(self.h)

    def set_qg_bound(self, enabled, sel_pages, local_pages, pool_pages=0):
        return lib.ep_sp_set_qg_bound(self.h, enabled, sel_pages, local_pages, pool_pages)

    def qg_bound(self):
        return lib.ep_sp_get_qg_bound(self.h)

    def set_ext(self, per_kv_head, q_subblock, max_gather_rows):
        return lib.ep_sp_set_ext(self.h, per_kv_head, q_subblock, max_gather_rows)

    def set_k_matrix(self, values):
        vals = [int(x) for x in values]
        arr = (c_int32 * max(1, len(vals)))(*vals) if vals else None
        return lib.ep_sp_set_k_matrix(self.h, arr, len(vals))

    def k_matrix_size(self):
        return lib.ep_sp_get_k_matrix_size(self.h)

    def set_prefill_mode(self, on):
        lib.ep_sp_set_prefill_mode(self.h, 1 if on else 0)

    def prefill_mode(self):
        return lib.ep_sp_get_prefill_mode(self.h)

    def set_ffn_skip(self, mask):
        lib.ep_sp_set_ffn_skip(self.h, mask)

    def ffn_skip(self):
        return lib.ep_sp_get_ffn_skip(self.h)

    def reset(self):
        return lib.ep_sp_reset(self.h)

    def query_blocks(self, n_tok):
        n = c_int32()
        rc = lib.ep_sp_query_blocks(self.h, n_tok, ctypes.byref(n))
        return rc, n.value

    def sync_status(self, stream=None):
        return lib.ep_sp_sync_status(self.h, _stream(stream))

    # compute ------------------------------------------------------------
    def attend_layer(self, layer, q, k, v, kv_len, n_tok, out, sel=None, cnt=None, sel_cap=0, stream=None):
        return lib.ep_sp_attend_layer(self.h, layer, _ptr(q), _ptr(k), _ptr(v), kv_len, n_tok, _ptr(out),
                                      _ptr(sel), _ptr(cnt), sel_cap, _stream(stream))

    def select_layer(self, layer, q, k, v, kv_len, n_tok, sel=None, cnt=None, sel_cap=0, stream=None):
        return lib.ep_sp_select_layer(self.h, layer, _ptr(q), _ptr(k), _ptr(v), kv_len, n_tok, _ptr(sel), _ptr(cnt),
                                      sel_cap, _stream(stream))

    def attend_rows(self, layer, kv_len, n_tok, row_begin, row_end, out, stream=None):
        return lib.ep_sp_attend_rows(self.h, layer, kv_len, n_tok, row_begin, row_end, _ptr(out), _stream(stream))

    # ---------------------------------------------- head-parallel exchange
    def xchg_alloc(self, rows, n_slots, ipc=True):
        """Allocates this rank's exchange buffer; returns (base, handle bytes or None)."""
        base = c_void_p()
        h = ctypes.create_string_buffer(XCHG_HANDLE_BYTES) if ipc else None
        self.check(lib.ep_sp_xchg_alloc(self.h, rows, n_slots, ctypes.byref(base), h))
        return base.value, (h.raw if ipc else None)

    def xchg_open(self, handle: bytes):
        base = c_void_p()
        buf = ctypes.create_string_buffer(handle, XCHG_HANDLE_BYTES)
        self.check(lib.ep_sp_xchg_open(self.h, buf, ctypes.byref(base)))
        return base.value

    def xchg_attach(self, rank, bases):
        arr = (c_void_p * len(bases))(*bases)
        return lib.ep_sp_xchg_attach(self.h, len(bases), rank, arr)

    def xchg_attach_buffers(self, rows, n_slots, rank, bases, mc_base=None):
        arr = (c_void_p * len(bases))(*bases)
        return lib.ep_sp_xchg_attach_buffers(self.h, rows, n_slots, len(bases), rank, arr, mc_base)

    def xchg_bytes(self, rows, n_slots):
        n = c_size_t()
        self.check(lib.ep_sp_xchg_bytes(self.h, rows, n_slots, ctypes.byref(n)))
        return n.value

    def xchg_slot(self, slot):
        p = c_void_p()
        self.check(lib.ep_sp_xchg_slot(self.h, slot, ctypes.byref(p)))
        return p.value

    def attend_rows_xchg(self, layer, kv_len, n_tok, row_begin, row_end, slot, stream=None):
        return lib.ep_sp_attend_rows_xchg(self.h, layer, kv_len, n_tok, row_begin, row_end, slot, _stream(stream))

    def xchg_wait(self, slot, rows, stream=None):
        return lib.ep_sp_xchg_wait(self.h, slot, rows, _stream(stream))

    def attend_ctas_xchg(self, layer, kv_len, n_tok, cta_begin, cta_end, slot, stream=None):
        return lib.ep_sp_attend_ctas_xchg(self.h, layer, kv_len, n_tok, cta_begin, cta_end, slot, _stream(stream))

    # ------------------------------------------------- splitting a layer
    def select_heads(self, layer, q, k, v, kv_len, n_tok, head_begin, head_end, stream=None):
        return lib.ep_sp_select_heads(self.h, layer, _ptr(q), _ptr(k), _ptr(v), kv_len, n_tok, head_begin, head_end,
                                      _stream(stream))

    def attend_ctas(self, layer, kv_len, n_tok, cta_begin, cta_end, out, stream=None):
        return lib.ep_sp_attend_ctas(self.h, layer, kv_len, n_tok, cta_begin, cta_end, _ptr(out), _stream(stream))

    def attention_grid(self, n_tok):
        n = c_int32()
        self.check(lib.ep_sp_attention_grid(self.h, n_tok, ctypes.byref(n)))
        return n.value

    def append_kv(self, layer, k_new, v_new, n_new, k_cache, v_cache, kv_pos, stream=None):
        return lib.ep_sp_append_kv(self.h, layer, _ptr(k_new), _ptr(v_new), n_new, _ptr(k_cache), _ptr(v_cache),
                                   kv_pos, _stream(stream))

    def set_attn_tiles(self, tiles_per_cta):
        return lib.ep_sp_set_attn_tiles(self.h, tiles_per_cta)

    def attn_tiles(self):
        return lib.ep_sp_get_attn_tiles(self.h)

    def set_paged_kv(self, block_rows, block_table=None, n_entries=0, pool_rows=0):
        return lib.ep_sp_set_paged_kv(self.h, block_rows, _ptr(block_table), n_entries, pool_rows)

    def set_head_routing(self, mode, threshold):
        return lib.ep_sp_set_head_routing(self.h, mode, threshold)

    def head_routing(self):
        m, t = c_int32(), c_double()
        self.check(lib.ep_sp_get_head_routing(self.h, ctypes.byref(m), ctypes.byref(t)))
        return m.value, t.value

    def pooled_pages(self, pages, counts, cap, stream=None):
        return lib.ep_sp_get_pooled_pages(self.h, _ptr(pages), _ptr(counts), cap, _stream(stream))

    def set_f32_attention(self, mode):
        return lib.ep_sp_set_f32_attention(self.h, mode)

    def f32_attention(self):
        return lib.ep_sp_get_f32_attention(self.h)

    def cta_work(self, layer, kv_len, n_tok, cta_begin, cta_end):
        out = (c_double * 3)()
        self.check(lib.ep_sp_cta_work(self.h, layer, kv_len, n_tok, cta_begin, cta_end, out))
        return list(out)

    def balance_ctas(self, layer, kv_len, n_tok, n_parts):
        cuts = (c_int32 * (n_parts + 1))()
        self.check(lib.ep_sp_balance_ctas(self.h, layer, kv_len, n_tok, n_parts, cuts))
        return list(cuts)

    def prefill(self, opts: PrefillOptions, qs, ks, vs, outs, n_tokens, n_ubatch, stream=None):
        n = len(qs)
        arr = lambda ts: (c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
        stats = PrefillStats()
        rc = lib.ep_sp_prefill(self.h, ctypes.byref(opts), n, arr(qs), arr(ks), arr(vs), arr(outs), n_tokens,
                               n_ubatch, ctypes.byref(stats), _stream(stream))
        return rc, stats

    def select_pages_noalloc(self, layer, q, k, kv_len, n_tok, sel, cnt, sel_cap, stream=None):
        return lib.ep_sp_select_pages_noalloc(self.h, layer, _ptr(q), _ptr(k), kv_len, n_tok, _ptr(sel), _ptr(cnt),
                                              sel_cap, _stream(stream))

    def ffn_compact(self, layer, x, keep, n_rows, hidden, x_kept, row_ids, n_keep, stream=None):
        return lib.ep_sp_ffn_compact(self.h, layer, _ptr(x), _ptr(keep), n_rows, hidden, _ptr(x_kept),
                                     _ptr(row_ids), _ptr(n_keep), _stream(stream))

    def ffn_scatter(self, layer, ffn_out, residual, row_ids, n_keep, n_rows, hidden, stream=None):
        return lib.ep_sp_ffn_scatter(self.h, layer, _ptr(ffn_out), _ptr(residual), _ptr(row_ids), _ptr(n_keep),
                                     n_rows, hidden, _stream(stream))


# host-side planning (no device) -----------------------------------------
def chunk_plan(n_tokens, chunk_size, n_ubatch, cap=1 << 16):
    buf = (c_uint32 * (2 * cap))()
    n = c_int32()
    rc = lib.ep_sp_chunk_plan(n_tokens, chunk_size, n_ubatch, buf, cap, ctypes.byref(n))
    if rc != OK:
        return rc, []
    return rc, [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)]


def ffn_auto_mask(n_layer, ratio):
    out = c_uint64()
    rc = lib.ep_sp_ffn_auto_mask(n_layer, ratio, ctypes.byref(out))
    return rc, out.value


def ffn_parse(spec, n_layer):
    out = c_uint64()
    warn = ctypes.create_string_buffer(64)
    rc = lib.ep_sp_ffn_parse(None if spec is None else spec.encode(), n_layer, ctypes.byref(out), warn, 64)
    return rc, out.value, warn.value.decode()


def parse_config(path):
    o = PrefillOptions(0, 1, 0, 8, 0, 0)
    rc = lib.ep_sp_parse_config(path.encode(), ctypes.byref(o))
    return rc, o
