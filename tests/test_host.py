"""Host-side tests (no GPU): the C ABI loads and exports every declared symbol,
and its validation / planning logic matches the reference.

Mirrors the reference's own unit tests for this path:
  tests/test_sparse_attn_exec.cpp:1571-1594  bound_gating_capi_validation
  tests/test_attention_sparsity.cpp:236-268  bound_gating_config_parse
  tests/test_chunk_scheduler.cpp             ChunkScheduler::plan
  tests/test_ffn_skip.cpp                    FfnSkipController
The planning functions are also compared case by case with the reference's
own sources compiled into oracle/_ref (when that build is present).
"""
import os
import re

import pytest

import epsp
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_exports_match_header():
    hdr = open(os.path.join(ROOT, "include", "epsp.h")).read()
    declared = set(re.findall(r"\b(ep_sp_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(epsp.EXPORTS)
    for name in declared:
        assert hasattr(epsp.lib, name), name


def make_ctx(**kw):
    args = dict(n_layer=4, n_head=8, n_head_kv=2, head_dim=64, dtype=epsp.BF16, max_ctx=4096, page_size=32)
    args.update(kw)
    return epsp.Context(**args)


def test_header_is_plain_c_and_links(tmp_path):
    """include/epsp.h is a C ABI: a C99 program that includes it compiles with
    -pedantic and no warnings, links against libepsp.so and calls into it (what
    a cgo / ctypes / JNI binding relies on)."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "use_epsp.c"
    src.write_text('#include "epsp.h"\n#include <string.h>\n'
                   "int main(void) {\n"
                   "    ep_sp_config c;\n    memset(&c, 0, sizeof c);\n"
                   "    c.n_layer = 1; c.n_head = 8; c.n_head_kv = 2; c.head_dim = 64; c.dtype = EP_SP_BF16;\n"
                   "    c.out_dtype = EP_SP_BF16; c.max_ctx = 1024; c.page_size = 32;\n"
                   "    ep_sp_ctx* ctx = 0;\n    if (ep_sp_create(&c, &ctx) != EP_SP_OK) return 2;\n"
                   "    int rc = ep_sp_set_qg_bound(ctx, 1, 8, 0, 0);\n    ep_sp_destroy(ctx);\n"
                   "    return rc == EP_SP_OK ? 0 : 3;\n}\n")
    exe = tmp_path / "use_epsp"
    lib_dir = os.path.join(root, "edge-prefill_b200")
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                         os.path.join(root, "include"), str(src), "-L", lib_dir, "-lepsp", f"-Wl,-rpath,{lib_dir}",
                         "-o", str(exe)], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    assert subprocess.run([str(exe)]).returncode == 0


def test_create_validation():
    bad = [dict(n_head=7), dict(head_dim=96), dict(page_size=48), dict(dtype=5), dict(max_ctx=0),
           dict(n_layer=0), dict(kv_head_offset=1), dict(n_head_kv_total=1)]
    for b in bad:
        with pytest.raises(epsp.EpspError) as e:
            make_ctx(**b)
        assert e.value.rc == epsp.INVALID_ARGUMENT, b
    make_ctx(kv_head_offset=2, n_head_kv_total=4)


def test_bound_gating_capi_validation():
    ctx = make_ctx()
    assert ctx.set_qg_bound(1, 129, 0, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_qg_bound(1, 0, 1025, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_qg_bound(2, 4, 0, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_qg_bound(1, -1, 0, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_qg_bound(1, 4, -1, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_qg_bound(1, 4, 0, -1) == epsp.INVALID_ARGUMENT
    assert ctx.qg_bound() == 0
    assert ctx.set_qg_bound(1, 4, 0, 0) == epsp.OK
    assert ctx.qg_bound() == 1
    assert ctx.set_qg_bound(1, 128, 1024, 7) == epsp.OK
    assert ctx.set_qg_bound(0, 0, 0, 0) == epsp.OK
    assert ctx.qg_bound() == 0
    # null context
    assert epsp.lib.ep_sp_set_qg_bound(None, 1, 4, 0, 0) == epsp.INVALID_ARGUMENT
    assert epsp.lib.ep_sp_get_qg_bound(None) == 0
    assert epsp.lib.ep_sp_get_prefill_mode(None) == 0
    assert epsp.lib.ep_sp_get_ffn_skip(None) == 0


def test_ext_and_k_matrix_rules():
    ctx = make_ctx()
    assert ctx.set_ext(2, 0, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_ext(1, -1, 0) == epsp.INVALID_ARGUMENT
    assert ctx.set_ext(1, 0, -1) == epsp.INVALID_ARGUMENT
    # shared (reference) mode rejects a k-matrix
    assert ctx.set_k_matrix([4] * 8) == epsp.INVALID_ARGUMENT
    assert ctx.set_ext(1, 128, 0) == epsp.OK
    assert ctx.set_k_matrix([4] * 7) == epsp.INVALID_ARGUMENT          # wrong length
    assert ctx.set_k_matrix([4] * 7 + [0]) == epsp.INVALID_ARGUMENT    # element 0
    assert ctx.set_k_matrix([4] * 7 + [-2]) == epsp.INVALID_ARGUMENT   # element < -1
    assert ctx.set_k_matrix([4] * 7 + [-1]) == epsp.OK
    assert ctx.k_matrix_size() == 8
    assert ctx.set_k_matrix([]) == epsp.OK
    assert ctx.k_matrix_size() == 0
    assert ctx.set_k_matrix([3] * 8) == epsp.OK
    assert ctx.set_ext(0, 0, 4096) == epsp.OK  # back to shared mode clears it
    assert ctx.k_matrix_size() == 0


def test_ffn_skip_mask_truncation():
    ctx = make_ctx(n_layer=4)
    ctx.set_ffn_skip(0xFF)
    assert ctx.ffn_skip() == 0xF
    big = make_ctx(n_layer=64)
    big.set_ffn_skip(0xFF)
    assert big.ffn_skip() == 0  # ffn patch :77-82: n_layer >= 64 forces 0
    ctx.set_prefill_mode(True)
    assert ctx.prefill_mode() == 1
    ctx.set_prefill_mode(False)
    assert ctx.prefill_mode() == 0


def test_compute_without_device_fails_loudly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    ctx = make_ctx()
    assert ctx.reserve() == epsp.UNAVAILABLE
    assert "no CUDA device" in ctx.last_error()


def test_new_entry_points_validate_before_any_device_work():
    """Append, head-range selection and exchange calls reject bad arguments
    with rc 2 on the host, before touching a device; valid arguments on a
    machine without a GPU fail with rc 13 (Unavailable), never silently."""
    import ctypes

    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    lib = epsp.lib
    ctx = make_ctx()
    h = ctx.h
    fake = ctypes.c_void_p(4096)  # never dereferenced on the host
    # ep_sp_append_kv: layer, rows, range, nulls
    assert lib.ep_sp_append_kv(h, 99, fake, fake, 16, fake, fake, 0, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_append_kv(h, 0, fake, fake, 0, fake, fake, 0, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_append_kv(h, 0, fake, fake, 16, fake, fake, -1, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_append_kv(h, 0, None, fake, 16, fake, fake, 0, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_append_kv(h, 0, fake, fake, 16, fake, fake, 0, None) == epsp.UNAVAILABLE
    # ep_sp_select_heads: empty or out-of-range head ranges
    assert lib.ep_sp_select_heads(h, 0, fake, fake, fake, 64, 64, 1, 1, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_select_heads(h, 0, fake, fake, fake, 64, 64, 0, 99, None) == epsp.INVALID_ARGUMENT
    # exchange: nothing allocated or attached yet
    bases = (ctypes.c_void_p * 1)(fake)
    assert lib.ep_sp_xchg_attach(h, 1, 0, bases) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_xchg_wait(h, 0, 1, None) == epsp.INVALID_ARGUMENT
    assert lib.ep_sp_attend_rows_xchg(h, 0, 64, 64, 0, 64, 0, None) == epsp.INVALID_ARGUMENT
    base = ctypes.c_void_p()
    assert lib.ep_sp_xchg_alloc(h, 0, 2, ctypes.byref(base), None) == epsp.INVALID_ARGUMENT   # rows
    assert lib.ep_sp_xchg_alloc(h, 64, 65, ctypes.byref(base), None) == epsp.INVALID_ARGUMENT  # slots


def test_query_blocks():
    ctx = make_ctx()
    assert ctx.query_blocks(4096) == (0, 1)
    assert ctx.set_ext(1, 512, 0) == 0
    assert ctx.query_blocks(4096) == (0, 8)
    assert ctx.query_blocks(4100) == (0, 9)
    assert ctx.query_blocks(0)[0] == epsp.INVALID_ARGUMENT


def test_error_names():
    names = {0: "Ok", 2: "InvalidArgument", 6: "Prefill", 9: "Unsupported", 10: "OutOfMemory", 11: "Io",
             12: "Internal", 13: "Unavailable"}
    for rc, n in names.items():
        assert epsp.error_name(rc) == n
    ref = oracle.load_ref()
    if ref is not None:
        for rc in range(0, 15):
            assert epsp.error_name(rc) == ref.ref_error_code_name(rc).decode()


# ---------------------------------------------------------------- chunk plan
CHUNK_CASES = [(8192, 512, 512), (8000, 512, 512), (1000, 512, 128), (1000, 0, 128), (1000, 0, 2048),
               (5000, 0, 2048), (1000, 1000, 2048), (1000, 1000, 128), (1, 512, 128), (65536, 0, 4096),
               (131072, 0, 8192), (4096, 4096, 4096), (7, 3, 2), (100, 7, 100)]


def test_chunk_scheduler_reference_cases():
    rc, r = epsp.chunk_plan(8192, 512, 512)
    assert rc == 0 and len(r) == 16 and r[0] == (0, 512) and r[-1] == (7680, 8192)
    rc, r = epsp.chunk_plan(8000, 512, 512)
    assert len(r) == 16 and r[-1][1] - r[-1][0] == 320
    rc, r = epsp.chunk_plan(1000, 0, 2048)
    assert r == [(0, 1000)]
    rc, r = epsp.chunk_plan(5000, 0, 2048)
    assert [b - a for a, b in r] == [2048, 2048, 904]
    rc, r = epsp.chunk_plan(1000, 1000, 128)
    assert r == [(0, 1000)]
    assert epsp.chunk_plan(0, 512, 512)[0] == epsp.INVALID_ARGUMENT
    assert epsp.chunk_plan(100, 512, 0)[0] == epsp.INVALID_ARGUMENT


@pytest.mark.parametrize("case", CHUNK_CASES)
def test_chunk_plan_matches_reference_build(case):
    ours = epsp.chunk_plan(*case)
    assert oracle.chunk_plan(*case) == ours
    ref = oracle.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import ctypes

    buf = (ctypes.c_uint32 * (1 << 18))()
    n = ctypes.c_int32()
    rc = ref.ref_chunk_plan(*case, buf, 1 << 17, ctypes.byref(n))
    assert rc == ours[0]
    assert [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)] == ours[1]


# ------------------------------------------------------------------ FFN skip
def test_ffn_skip_reference_cases():
    assert epsp.ffn_auto_mask(28, 0.25) == (0, sum(1 << l for l in (0, 4, 8, 12, 16, 20, 24)))
    assert epsp.ffn_auto_mask(28, 0.0) == (0, 0)
    assert epsp.ffn_auto_mask(28, 1.0) == (0, (1 << 28) - 1)
    assert epsp.ffn_parse("0,3-5", 28) == (0, 1 | 8 | 16 | 32, "")
    assert epsp.ffn_parse(" 2 , 2 ", 28)[:2] == (0, 4)
    assert epsp.ffn_parse("50%", 28)[1] == sum(1 << (2 * i) for i in range(14))
    assert epsp.ffn_parse("0-100", 28) == (0, (1 << 28) - 1, "mask-bit-out-of-range")
    for bad in ("", "abc", "1,,2", "-1", "x%"):
        assert epsp.ffn_parse(bad, 28)[0] == epsp.INVALID_ARGUMENT, bad
    assert epsp.ffn_parse("0", 0)[0] == epsp.INVALID_ARGUMENT
    assert epsp.ffn_parse("0", 65)[0] == epsp.INVALID_ARGUMENT
    for n, r in ((0, 0.25), (65, 0.25), (28, -0.1), (28, 1.1)):
        assert epsp.ffn_auto_mask(n, r)[0] == epsp.INVALID_ARGUMENT


FFN_SPECS = ["0,3-5", " 2 , 2 ", "50%", "0-100", "5-2", "", "abc", "1,,2", "-1", "x%", "12.5%", "63", "1-1",
             "+3", "7,", "100%", "0%", "33.3%"]


@pytest.mark.parametrize("spec", FFN_SPECS)
@pytest.mark.parametrize("n_layer", [1, 24, 28, 32, 64])
def test_ffn_parse_matches_reference_build(spec, n_layer):
    ref = oracle.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import ctypes

    out = ctypes.c_uint64()
    warn = ctypes.create_string_buffer(64)
    rc = ref.ref_ffn_parse(spec.encode(), n_layer, ctypes.byref(out), warn, 64)
    ours = epsp.ffn_parse(spec, n_layer)
    assert ours[0] == rc
    if rc == 0:
        assert ours[1] == out.value and ours[2] == warn.value.decode()


@pytest.mark.parametrize("n_layer", [1, 7, 24, 28, 32, 64])
def test_ffn_auto_mask_matches_reference_build(n_layer):
    ref = oracle.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import ctypes

    for ratio in (0.0, 0.1, 0.25, 0.3333, 0.5, 0.85, 1.0):
        out = ctypes.c_uint64()
        rc = ref.ref_ffn_auto_mask(n_layer, ratio, ctypes.byref(out))
        ours = epsp.ffn_auto_mask(n_layer, ratio)
        assert ours[0] == rc
        if rc == 0:
            assert ours[1] == out.value


# -------------------------------------------------------------------- config
def test_bound_gating_config_parse(tmp_path):
    p = tmp_path / "bound.conf"
    p.write_text("qg_bound = true\nqg_sel_pages = 16\nqg_local_rows = 512\nqg_pool_pages = 4\n")
    rc, o = epsp.parse_config(str(p))
    assert rc == 0 and o.enable_qg_bound == 1 and o.qg_sel_pages == 16 and o.qg_local_rows == 512
    assert o.qg_pool_pages == 4
    # defaults: off, 8 pages, ubatch-sized window, no pool pages
    d = epsp.PrefillOptions(0, 1, 0, 8, 0, 0)
    assert (d.enable_qg_bound, d.qg_sel_pages, d.qg_local_rows, d.qg_pool_pages) == (0, 8, 0, 0)
    bad = tmp_path / "bad.conf"
    bad.write_text("qg_sel_pages = 129\n")
    assert epsp.parse_config(str(bad))[0] == epsp.INVALID_ARGUMENT
    for text in ("qg_local_rows = 32769\n", "qg_pool_pages = 4097\n", "qg_bound = maybe\n", "qg_sel_pages = -1\n",
                 "qg_sel_pages\n"):
        bad.write_text(text)
        assert epsp.parse_config(str(bad))[0] == epsp.INVALID_ARGUMENT, text
    ok = tmp_path / "ok.conf"
    ok.write_text("# comment\nmodel = x.gguf\nqg_bound = on  # trailing\nqg_local_rows = 32768\n")
    rc, o = epsp.parse_config(str(ok))
    assert rc == 0 and o.enable_qg_bound == 1 and o.qg_local_rows == 32768
    assert epsp.parse_config(str(tmp_path / "missing.conf"))[0] == epsp.IO
