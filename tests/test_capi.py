"""The C-ABI library loads on a CPU-only host and exports every function include/pbk.h
declares; the ctypes structures match the header's layout. No compute calls."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADER_DIR = os.path.join(ROOT, "include")


def _declared_functions() -> set[str]:
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(pbk_\w+)\s*\(", text, flags=re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from pseudobrain_b200 import build
    build.build()
    return ctypes.CDLL(build.LIB_PATH)


def test_header_declares_entry_points():
    names = _declared_functions()
    assert {"pbk_abi_version", "pbk_status_string", "pbk_device_check", "pbk_gdn_decode"} <= names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in sorted(_declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"declared in include/ but not exported: {missing}"


def test_ctypes_binding_covers_the_header(lib):
    from pseudobrain_b200 import _capi
    assert set(_capi.SIGNATURES) == _declared_functions()


def test_abi_version_and_status_strings(lib):
    from pseudobrain_b200 import _capi
    assert _capi.LIB.pbk_abi_version() == _capi.PBK_ABI_VERSION
    assert _capi.LIB.pbk_status_string(0) == b"ok"
    assert _capi.LIB.pbk_status_string(-7) == b"device-side wait timed out"


@pytest.mark.parametrize("cname,pyname", [("pbk_gdn_desc", "PbkGdnDesc"), ("pbk_quest_desc", "PbkQuestDesc"),
                                          ("pbk_swa_desc", "PbkSwaDesc"), ("pbk_view", "PbkView"),
                                          ("pbk_conv_desc", "PbkConvDesc"), ("pbk_gating_desc", "PbkGatingDesc"),
                                          ("pbk_out_norm_desc", "PbkOutNormDesc"),
                                          ("pbk_quest_levels", "PbkQuestLevels"),
                                          ("pbk_rope_gather_desc", "PbkRopeGatherDesc"),
                                          ("pbk_archive_write_desc", "PbkArchiveWriteDesc"),
                                          ("pbk_decode_ext", "PbkDecodeExt"), ("pbk_token_desc", "PbkTokenDesc"),
                                          ("pbk_gdn_layer_desc", "PbkGdnLayerDesc")])
def test_descriptor_layout_matches_header(cname, pyname):
    """Offsets of every field of the ctypes mirror equal the C struct's (checked by
    compiling a probe against include/pbk.h)."""
    import subprocess
    import tempfile
    from pseudobrain_b200 import _capi
    cls = getattr(_capi, pyname)
    fields = [f for f, _ in cls._fields_]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"pbk.h\"\nint main(void){\n"
    src += "".join(f'printf("%zu\\n", offsetof({cname}, {f}));\n' for f in fields)
    src += f'printf("%zu\\n", sizeof({cname})); return 0; }}\n'
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", HEADER_DIR, c, "-o", exe], check=True)
        got = [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(cls, f).offset for f in fields] + [ctypes.sizeof(cls)]
    assert got == want


def test_no_device_returns_error_without_launching(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    from pseudobrain_b200 import _capi
    assert _capi.LIB.pbk_device_check(0) == -5


def test_every_module_imports(lib):
    """The Python mirrors import on a host without a GPU (they fail only when called)."""
    import importlib
    for m in ("gated_deltanet", "gdn_prefill", "exact_memory", "transplant", "serving", "pertoken", "sharding",
              "synthetic"):
        importlib.import_module(f"pseudobrain_b200.{m}")


def test_noalloc_select_too_large_when_scores_are_given(lib):
    """With desc->scores given, only the segment and tile maxima go to the fixed array; a
    problem whose maxima alone exceed it returns PBK_ERR_TOO_LARGE on the host, before any
    device call (the pointers below are never dereferenced)."""
    from pseudobrain_b200 import _capi
    d = _capi.PbkQuestDesc()
    d.nq, d.t, d.h, d.kv, d.d, d.page = 64, 1, 64, 64, 128, 16
    d.n_arch, d.budget = 65536 * 16, 256  # 64 x 64 rows of 65536 pages: 8.4M segment maxima
    fake = 1 << 20                         # 16-byte aligned, never read
    d.q = d.kmax = d.kmin = fake
    d.pages = fake
    d.scores = fake
    d.q_stride_n, d.q_stride_t, d.q_stride_h = 64 * 128, 64 * 128, 128
    d.bnd_stride_kv, d.bnd_stride_p = 65536 * 128, 128
    assert _capi.LIB.pbk_quest_select_noalloc(ctypes.byref(d), None) == _capi.PBK_ERR_TOO_LARGE


def test_token_entry_points_validate_on_the_host(lib):
    """The per-token selector's entry points reject bad shapes before touching the device."""
    from pseudobrain_b200 import _capi
    d = _capi.PbkTokenDesc(t=1, h=40, kv=1, d=128, n_pool=4, full=4)
    assert _capi.LIB.pbk_quest_token_scores(ctypes.byref(d), None) == -2  # 40 heads per key head
    d = _capi.PbkTokenDesc(t=1, h=8, kv=2, d=192, n_pool=4, full=4)
    assert _capi.LIB.pbk_quest_token_scores(ctypes.byref(d), None) == -2  # head dims 128 and 256 only
    d = _capi.PbkTokenDesc(t=1, h=8, kv=2, d=256, n_pool=4, full=4)
    assert _capi.LIB.pbk_quest_token_scores(ctypes.byref(d), None) == -1  # 256 is a shape; q is missing
    d = _capi.PbkTokenDesc(t=0, h=8, kv=2, d=128, n_pool=4, full=4)
    assert _capi.LIB.pbk_quest_token_rerank(ctypes.byref(d), None) == 0   # nothing to do
    assert _capi.LIB.pbk_quest_row_ranks(None, 20000, 1, 20000, None, 20000, None) == -2
    assert _capi.LIB.pbk_quest_row_ranks(None, 8, 1, 8, None, 8, None) == -1


def _layer_desc(hk=2, hv=8, width=4, t=16):
    """A pbk_gdn_layer_desc with 16-byte aligned fake pointers (never dereferenced: every case
    below is rejected on the host before any device call)."""
    from pseudobrain_b200 import _capi
    fake = 1 << 20
    c = (2 * hk + hv) * 128
    v = lambda sb, st, sh, dt=_capi.PBK_BF16: _capi.PbkView(fake, sb, st, sh, dt, 0)  # noqa: E731
    d = _capi.PbkGdnLayerDesc()
    d.batch, d.seqlen, d.hk, d.hv, d.width, d.l2mode = 2, t, hk, hv, width, 1
    d.l2_eps, d.norm_eps, d.scale, d.state_layout = 1e-6, 1e-5, 128 ** -0.5, _capi.PBK_STATE_KV
    d.qkv = v(t * c, c, 1)
    d.tail = v((width - 1) * c, c, 1)
    d.new_tail = v((width - 1) * c, c, 1)
    d.new_tail.data = fake + (1 << 16)
    d.conv_weight = d.a_log = d.dt_bias = d.o_norm = fake
    d.decay = v(t * 2 * hv, 2 * hv, 1)
    d.gate = v(t * hv * 128, hv * 128, 1)
    d.out = v(t * hv * 128, hv * 128, 128, _capi.PBK_F32)
    d.o_norm_dtype = _capi.PBK_F32
    d.state = fake
    d.state_slot_stride = hv * 128 * 128
    return d


def test_layer_entry_points_validate_on_the_host(lib):
    """pbk_gdn_decode_layer / pbk_gdn_prefill_layer reject what they cannot run before any
    device call: an in-place tail whose key head is shared by more than 8 value heads (one
    thread-block cluster per key head), an in-place tail in the prefill (read and written by
    different CTAs), fp32 or strided projection channels in the prefill, conv widths past 8,
    a missing or short workspace."""
    from pseudobrain_b200 import _capi
    L = _capi.LIB
    d = _layer_desc()
    assert L.pbk_gdn_prefill_layer_workspace(ctypes.byref(d)) > 0
    d.width = 9
    assert L.pbk_gdn_decode_layer(ctypes.byref(d), None) == _capi.PBK_ERR_SHAPE
    assert L.pbk_gdn_prefill_layer_workspace(ctypes.byref(d)) == 0
    d = _layer_desc(hk=1, hv=16)
    d.new_tail = d.tail  # in place, 16 value heads per key head
    assert L.pbk_gdn_decode_layer(ctypes.byref(d), None) == _capi.PBK_ERR_SHAPE
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), 1 << 20, 1 << 40, None) == _capi.PBK_ERR_INVALID
    d = _layer_desc()
    d.qkv.dtype = _capi.PBK_F32
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), 1 << 20, 1 << 40, None) == _capi.PBK_ERR_DTYPE
    d = _layer_desc()
    d.qkv.stride_h = 2
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), 1 << 20, 1 << 40, None) == _capi.PBK_ERR_ALIGN
    d = _layer_desc()
    need = L.pbk_gdn_prefill_layer_workspace(ctypes.byref(d))
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), None, need, None) == _capi.PBK_ERR_WORKSPACE
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), 1 << 20, need - 1, None) == _capi.PBK_ERR_WORKSPACE
    d.hv = 7  # not a multiple of the key heads
    assert L.pbk_gdn_decode_layer(ctypes.byref(d), None) == _capi.PBK_ERR_SHAPE
    d = _layer_desc()
    d.batch = 0  # nothing to do
    assert L.pbk_gdn_decode_layer(ctypes.byref(d), None) == _capi.PBK_OK
    assert L.pbk_gdn_prefill_layer(ctypes.byref(d), None, 0, None) == _capi.PBK_OK
