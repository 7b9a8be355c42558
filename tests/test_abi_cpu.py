"""The C-ABI library on a host without a GPU: it loads, exports every entry
point the header declares, and rejects bad arguments on the host (before any
CUDA call) with the documented return codes and a message."""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lsrm_sparse.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[A-Za-z_][\w \*]*?\b(lsrm_\w+)\s*\(", text, flags=re.M)))


def _header_define(name):
    m = re.search(rf"#define\s+{name}\s+\(?(-?\w+)\)?", open(HEADER).read())
    return int(m.group(1), 0)


@pytest.fixture(scope="module")
def lib():
    from lsrm_sparse import _lib

    if not os.path.exists(_lib.LIB_PATH):
        if shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"):
            pytest.skip("library not built and nvcc absent")
        subprocess.run(["python", os.path.join(ROOT, "large-sparse-reconstruction-model_b200", "build.py")],
                       check=True)
    return _lib


def test_header_declares_the_expected_entry_points():
    names = _declared()
    assert len(names) >= 21
    for must in ("lsrm_select_attn_fwd", "lsrm_select_attn_bwd", "lsrm_select_attn_fwd_noalloc", "lsrm_block_topk",
                 "lsrm_dense_attn_fwd", "lsrm_dense_attn_bwd", "lsrm_block_mean_fwd", "lsrm_gate_merge_fwd"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    declared = _declared()
    h = lib.lib()
    missing = [n for n in declared if not hasattr(h, n)]
    assert not missing, missing
    # the ctypes table binds exactly the header's entry points
    assert sorted(lib.EXPORTED) == declared
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", lib.LIB_PATH], capture_output=True, text=True).stdout
        exported = {l.split()[-1] for l in out.splitlines() if l.strip()}
        assert set(declared) <= exported


def test_abi_version_matches_header(lib):
    assert lib.lib().lsrm_abi_version() == _header_define("LSRM_ABI_VERSION")


def _meta(total=256, blocks=4):
    return lib_mod().Varlen(1, total, total, blocks, None, None, None, None)


def lib_mod():
    from lsrm_sparse import _lib

    return _lib


def _shape(Hq=4, Hkv=2, D=64, dtype=1):
    L = lib_mod()
    return L.AttnShape(Hq, Hkv, D, dtype, Hq * D, Hkv * D, 0.0)


def _fwd(lib, meta, shape, topk=4, ws=None, ws_bytes=0):
    h = lib.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: every case fails host validation first
    return h.lsrm_select_attn_fwd(ctypes.byref(meta), ctypes.byref(shape), p, p, p, p, topk, None, 0, p, p, ws,
                                  ws_bytes, None, None)


@pytest.mark.parametrize("bad,code,msg", [
    (dict(D=48), "LSRM_ERR_INVALID_ARG", "head_dim"),
    (dict(dtype=7), "LSRM_ERR_INVALID_ARG", "dtype"),
    (dict(Hq=6, Hkv=2), "LSRM_ERR_INVALID_ARG", "power of two"),
    (dict(Hq=5, Hkv=2), "LSRM_ERR_INVALID_ARG", "multiple"),
])
def test_select_fwd_rejects_bad_shapes_on_host(lib, bad, code, msg):
    rc = _fwd(lib, _meta(), _shape(**bad))
    assert rc == _header_define(code)
    assert msg in lib.lib().lsrm_last_error().decode()


def test_select_fwd_rejects_topk_and_small_workspace(lib):
    rc = _fwd(lib, _meta(), _shape(), topk=0)
    assert rc == _header_define("LSRM_ERR_INVALID_ARG")
    assert "topk" in lib.lib().lsrm_last_error().decode()
    rc = _fwd(lib, _meta(), _shape(), topk=4, ws=ctypes.c_void_p(256), ws_bytes=8)
    assert rc == _header_define("LSRM_ERR_WORKSPACE")
    assert "workspace" in lib.lib().lsrm_last_error().decode()


def test_workspace_queries_are_host_only_and_grow_with_the_problem(lib):
    h = lib.lib()
    small = h.lsrm_select_workspace_bytes(ctypes.byref(_meta(1024, 8)), ctypes.byref(_shape()), 8, 0)
    big = h.lsrm_select_workspace_bytes(ctypes.byref(_meta(65536, 400)), ctypes.byref(_shape()), 16, 0)
    assert 0 < small < big
    assert h.lsrm_select_workspace_bytes(ctypes.byref(_meta()), ctypes.byref(_shape(D=48)), 8, 0) == 0
    for mode in (0, 1, 2):
        assert h.lsrm_dense_workspace_bytes(ctypes.byref(_meta(4096, 32)), ctypes.byref(_shape()), mode) > 0


def test_dense_workspace_covers_regrouped_heads(lib):
    """Dense branches with several query heads per kv head run over kv heads
    repeated to one query head each: the workspace adds the repeated k / v and
    their gradients (4 x rows x Hq x D x 2 bytes at least)."""
    h = lib.lib()
    meta = _meta(4096, 64)
    for mode in (0, 1, 2):
        g1 = h.lsrm_dense_workspace_bytes(ctypes.byref(meta), ctypes.byref(_shape(Hq=4, Hkv=4)), mode)
        g8 = h.lsrm_dense_workspace_bytes(ctypes.byref(meta), ctypes.byref(_shape(Hq=16, Hkv=2)), mode)
        rows = 64 if mode == 0 else 4096
        assert 0 < g1 < g8 and g8 >= 4 * rows * 16 * 64 * 2


def test_noalloc_scratch_bound_is_the_header_constant(lib):
    m = re.search(r"#define\s+LSRM_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", open(HEADER).read())
    assert m and int(m.group(1)) << int(m.group(2)) == 16 << 20


def test_noalloc_rejects_an_oversized_plan_on_host(lib):
    """The size check of the allocation-free forward runs before any CUDA
    call: a per-token selection over 32768 queries, 4096 blocks and top-64
    needs far more than the fixed scratch (the pointers are never used)."""
    h = lib.lib()
    p = ctypes.c_void_p(256)
    meta = _meta(32768, 4096)
    shape = _shape(Hq=4, Hkv=4)
    rc = h.lsrm_select_attn_fwd_noalloc(ctypes.byref(meta), ctypes.byref(shape), p, p, p, p, 64, None, 0, p, p,
                                        None, None)
    assert rc == _header_define("LSRM_ERR_WORKSPACE")
    assert "plan scratch" in h.lsrm_last_error().decode()
    # a bad shape is still reported as such, before the size check
    rc = h.lsrm_select_attn_fwd_noalloc(ctypes.byref(meta), ctypes.byref(_shape(D=48)), p, p, p, p, 64, None, 0, p,
                                        p, None, None)
    assert rc == _header_define("LSRM_ERR_INVALID_ARG")


def test_ops_fail_loudly_without_a_device():
    import torch

    from lsrm_sparse import ops

    if torch.cuda.is_available():
        pytest.skip("host-only check")
    q = torch.zeros(8, 2, 64, dtype=torch.bfloat16)
    cu = torch.tensor([0, 8], dtype=torch.int32)
    meta = ops.Meta(cu, cu, torch.tensor([0, 1], dtype=torch.int32), cu)
    with pytest.raises(Exception):
        ops.select_attn_fwd(q, q, q, torch.zeros(2, 8, 1, dtype=torch.int32), meta)


def test_view_block_topk_workspace_query_validates_geometry(lib):
    """lsrm_view_block_topk_workspace_bytes runs on the host: a positive size
    for a supported view geometry, 0 with a message for the unsupported ones
    (window > 25, views x window > 512, unequal blocks per side)."""
    h = lib.lib()
    ok = h.lsrm_view_block_topk_workspace_bytes(1, 16, 768, 768, 384, 8, 8, 9, 131072)
    assert ok > 131072 * 16 * 9 * 8  # at least the candidate lists
    assert h.lsrm_view_block_topk_workspace_bytes(1, 16, 768, 768, 384, 8, 8, 26, 1024) == 0
    assert "window" in h.lsrm_last_error().decode()
    assert h.lsrm_view_block_topk_workspace_bytes(1, 64, 768, 768, 384, 8, 8, 9, 1024) == 0
    assert "512" in h.lsrm_last_error().decode()
    assert h.lsrm_view_block_topk_workspace_bytes(1, 4, 768, 512, 384, 8, 8, 4, 1024) == 0
    assert "blocks per side" in h.lsrm_last_error().decode()


def test_new_entry_points_reject_bad_arguments_on_host(lib):
    """Argument checks of the map, token and norm entry points run before any
    launch (the dummy pointers below are never dereferenced)."""
    h = lib.lib()
    p = ctypes.c_void_p(16)
    bad = _header_define("LSRM_ERR_INVALID_ARG")
    # top-k beyond 64
    assert h.lsrm_volume_block_topk(p, 100, p, p, 1, 32, 0.5, 65, p, p, p, None) == bad
    assert "topk" in h.lsrm_last_error().decode()
    assert h.lsrm_points_volume_block_topk(p, p, 100, p, 100, p, p, 1, 32, 0.5, 0, p, p, p, None) == bad
    # surface grid not a multiple of the patch grid
    assert h.lsrm_image_token_points(p, 10, p, p, 1, 1, 30, 16, p, p, None) == bad
    assert "multiple" in h.lsrm_last_error().decode()
    # head_dim outside 16..256 powers of two; heads not divisible by the world size
    assert h.lsrm_head_layernorm_pack(10, 16, 48, 1, 1, 16 * 48, 1e-5, p, p, None) == bad
    assert "head_dim" in h.lsrm_last_error().decode()
    assert h.lsrm_head_layernorm_pack(10, 6, 64, 4, 1, 6 * 64, 1e-5, p, p, None) == bad
    # misaligned coordinates
    assert h.lsrm_image_sort_keys(10, ctypes.c_void_p(20), 2, 16, 4, p, None) == bad
    assert "aligned" in h.lsrm_last_error().decode()


def test_block_topk_workspace_query_and_host_rejection(lib):
    """The per-query-block scorer needs a workspace (key norms and score
    bounds), the per-token scorer none; a call with a short workspace is
    rejected on the host before anything runs."""
    h = lib.lib()
    meta, shape = _meta(4096, 64), _shape(Hq=8, Hkv=8)
    per_qb = h.lsrm_block_topk_workspace_bytes(ctypes.byref(meta), ctypes.byref(shape), 8, 64)
    assert per_qb >= 8 * 64 * 64 * 2 * 4  # [Hkv, nqb, 2, blocks] fp32 bounds at least
    assert h.lsrm_block_topk_workspace_bytes(ctypes.byref(meta), ctypes.byref(shape), 8, 0) == 0
    assert h.lsrm_block_topk_workspace_bytes(ctypes.byref(meta), ctypes.byref(_shape(D=48)), 8, 64) == 0
    p = ctypes.c_void_p(256)
    rc = h.lsrm_block_topk(ctypes.byref(meta), ctypes.byref(shape), p, p, p, 8, p, 64, 1, 0.0, p, p, 1024, p, None)
    assert rc == _header_define("LSRM_ERR_WORKSPACE")
    assert "workspace" in h.lsrm_last_error().decode()


def test_qkv_norm_host_checks():
    """lsrm_qkv_norm_fwd / _bwd reject bad shapes and segment tables on the
    host, before any CUDA call, with a message naming the problem."""
    from lsrm_sparse import _lib as lib

    h = lib.lib()
    one = (lib.QkvSegment * 1)(lib.QkvSegment(128, 0, 16, None))
    assert h.lsrm_qkv_norm_fwd(10, 100, 128, 64, 16, 100, 16, None, one, 1, 1e-5, None, 16, None) == -1
    assert "multiple of 64" in h.lsrm_last_error().decode()
    assert h.lsrm_qkv_norm_fwd(10, 128, 128, 48, 16, 128, 16, None, one, 1, 1e-5, None, 16, None) == -1
    assert "head_dim" in h.lsrm_last_error().decode()
    short = (lib.QkvSegment * 1)(lib.QkvSegment(64, 0, 16, None))
    assert h.lsrm_qkv_norm_fwd(10, 128, 128, 64, 16, 128, 16, None, short, 1, 1e-5, None, 16, None) == -1
    assert "segments cover 64 columns" in h.lsrm_last_error().decode()
    norm_no_rstd = (lib.QkvSegment * 1)(lib.QkvSegment(128, 0, None, 16))
    assert h.lsrm_qkv_norm_fwd(10, 128, 128, 64, 16, 128, 16, None, norm_no_rstd, 1, 1e-5, None, 16, None) == -1
    assert "rstd is required" in h.lsrm_last_error().decode()
    assert h.lsrm_qkv_norm_fwd(0, 128, 128, 64, 16, 128, 16, None, one, 1, 1e-5, None, 16, None) == 0
    g = (lib.QkvGradSegment * 1)(lib.QkvGradSegment(128, 0, None, None, 16))
    assert h.lsrm_qkv_norm_bwd(10, 128, 64, g, 1, None, 16, None) == -1
    assert "needs out_norm and rstd" in h.lsrm_last_error().decode()
