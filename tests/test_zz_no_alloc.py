"""GPU test of lsrm_select_attn_fwd_noalloc.

That entry point serves callers that may not allocate device memory: plugin
hosts that own every device allocation (an inference server's fixed arena,
another framework's operator interface) and latency-bound loops that must not
enter the driver allocator.  It keeps its selection plan in a fixed device
array inside the library, shared by all calls.  Here it is called through the
C ABI twice in a row, on two different problems, and each result must match
lsrm_select_attn_fwd (which uses a caller-provided workspace) within the bf16
tolerance of the other selection tests.  The file is named to be collected
last, and passes alone in a fresh process as well as after the other tests.
"""

import ctypes

import pytest
import torch

from tests.cases import random_problem

pytestmark = pytest.mark.gpu

ATOL_BF16 = 2e-2
LSRM_ERR_WORKSPACE = -5


def _noalloc(q, k, v, bt, meta, cqb):
    from lsrm_sparse import _lib, ops

    L = _lib.lib()
    vl = meta.struct(q.shape[0], k.shape[0])
    sh = ops._shape(q, k, None)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    nqb = 0 if cqb is None else cqb.numel() - 1
    rc = L.lsrm_select_attn_fwd_noalloc(
        ctypes.byref(vl), ctypes.byref(sh), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(bt.data_ptr()), bt.shape[-1],
        ctypes.c_void_p(cqb.data_ptr()) if cqb is not None else None, nqb, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(lse.data_ptr()), ctypes.c_void_p(err.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "lsrm_select_attn_fwd_noalloc")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out, lse


def _problem(seed, sbl, Hq, Hkv, D, topk, qblock):
    from lsrm_sparse import ops

    p = random_problem(seed, sbl, Hq, Hkv, D, topk, qblock=qblock)
    dev = "cuda"
    meta = ops.Meta(p["cu_seqlens"].to(dev), p["cu_seqlens"].to(dev), p["cu_seqblocks"].to(dev), p["cu_blk"].to(dev))
    cqb = p["cu_blk"].to(dev) if qblock else None
    return p["q"].to(dev), p["k"].to(dev), p["v"].to(dev), p["block_topk"].to(dev), meta, cqb


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    from lsrm_sparse import ops

    cases = [
        _problem(31, [[40, 70, 33, 90, 64, 21, 128, 55] * 4], 4, 2, 64, 4, False),
        _problem(32, [[64, 256, 100, 130, 77, 190, 64], [30, 12, 99]], 2, 2, 32, 3, True),
    ]
    for q, k, v, bt, meta, cqb in cases:
        got, got_lse = _noalloc(q, k, v, bt, meta, cqb)
        ref, ref_lse, _ = ops.select_attn_fwd(q, k, v, bt, meta, cu_query_blocks=cqb)
        torch.cuda.synchronize()
        assert ops.read_errors() == 0
        assert (got.float() - ref.float()).abs().max().item() <= ATOL_BF16
        assert (got_lse - ref_lse).abs().max().item() <= 1e-2


def test_noalloc_rejects_problems_beyond_its_scratch():
    from lsrm_sparse import _lib, ops

    # per-token selection with many blocks: the plan needs far more than 16 MiB
    Hkv, D, N, nb, topk = 4, 64, 32768, 4096, 64
    dev = "cuda"
    q = torch.zeros(N, Hkv, D, dtype=torch.bfloat16, device=dev)
    k = torch.zeros_like(q)
    bt = torch.full((Hkv, N, topk), -1, dtype=torch.int32, device=dev)
    cu_seq = torch.tensor([0, N], dtype=torch.int32, device=dev)
    cu_sb = torch.tensor([0, nb], dtype=torch.int32, device=dev)
    cu_blk = torch.arange(0, N + 1, N // nb, dtype=torch.int32, device=dev)
    meta = ops.Meta(cu_seq, cu_seq, cu_sb, cu_blk)
    L = _lib.lib()
    vl = meta.struct(N, N)
    sh = ops._shape(q, k, None)
    out = torch.empty_like(q)
    lse = torch.empty(Hkv, N, dtype=torch.float32, device=dev)
    rc = L.lsrm_select_attn_fwd_noalloc(
        ctypes.byref(vl), ctypes.byref(sh), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(bt.data_ptr()), topk, None, 0, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(lse.data_ptr()), None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == LSRM_ERR_WORKSPACE
    assert "plan scratch" in L.lsrm_last_error().decode()
