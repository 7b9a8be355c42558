"""Thin torch-tensor wrappers over the C ABI (include/lsrm_sparse.h).

Tensors must live on a CUDA device; every call enqueues on the current torch
stream and never synchronises, except where a function says so.  Device-side
error bits accumulate in a per-device word that ``read_errors()`` returns and
clears (with a synchronisation).
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import AttnShape, Varlen, check

_ERR_WORDS = {}


def _err_word(device: torch.device) -> torch.Tensor:
    key = device.index if device.index is not None else torch.cuda.current_device()
    w = _ERR_WORDS.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR_WORDS[key] = w
    return w


def read_errors(device=None, clear: bool = True) -> int:
    """Synchronise and return the OR of device error bits (LSRM_ERR_*)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    w = _err_word(dev)
    v = int(w.item())
    if clear and v:
        w.zero_()
    return v


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return 1
    if t.dtype == torch.float16:
        return 0
    raise TypeError(f"only bf16/fp16 are supported, got {t.dtype}")


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


class Meta:
    """Device int32 metadata of one varlen problem (keeps the tensors alive)."""

    def __init__(self, cu_seqlens_q, cu_seqlens_k, cu_seqblocks, cu_block_include_tokens, total_q=None, total_k=None):
        self.cu_seqlens_q = _i32(cu_seqlens_q)
        self.cu_seqlens_k = _i32(cu_seqlens_k)
        self.cu_seqblocks = _i32(cu_seqblocks)
        self.cu_block_include_tokens = _i32(cu_block_include_tokens)
        self.num_seqs = self.cu_seqlens_q.numel() - 1
        self.num_blocks = self.cu_block_include_tokens.numel() - 1
        self.total_q = int(total_q) if total_q is not None else None
        self.total_k = int(total_k) if total_k is not None else None

    def struct(self, total_q: int, total_k: int) -> Varlen:
        return Varlen(
            self.num_seqs, int(total_q), int(total_k), self.num_blocks,
            self.cu_seqlens_q.data_ptr(), self.cu_seqlens_k.data_ptr(), self.cu_seqblocks.data_ptr(),
            self.cu_block_include_tokens.data_ptr(),
        )


def _shape(q: torch.Tensor, k: torch.Tensor, softmax_scale: Optional[float]) -> AttnShape:
    assert q.dim() == 3 and k.dim() == 3, "q/k must be [tokens, heads, head_dim]"
    assert q.stride(-1) == 1 and q.stride(-2) == q.shape[-1], "q must have contiguous [heads, head_dim]"
    assert k.stride(-1) == 1 and k.stride(-2) == k.shape[-1], "k must have contiguous [heads, head_dim]"
    return AttnShape(
        q.shape[1], k.shape[1], q.shape[2], _dtype_code(q), q.stride(0), k.stride(0),
        float(softmax_scale) if softmax_scale else 0.0,
    )


def _rows(*ts):
    """The kernels address q, out, dout and dq with q's token stride and k, v,
    dk and dv with k's: hand them dense [tokens, heads, head_dim] tensors (a
    no-op for contiguous inputs; a copy for any other layout)."""
    return tuple(t if t is None or t.is_contiguous() else t.contiguous() for t in ts)


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# Selected-block attention
# ---------------------------------------------------------------------------


def _check_block_topk(block_topk, num_kv_heads: int, rows: int):
    """The kernels read block_topk as [num_kv_heads, rows, topk]: reject any
    other shape before it reaches them."""
    if block_topk.dim() != 3 or tuple(block_topk.shape[:2]) != (num_kv_heads, rows):
        raise ValueError(f"block_topk must be [num_kv_heads={num_kv_heads}, {rows}, topk], got "
                         f"{tuple(block_topk.shape)}")


def select_attn_fwd(q, k, v, block_topk, meta: Meta, softmax_scale=None, cu_query_blocks=None,
                    workspace: Optional[torch.Tensor] = None):
    """Returns (out [Nq,Hq,D], lse_log2 [Hq,Nq] fp32, workspace)."""
    L = _lib.lib()
    assert q.dtype == k.dtype == v.dtype
    q, k, v = _rows(q, k, v)
    block_topk = _i32(block_topk)
    topk = block_topk.shape[-1]
    nqb = 0 if cu_query_blocks is None else cu_query_blocks.numel() - 1
    _check_block_topk(block_topk, k.shape[1], nqb if nqb > 0 else q.shape[0])
    cqb = _i32(cu_query_blocks) if cu_query_blocks is not None else None
    vl = meta.struct(q.shape[0], k.shape[0])
    sh = _shape(q, k, softmax_scale)
    need = L.lsrm_select_workspace_bytes(ctypes.byref(vl), ctypes.byref(sh), topk, nqb)
    if need == 0:
        raise _lib.LsrmError("invalid selection problem: " + L.lsrm_last_error().decode())
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, q.device)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    rc = L.lsrm_select_attn_fwd(
        ctypes.byref(vl), ctypes.byref(sh), _ptr(q), _ptr(k), _ptr(v), _ptr(block_topk), topk, _ptr(cqb), nqb,
        _ptr(out), _ptr(lse), _ptr(workspace), workspace.numel(), _ptr(_err_word(q.device)), _stream(),
    )
    check(rc, "lsrm_select_attn_fwd")
    return out, lse, workspace


def select_attn_bwd(q, k, v, out, lse, dout, block_topk, meta: Meta, softmax_scale=None, cu_query_blocks=None,
                    workspace: Optional[torch.Tensor] = None):
    """Returns (dq, dk, dv)."""
    L = _lib.lib()
    q, k, v, out, dout = _rows(q, k, v, out, dout)
    block_topk = _i32(block_topk)
    topk = block_topk.shape[-1]
    nqb = 0 if cu_query_blocks is None else cu_query_blocks.numel() - 1
    _check_block_topk(block_topk, k.shape[1], nqb if nqb > 0 else q.shape[0])
    cqb = _i32(cu_query_blocks) if cu_query_blocks is not None else None
    vl = meta.struct(q.shape[0], k.shape[0])
    sh = _shape(q, k, softmax_scale)
    need = L.lsrm_select_workspace_bytes(ctypes.byref(vl), ctypes.byref(sh), topk, nqb)
    if workspace is None or workspace.numel() < need:
        workspace = _workspace(need, q.device)
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    delta = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    rc = L.lsrm_select_attn_bwd(
        ctypes.byref(vl), ctypes.byref(sh), _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse), _ptr(dout),
        _ptr(block_topk), topk, _ptr(cqb), nqb, _ptr(dq), _ptr(dk), _ptr(dv), _ptr(delta), _ptr(workspace),
        workspace.numel(), _ptr(_err_word(q.device)), _stream(),
    )
    check(rc, "lsrm_select_attn_bwd")
    return dq, dk, dv


# ---------------------------------------------------------------------------
# Dense-range branches
# ---------------------------------------------------------------------------

DENSE_COMPRESSED = _lib.DENSE_COMPRESSED
DENSE_INTRA_BLOCK = _lib.DENSE_INTRA_BLOCK
DENSE_SLIDING = _lib.DENSE_SLIDING


def dense_attn_fwd(q, k, v, meta: Meta, mode: int, window: int = 0, softmax_scale=None):
    """Returns (out, lse).  lse is natural-log for DENSE_COMPRESSED, log2
    otherwise; [Hq, Nq] fp32."""
    L = _lib.lib()
    q, k, v = _rows(q, k, v)
    vl = meta.struct(q.shape[0], k.shape[0])
    sh = _shape(q, k, softmax_scale)
    need = L.lsrm_dense_workspace_bytes(ctypes.byref(vl), ctypes.byref(sh), mode)
    if need == 0:
        raise _lib.LsrmError("invalid dense problem: " + L.lsrm_last_error().decode())
    ws = _workspace(need, q.device)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    rc = L.lsrm_dense_attn_fwd(ctypes.byref(vl), ctypes.byref(sh), mode, int(window), _ptr(q), _ptr(k), _ptr(v),
                               _ptr(out), _ptr(lse), _ptr(ws), ws.numel(), _ptr(_err_word(q.device)), _stream())
    check(rc, "lsrm_dense_attn_fwd")
    return out, lse


def dense_attn_bwd(q, k, v, out, lse, dout, meta: Meta, mode: int, window: int = 0, softmax_scale=None):
    L = _lib.lib()
    q, k, v, out, dout = _rows(q, k, v, out, dout)
    vl = meta.struct(q.shape[0], k.shape[0])
    sh = _shape(q, k, softmax_scale)
    need = L.lsrm_dense_workspace_bytes(ctypes.byref(vl), ctypes.byref(sh), mode)
    ws = _workspace(need, q.device)
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    delta = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    rc = L.lsrm_dense_attn_bwd(ctypes.byref(vl), ctypes.byref(sh), mode, int(window), _ptr(q), _ptr(k), _ptr(v),
                               _ptr(out), _ptr(lse), _ptr(dout), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(delta), _ptr(ws),
                               ws.numel(), _ptr(_err_word(q.device)), _stream())
    check(rc, "lsrm_dense_attn_bwd")
    return dq, dk, dv


def umma_selftest(a, b, p, v):
    L = _lib.lib()
    D = a.shape[1]
    c1 = torch.empty(128, 128, dtype=torch.float32, device=a.device)
    c2 = torch.empty(128, D, dtype=torch.float32, device=a.device)
    rc = L.lsrm_umma_selftest(D, _ptr(a), _ptr(b), _ptr(p), _ptr(v), _ptr(c1), _ptr(c2), _ptr(_err_word(a.device)),
                              _stream())
    check(rc, "lsrm_umma_selftest")
    return c1, c2


# ---------------------------------------------------------------------------
# Scoring, compression, gated merge
# ---------------------------------------------------------------------------


def block_topk(q, ck, lse_ln, topk: int, meta: Meta, cu_query_blocks=None, force_self: bool = False,
               sm_scale: Optional[float] = None):
    """Deterministic block selection; returns int32 [Hkv, rows, topk]."""
    L = _lib.lib()
    q, ck = _rows(q, ck)
    vl = meta.struct(q.shape[0], ck.shape[0])
    sh = _shape(q, ck, None)
    nqb = 0 if cu_query_blocks is None else cu_query_blocks.numel() - 1
    rows = nqb if nqb else q.shape[0]
    out = torch.empty(ck.shape[1], rows, topk, dtype=torch.int32, device=q.device)
    cqb = _i32(cu_query_blocks) if cu_query_blocks is not None else None
    lse_ln = lse_ln.float().contiguous()
    nbytes = L.lsrm_block_topk_workspace_bytes(ctypes.byref(vl), ctypes.byref(sh), int(topk), nqb)
    ws = _workspace(nbytes, q.device) if nbytes else None
    rc = L.lsrm_block_topk(ctypes.byref(vl), ctypes.byref(sh), _ptr(q), _ptr(ck), _ptr(lse_ln), int(topk), _ptr(cqb),
                           nqb, int(bool(force_self)), float(sm_scale) if sm_scale else 0.0, _ptr(out), _ptr(ws),
                           int(nbytes), _ptr(_err_word(q.device)), _stream())
    check(rc, "lsrm_block_topk")
    return out


def block_mean_fwd(x: torch.Tensor, cu_block_include_tokens: torch.Tensor) -> torch.Tensor:
    """x [N, C] (row stride may exceed C) -> [nb, C]."""
    L = _lib.lib()
    assert x.dim() == 2 and x.stride(1) == 1
    cu_ = _i32(cu_block_include_tokens)
    nb = cu_.numel() - 1
    out = torch.empty(nb, x.shape[1], dtype=x.dtype, device=x.device)
    rc = L.lsrm_block_mean_fwd(nb, x.shape[1], _dtype_code(x), _ptr(cu_), _ptr(x), x.stride(0), _ptr(out), _stream())
    check(rc, "lsrm_block_mean_fwd")
    return out


def block_mean_bwd(dout: torch.Tensor, cu_block_include_tokens: torch.Tensor, total_tokens: int) -> torch.Tensor:
    L = _lib.lib()
    dout = dout.contiguous()
    cu_ = _i32(cu_block_include_tokens)
    dx = torch.empty(total_tokens, dout.shape[1], dtype=dout.dtype, device=dout.device)
    rc = L.lsrm_block_mean_bwd(cu_.numel() - 1, dout.shape[1], _dtype_code(dout), _ptr(cu_), int(total_tokens),
                               _ptr(dout), _ptr(dx), _stream())
    check(rc, "lsrm_block_mean_bwd")
    return dx


def resnorm_mean_fwd(x, h, cu_block_include_tokens, eps: float = 1e-5, want_y: bool = False):
    """Returns (block_mean [nb, C], y or None, mean [N], rstd [N])."""
    L = _lib.lib()
    x = x.contiguous()
    h = h.contiguous()
    cu_ = _i32(cu_block_include_tokens)
    nb = cu_.numel() - 1
    N, C = x.shape
    out = torch.empty(nb, C, dtype=x.dtype, device=x.device)
    y = torch.empty_like(x) if want_y else None
    mean = torch.empty(N, dtype=torch.float32, device=x.device)
    rstd = torch.empty(N, dtype=torch.float32, device=x.device)
    rc = L.lsrm_resnorm_mean_fwd(nb, N, C, _dtype_code(x), _ptr(cu_), _ptr(x), _ptr(h), float(eps), _ptr(y),
                                 _ptr(out), _ptr(mean), _ptr(rstd), _stream())
    check(rc, "lsrm_resnorm_mean_fwd")
    return out, y, mean, rstd


def resnorm_mean_bwd(x, h, cu_block_include_tokens, mean, rstd, dout):
    L = _lib.lib()
    cu_ = _i32(cu_block_include_tokens)
    N, C = x.shape
    dr = torch.empty_like(x)
    rc = L.lsrm_resnorm_mean_bwd(cu_.numel() - 1, N, C, _dtype_code(x), _ptr(cu_), _ptr(x), _ptr(h), _ptr(mean),
                                 _ptr(rstd), _ptr(dout.contiguous()), _ptr(dr), _stream())
    check(rc, "lsrm_resnorm_mean_bwd")
    return dr


def _ptr_array(ts):
    arr = (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    return arr


def gate_merge_fwd(z, branches: Sequence[torch.Tensor], per_head: bool = False, head_dim: int = 0):
    L = _lib.lib()
    z = z.contiguous()
    branches = [b.contiguous() for b in branches]
    N, C = branches[0].shape
    out = torch.empty(N, C, dtype=branches[0].dtype, device=z.device)
    arr = _ptr_array(branches)
    rc = L.lsrm_gate_merge_fwd(N, C, len(branches), int(per_head), int(head_dim), _dtype_code(z), _ptr(z), arr,
                               _ptr(out), _stream())
    check(rc, "lsrm_gate_merge_fwd")
    return out


def gate_merge_bwd(z, branches: Sequence[torch.Tensor], dout, per_head: bool = False, head_dim: int = 0):
    L = _lib.lib()
    z = z.contiguous()
    branches = [b.contiguous() for b in branches]
    N, C = branches[0].shape
    dz = torch.empty_like(z)
    dbr = [torch.empty_like(b) for b in branches]
    rc = L.lsrm_gate_merge_bwd(N, C, len(branches), int(per_head), int(head_dim), _dtype_code(z), _ptr(z),
                               _ptr_array(branches), _ptr(dout.contiguous()), _ptr(dz), _ptr_array(dbr), _stream())
    check(rc, "lsrm_gate_merge_bwd")
    return dz, dbr


def ulysses_pack(x: torch.Tensor, world: int) -> torch.Tensor:
    """[n, H, D] -> [W, n, hp, D]: the head slice of every rank, rank-major
    (hp = H/W, or one replicated head when H < W)."""
    L = _lib.lib()
    n, H, D = x.shape
    if x.stride(2) != 1 or x.stride(1) != D:
        x = x.contiguous()
    hp = H // world if H >= world else 1
    out = torch.empty(world, n, hp, D, dtype=x.dtype, device=x.device)
    rc = L.lsrm_ulysses_pack(n, H, D, world, _dtype_code(x), x.stride(0), _ptr(x), _ptr(out), _stream())
    check(rc, "lsrm_ulysses_pack")
    return out


def ulysses_unpack(y: torch.Tensor, num_heads: int) -> torch.Tensor:
    """[W, n, hp, D] -> [n, H, D]; replicas of one head are summed in rank
    order (fp32)."""
    L = _lib.lib()
    world, n, hp, D = y.shape
    y = y.contiguous()
    out = torch.empty(n, num_heads, D, dtype=y.dtype, device=y.device)
    rc = L.lsrm_ulysses_unpack(n, num_heads, D, world, _dtype_code(y), _ptr(y), out.stride(0), _ptr(out), _stream())
    check(rc, "lsrm_ulysses_unpack")
    return out


def head_layernorm_pack(x: torch.Tensor, world: int = 1, eps: float = 1e-5) -> torch.Tensor:
    """Per-head non-affine LayerNorm (fp32, cast back) of x [n, H, D] written
    straight into the Ulysses send layout [W, n, H/W, D] (W = 1: [1, n, H, D])."""
    L = _lib.lib()
    n, H, D = x.shape
    if x.stride(2) != 1 or x.stride(1) != D:
        x = x.contiguous()
    out = torch.empty(world, n, H // world, D, dtype=x.dtype, device=x.device)
    rc = L.lsrm_head_layernorm_pack(n, H, D, world, _dtype_code(x), x.stride(0), float(eps), _ptr(x), _ptr(out),
                                    _stream())
    check(rc, "lsrm_head_layernorm_pack")
    return out


def head_layernorm_pack_bwd(x: torch.Tensor, grad_packed: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Gradient of ``head_layernorm_pack`` with respect to x [n, H, D]."""
    L = _lib.lib()
    n, H, D = x.shape
    if x.stride(2) != 1 or x.stride(1) != D:
        x = x.contiguous()
    world = grad_packed.shape[0]
    g = grad_packed.contiguous()
    out = torch.empty(n, H, D, dtype=x.dtype, device=x.device)
    rc = L.lsrm_head_layernorm_pack_bwd(n, H, D, world, _dtype_code(x), x.stride(0), float(eps), _ptr(x), _ptr(g),
                                        _ptr(out), _stream())
    check(rc, "lsrm_head_layernorm_pack_bwd")
    return out


# ---------------------------------------------------------------------------
# Projection GEMM with the per-head LayerNorm in its epilogue
# ---------------------------------------------------------------------------


def _addr(t: Optional[torch.Tensor]):
    return t.data_ptr() if t is not None else None


def qkv_norm_fwd(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], segments, head_dim: int,
                 eps: float = 1e-5):
    """x [M, K] bf16 (row stride >= K), w [N, K] bf16 (stacked Linear
    weights), ``segments`` a list of (cols, raw, norm) in column order.
    Returns (outputs, rstd): per segment the bf16 result [M, cols] if ``raw``
    and its per-head LayerNorm [M, cols] if ``norm`` (None otherwise), and
    rstd [M, N / head_dim] fp32."""
    L = _lib.lib()
    assert x.dim() == 2 and x.stride(1) == 1 and x.dtype == torch.bfloat16, "x must be [M, K] bf16, unit column stride"
    w = w.contiguous()
    M, K = x.shape
    N = w.shape[0]
    dev = x.device
    segs = (_lib.QkvSegment * len(segments))()
    outs = []
    for i, (cols, raw, norm) in enumerate(segments):
        o = torch.empty(M, cols, dtype=x.dtype, device=dev) if raw else None
        on = torch.empty(M, cols, dtype=x.dtype, device=dev) if norm else None
        segs[i] = _lib.QkvSegment(int(cols), 0, _addr(o), _addr(on))
        outs.append((o, on))
    rstd = torch.empty(M, N // head_dim, dtype=torch.float32, device=dev)
    b = bias.contiguous() if bias is not None else None
    rc = L.lsrm_qkv_norm_fwd(M, K, N, int(head_dim), _ptr(x), x.stride(0), _ptr(w), _ptr(b), segs, len(segments),
                             float(eps), _ptr(rstd), _ptr(_err_word(dev)), _stream())
    check(rc, "lsrm_qkv_norm_fwd")
    return outs, rstd


def qkv_norm_bwd(M: int, N: int, head_dim: int, segments, rstd: torch.Tensor, device, dtype=torch.bfloat16):
    """``segments``: per segment (cols, out_norm, grad_out, grad_norm) with
    None for absent tensors.  Returns the gradient of the pre-norm result
    [M, N]."""
    L = _lib.lib()
    segs = (_lib.QkvGradSegment * len(segments))()
    keep = []
    for i, (cols, on, go, gn) in enumerate(segments):
        go = go.contiguous() if go is not None else None
        gn = gn.contiguous() if gn is not None else None
        keep += [go, gn]
        segs[i] = _lib.QkvGradSegment(int(cols), 0, _addr(on), _addr(go), _addr(gn))
    out = torch.empty(M, N, dtype=dtype, device=device)
    rc = L.lsrm_qkv_norm_bwd(M, N, int(head_dim), segs, len(segments), _ptr(rstd), _ptr(out), _stream())
    check(rc, "lsrm_qkv_norm_bwd")
    return out
