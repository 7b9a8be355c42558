"""The sequence-parallel decoder block on 2 GPUs (NCCL): tokens distributed by
``ulysses.seq_parallel_token_blocks`` (whole blocks), ``BlockMix`` with
``use_sequence_parallel=True`` (Ulysses exchanges around the attention
cores), against the same block run on one GPU over all tokens: every rank's
outputs, its tokens' input gradients and the rank-summed weight gradients
within 2e-2 (relative to the tensor's scale) and >= 0.9995 cosine.  Runs the
ranks as child processes: over NCCL on 2 GPUs (skipped with fewer), and over
gloo with both ranks on one GPU (the exchanges staged through host memory),
so a one-GPU machine checks the per-rank path as well."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import os, sys, datetime, copy, torch, torch.distributed as dist
sys.path[:0] = [ROOT, os.path.join(ROOT, "large-sparse-reconstruction-model_b200")]
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
BACKEND = "BK"  # nccl: one GPU per rank; gloo: every rank on GPU 0, exchanges through host memory
dev = torch.device("cuda", rank if BACKEND == "nccl" else 0)
torch.cuda.set_device(dev)
if BACKEND == "nccl":
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
else:
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
from tests.test_gpu_decoder import _scene
from lsrm_sparse import decoder, ulysses, ops
dim, Hq, Hkv = 128, 4, HKV
maps, cu_x, cu_y, nx, ny, M = _scene()
for m in maps.values():  # one copy of the head-independent selection per kv head
    m["block_topk"] = m["block_topk"][:1].expand(Hkv, -1, -1).contiguous()
torch.manual_seed(3)
ref_blk = decoder.BlockMix(dim, num_q_heads=Hq, num_kv_heads=Hkv).to(dev).bfloat16()
sp_blk = decoder.BlockMix(dim, num_q_heads=Hq, num_kv_heads=Hkv, use_sequence_parallel=True).to(dev).bfloat16()
sp_blk.load_state_dict(ref_blk.state_dict())
g = torch.Generator().manual_seed(4)
x = torch.randn(nx, dim, generator=g).bfloat16().to(dev)
y = torch.randn(ny, dim, generator=g).bfloat16().to(dev)
gx = (0.1 * torch.randn(nx, dim, generator=g)).bfloat16().to(dev)
gy = (0.1 * torch.randn(ny, dim, generator=g)).bfloat16().to(dev)
# one GPU, all tokens
xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
ox, oy, _ = ref_blk(xr, cu_x, yr, cu_y, maps, M)
((ox.float() * gx.float()).sum() + (oy.float() * gy.float()).sum()).backward()
# sequence parallel: this rank's whole blocks
(xl,), (yl,), cxl, cyl, smaps = ulysses.seq_parallel_token_blocks([x], [y], maps, "distribute")
xl, yl = xl.clone().requires_grad_(), yl.clone().requires_grad_()
sx, sy, _ = sp_blk(xl, cxl, yl, cyl, smaps, M)
(vs, ve), (is_, ie) = smaps["sp"].vol.local, smaps["sp"].img.local
((sx.float() * gx[vs:ve].float()).sum() + (sy.float() * gy[is_:ie].float()).sum()).backward()
torch.cuda.synchronize()
assert ops.read_errors() == 0
for p in sp_blk.parameters():
    if BACKEND == "nccl":
        dist.all_reduce(p.grad)
    else:
        c = p.grad.float().cpu()
        dist.all_reduce(c)
        p.grad.copy_(c)
ok = True
def close(name, a, b):
    global ok
    a, b = a.detach().float().flatten(), b.detach().float().flatten()
    err = (a - b).abs().max().item()
    bound = 2e-2 * max(1.0, b.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(a.double(), b.double(), dim=0).item() if b.abs().max() > 0 else 1.0
    if not (err <= bound and cos >= 0.9995):
        print("rank", rank, name, err, bound, cos, flush=True)
        ok = False
close("out x", sx, ox[vs:ve]); close("out y", sy, oy[is_:ie])
close("dx", xl.grad, xr.grad[vs:ve]); close("dy", yl.grad, yr.grad[is_:ie])
for (n, a), (_, b) in zip(sp_blk.named_parameters(), ref_blk.named_parameters()):
    close("d" + n, a.grad, b.grad)
# collect brings every rank's volume tokens back in order
(full,), _, _, _, _ = ulysses.seq_parallel_token_blocks([sx.detach()], [], smaps, "collect")
close("collect", full[vs:ve], sx)
ok = ok and full.shape[0] == nx
flag = torch.tensor([int(ok)], device=dev if BACKEND == "nccl" else "cpu")
dist.all_reduce(flag, op=dist.ReduceOp.MIN)
dist.destroy_process_group()
sys.exit(0 if flag.item() == 1 else 3)
'''


@pytest.mark.parametrize("backend", ["nccl", "gloo_one_gpu"])
@pytest.mark.parametrize("hkv", [4, 2])
def test_sequence_parallel_blockmix_matches_single_gpu(hkv, backend, tmp_path):
    """``nccl``: two GPUs; ``gloo_one_gpu``: both ranks on one GPU with the
    exchanges staged through host memory (the same per-rank code path, so a
    one-GPU machine checks it too)."""
    if backend == "nccl" and torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(CHILD.replace("ROOT", repr(ROOT)).replace("HKV", str(hkv))
                      .replace('"BK"', repr(backend.split("_")[0])))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
