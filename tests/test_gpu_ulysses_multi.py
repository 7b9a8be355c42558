"""Ulysses sequence parallelism on 2+ GPUs (NCCL): every rank's output equals
the single-GPU whole-sequence op bit for bit (heads are computed by the same
kernels), and its gradients agree within the bf16 tolerance (the compressed
branch's dK/dV split count depends on how many heads one launch holds).  Runs
the ranks as child processes: over NCCL on 2 GPUs (skipped with fewer), and
over gloo with both ranks on one GPU (the exchanges staged through host
memory), so a one-GPU machine checks the per-rank path as well."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import os, sys, datetime, torch, torch.distributed as dist
sys.path[:0] = [ROOT, os.path.join(ROOT, "large-sparse-reconstruction-model_b200")]
from lsrm_sparse import ulysses, synth, ops
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
BACKEND = "BK"  # nccl: one GPU per rank; gloo: every rank on GPU 0, exchanges through host memory
dev = torch.device("cuda", rank if BACKEND == "nccl" else 0)
torch.cuda.set_device(dev)
if BACKEND == "nccl":
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
else:
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
lens = synth.uniform_blocks(6000, 40, 64, 256, 5)
cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
N, H, Hkv, D = int(cu[-1]), 8, HKV, 64
g = torch.Generator().manual_seed(11)
q = torch.randn(N, H, D, generator=g).bfloat16()
k = torch.randn(N, Hkv, D, generator=g).bfloat16()
v = torch.randn(N, Hkv, D, generator=g).bfloat16()
z = torch.randn(N, 3 * H, generator=g).bfloat16()
dout = (0.1 * torch.randn(N, H, D, generator=g)).bfloat16()
cu_d = cu.to(dev)
# whole sequence on this GPU
ts = [t.to(dev).requires_grad_(True) for t in (q, k, v, z)]
ref = ulysses.whole_sequence_branches(*ts, cu_d, 8, 128)
ref.backward(dout.to(dev))
plan = ulysses.ShardPlan(cu.tolist(), world, rank)
s, e = plan.local
ls = [t[s:e].to(dev).requires_grad_(True) for t in (q, k, v, z)]
out = ulysses.three_branch_attention(*ls, plan, cu_d, 8, 128)
out.backward(dout[s:e].to(dev))
torch.cuda.synchronize()
assert ops.read_errors() == 0
ok = torch.equal(out, ref[s:e])
if not ok:
    print("rank", rank, "output differs:", (out.float() - ref[s:e].float()).abs().max().item(), flush=True)
for name, a, b in zip("qkvz", ls, ts):
    x, y = a.grad.float().flatten(), b.grad[s:e].float().flatten()
    err = (x - y).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(x, y, dim=0).item()
    if not (err <= 2e-2 and cos >= 0.9995):
        print("rank", rank, "d" + name, err, cos, flush=True)
        ok = False
flag = torch.tensor([int(ok)], device=dev if BACKEND == "nccl" else "cpu")
dist.all_reduce(flag, op=dist.ReduceOp.MIN)
dist.destroy_process_group()
sys.exit(0 if flag.item() == 1 else 3)
'''


@pytest.mark.parametrize("backend", ["nccl", "gloo_one_gpu"])
@pytest.mark.parametrize("hkv", [8, 2])
def test_ulysses_two_gpus_bit_identical_to_single_gpu(hkv, backend, tmp_path):
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
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
