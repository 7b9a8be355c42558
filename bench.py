"""Benchmark of the B200 variable-block native sparse attention (LSRM hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg2]

One step = forward + backward of the full three-branch sparse-attention op on
one synthetic voxel sequence (BASELINE config 2 by default): block-mean
compression of K/V, compressed attention, bit-exact per-query-block top-16
scoring (own block forced), selected-block attention, sliding window 512,
per-head sigmoid-gated merge, then the backward of everything.
With N > 1 processes the same sequence is split over the ranks by Ulysses
sequence parallelism (strong scaling: NCCL all-to-all exchanges of q/k/v and
the outputs).  Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "large-sparse-reconstruction-model_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "Sparse-attn TFLOP/s (fwd+bwd) & decoder tokens/s at 1/2/4/8 B200; % bf16 peak"

CONFIGS = {
    # the headline single-GPU workload
    "cfg2": dict(n=131072, heads=16, head_dim=64, res=256, blk_min=64, blk_max=256, topk=16, window=512,
                 gate="per_head", voxel=True),
    # configs[0] at its sizes (contiguous uniform blocks), on the GPU
    "cfg1": dict(n=4096, heads=8, head_dim=64, n_blocks=64, blk_min=32, blk_max=96, topk=8, window=128,
                 gate="per_head", voxel=False, qkv_scale=0.5),
    # half-size cfg2 (same grid, block sizes, top-k, window) for full ncu captures
    "cfg2s": dict(n=65536, heads=16, head_dim=64, res=256, blk_min=64, blk_max=256, topk=16, window=512,
                  gate="per_head", voxel=True),
    # 512^3 shell, blocks 32-512, window 1024, K/V compressed by the token-wise ResBlock
    # (2 x Linear(C -> C), C = H * head_dim) before the block mean
    "cfg3": dict(n=262144, heads=16, head_dim=64, res=512, blk_min=32, blk_max=512, topk=16, window=1024,
                 gate="per_head", voxel=True, compression="resblock"),
}


def _check_device_errors(ops):
    """Raise if a kernel set a bit in the library's device error word."""
    err = ops.read_errors()
    if err:
        raise RuntimeError(f"device error word 0x{err:x} (LSRM_ERR_* bits of include/lsrm_sparse.h)")


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------


def block_lengths(cfg, seed):
    from lsrm_sparse import synth

    if cfg["voxel"]:
        w = synth.voxel_workload(cfg["n"], cfg["res"], cfg["blk_min"], cfg["blk_max"], seed)
        return w.block_lens, w.shell_size
    return synth.uniform_blocks(cfg["n"], cfg["n_blocks"], cfg["blk_min"], cfg["blk_max"], seed), cfg["n"]


class Problem:
    def __init__(self, cfg, seed, device, pin=True):
        self.cfg = cfg
        lens, self.shell = block_lengths(cfg, seed)
        self.lens = lens
        N, H, D = cfg["n"], cfg["heads"], cfg["head_dim"]
        self.N, self.H, self.D, self.nb = N, H, D, len(lens)
        self.hidden = H * D
        g = torch.Generator(device="cpu").manual_seed(seed)
        pinned = (lambda t: t.pin_memory()) if pin else (lambda t: t)
        # host copies (pinned) for the end-to-end path
        sc = cfg.get("qkv_scale", 1.0)
        self.h_q = pinned((torch.randn(N, H, D, generator=g) * sc).bfloat16())
        self.h_k = pinned((torch.randn(N, H, D, generator=g) * sc).bfloat16())
        self.h_v = pinned((torch.randn(N, H, D, generator=g) * sc).bfloat16())
        self.h_x = pinned(torch.randn(N, self.hidden, generator=g).bfloat16())
        self.h_g = pinned((torch.randn(N, self.hidden, generator=g) * 0.1).bfloat16())
        n_gate = 3 * H if cfg["gate"] == "per_head" else 3 * self.hidden
        self.gate_w = (torch.randn(n_gate, self.hidden, generator=g) / math.sqrt(self.hidden)).bfloat16()
        # ResBlock compression weights (nn.Linear's default init range), bf16 like the step
        self.compression = cfg.get("compression", "mean")
        self.res_w = None
        if self.compression == "resblock":
            C, bound = self.hidden, 1.0 / math.sqrt(self.hidden)
            u = lambda *shape: ((torch.rand(*shape, generator=g) * 2 - 1) * bound).bfloat16()  # noqa: E731
            self.res_w = {s: (u(C, C), u(C), u(C, C), u(C)) for s in ("k", "v")}
        cu_blk = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
        self.h_cu_blk = pinned(cu_blk)
        self.h_cu_seq = pinned(torch.tensor([0, N], dtype=torch.int32))
        self.h_cu_sb = pinned(torch.tensor([0, len(lens)], dtype=torch.int32))
        self.device = device
        if device != "cpu":
            self.to_device()

    def host_inputs(self):
        return [self.h_q, self.h_k, self.h_v, self.h_x, self.h_g, self.h_cu_blk, self.h_cu_seq, self.h_cu_sb]

    def adopt(self, ts):
        q, k, v, x, self.g, self.cu_blk, self.cu_seq, self.cu_sb = ts
        self.q, self.k, self.v, self.x = (t.requires_grad_() for t in (q, k, v, x))
        if not hasattr(self, "wg"):
            self.wg = self.gate_w.to(self.device).requires_grad_()
            self.compress = make_compress(self.res_w, self.device)

    def params(self):
        ps = [self.wg]
        if self.compress is not None:
            ps += list(self.compress.params)
        return ps

    def to_device(self, non_blocking=False):
        self.adopt([t.to(self.device, non_blocking=non_blocking) for t in self.host_inputs()])

    def h2d_bytes(self):
        return int(sum(t.numel() * t.element_size() for t in self.host_inputs()))


def make_compress(res_w, device):
    """The ResBlock compression of SpatialSparseAttentionIn (a SparseResBlock
    per K and V, then the block mean; spatial_sparse_attention.py:46-66) with
    the given weights, or None for the plain block mean."""
    if res_w is None:
        return None
    from lsrm_sparse.module import SparseResBlock

    mods = {}
    for s in ("k", "v"):
        m = SparseResBlock(res_w[s][0].shape[0]).to(device).bfloat16()
        with torch.no_grad():
            m.act_layers[0].weight.copy_(res_w[s][0])
            m.act_layers[0].bias.copy_(res_w[s][1])
            m.act_layers[2].weight.copy_(res_w[s][2])
            m.act_layers[2].bias.copy_(res_w[s][3])
        mods[s] = m

    def compress(k2, v2, cu_blk):
        return mods["k"].forward_block_mean(k2, cu_blk), mods["v"].forward_block_mean(v2, cu_blk)

    compress.params = [t for m in mods.values() for t in m.parameters()]
    compress.modules = mods
    return compress


def forward_backward(p: Problem, want_loss=False, capture=None):
    """One step through the public API: lsrm_sparse.functional.three_branch_attention
    (the same function every rank runs under sequence parallelism), the gate
    Linear, and the backward of all of it."""
    from lsrm_sparse import functional as F

    cfg = p.cfg

    def gate_logits():
        ready = getattr(p, "ready", None)  # e2e run: the copy of x may still be in flight
        if ready:
            torch.cuda.current_stream().wait_event(ready["x"])
        return torch.nn.functional.linear(p.x, p.wg)

    out = F.three_branch_attention(p.q, p.k, p.v, p.cu_blk, cfg["topk"], cfg["window"], gate_logits,
                                   compress=p.compress, per_head=cfg["gate"] == "per_head", capture=capture)
    ready = getattr(p, "ready", None)
    if ready:
        torch.cuda.current_stream().wait_event(ready["g"])
    loss = (out.float() * p.g.float()).sum() if want_loss else None
    out.backward(p.g)
    return loss


class ShardedProblem:
    """One rank's view of the whole cfg problem under Ulysses sequence
    parallelism: its token shard on the device (whole blocks, token-balanced),
    the whole block table, the gate weight."""

    def __init__(self, full: Problem, plan, device):
        self.full, self.plan, self.device = full, plan, device
        self.cfg, self.lens, self.shell = full.cfg, full.lens, full.shell
        self.N, self.H, self.D, self.nb = full.N, full.H, full.D, full.nb
        s, e = plan.local
        self.h_local = [t[s:e] for t in (full.h_q, full.h_k, full.h_v, full.h_x, full.h_g)]
        self.h_cu_blk = full.h_cu_blk
        self.to_device()
        self.wg = full.gate_w.to(device).requires_grad_()

    def host_inputs(self):
        return self.h_local + [self.h_cu_blk]

    def adopt(self, ts):
        q, k, v, x, self.g, self.cu_blk = ts
        self.q, self.k, self.v, self.x = (t.requires_grad_() for t in (q, k, v, x))

    def to_device(self, non_blocking=False):
        self.adopt([t.to(self.device, non_blocking=non_blocking) for t in self.host_inputs()])

    def h2d_bytes(self):
        return int(sum(t.numel() * t.element_size() for t in self.host_inputs()))


def forward_backward_sp(p: ShardedProblem, want_loss=False, capture=None):
    """One sequence-parallel step: gate logits on the local tokens, Ulysses
    exchange, whole-sequence three-branch op for this rank's heads, exchange
    back, backward through the same path."""
    from lsrm_sparse import ulysses

    cfg = p.cfg
    n = p.q.shape[0]
    z = torch.nn.functional.linear(p.x, p.wg)
    fn = None
    if capture is not None:
        def fn(*a):
            return ulysses.whole_sequence_branches(*a, capture=capture)
    out = ulysses.three_branch_attention(p.q, p.k, p.v, z, p.plan, p.cu_blk, cfg["topk"], cfg["window"],
                                         branch_fn=fn)
    out = out.view(n, -1)
    loss = (out.float() * p.g.float()).sum() if want_loss else None
    out.backward(p.g)
    return loss


def zero_grads(p: Problem):
    for t in [p.q, p.k, p.v, p.x] + (p.params() if hasattr(p, "params") else [p.wg]):
        t.grad = None


def capture_step(step, p, lib_launches):
    """One whole step — forward, backward, every gradient — captured as a CUDA
    graph, so replaying it costs one launch on the host instead of issuing
    each kernel (and, under sequence parallelism, each NCCL exchange) from
    Python.  The gradients are None when the capture starts, so the captured
    backward writes them into buffers of the graph's pool and every replay
    recomputes them there.  Returns (graph, launches of this library's kernels
    per replay)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # the allocator and the libraries settle on the capture stream first
        for _ in range(2):
            step(p)
            zero_grads(p)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = lib_launches()
    # thread_local: NCCL's watchdog thread keeps polling its events during the capture
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step(p)
    return graph, lib_launches() - n0


def grads_of(p):
    return [t.grad for t in [p.q, p.k, p.v, p.x] + (p.params() if hasattr(p, "params") else [p.wg])]


def _eager_grads(step, p):
    zero_grads(p)
    step(p)
    torch.cuda.synchronize()
    return grads_of(p)


def count_pairs(p: Problem, bt: torch.Tensor):
    """Attended (query, key) pairs per head of the three branches."""
    lens = torch.tensor(p.lens, dtype=torch.int64)
    sel = bt.cpu().long()  # [H, nqb, k]
    valid = sel >= 0
    sel_len = torch.where(valid, lens[sel.clamp(min=0)], torch.zeros_like(sel)).sum(-1)  # [H, nqb]
    sel_pairs = (sel_len * lens[None]).sum().item()  # summed over heads
    comp_pairs = p.N * p.nb * p.H
    half = p.cfg["window"] // 2
    i = torch.arange(p.N, dtype=torch.int64)
    band = (torch.clamp(i + half, max=p.N - 1) - torch.clamp(i - half, min=0) + 1).sum().item()
    slide_pairs = band * p.H
    return dict(select=sel_pairs, compressed=comp_pairs, sliding=slide_pairs)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi clock / throttle samples every 200 ms.  Entering starts the
    sampler and returns once its first sample arrived (up to 5 s), so the
    timed region that follows is covered; only samples taken between enter
    and exit count."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self._all.append((time.perf_counter(), line))

    def __enter__(self):
        import threading

        self._all = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        t0 = time.perf_counter()
        while not self._all and time.perf_counter() - t0 < 5.0:
            time.sleep(0.02)
        self.t_enter = time.perf_counter()
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is None:
            return
        t_exit = time.perf_counter()
        time.sleep(0.25)  # one more sample of the tail of the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self._thread.join(timeout=5)
        inside = [l for t, l in self._all if self.t_enter - 0.2 <= t <= t_exit + 0.25]
        self.lines = inside or [l for _, l in self._all[-1:]]

    def summary(self):
        rows = []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(dict(sm=float(f[1]), sm_max=float(f[2]), power=float(f[3]), active=f[4], hw=f[5],
                                 hw_th=f[6], sw_th=f[7], sw_pc=f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        pmax = max(r["power"] for r in rows)
        load = [r for r in rows if r["power"] > 0.5 * pmax] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hw_th", "hw_thermal_slowdown"),
                              ("sw_th", "sw_thermal_slowdown"), ("sw_pc", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["sm_max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(load), "power_w_max": pmax}


# ---------------------------------------------------------------------------
# CPU baseline (oracle restatement on the host cores)
# ---------------------------------------------------------------------------


def cpu_sample(p: Problem, n_qblocks: int, seed: int):
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    qbs = sorted(rng.choice(p.nb, size=min(n_qblocks, p.nb), replace=False).tolist())
    t0 = time.perf_counter()
    _, flops = oracle.three_branch_sample_step(p.h_q, p.h_k, p.h_v, p.h_x, p.gate_w, p.h_g, p.h_cu_blk, qbs,
                                               p.cfg["topk"], p.cfg["window"], per_head=p.cfg["gate"] == "per_head")
    tokens = int(sum(p.lens[i] for i in qbs))
    what = "three-branch fwd+bwd incl. exact scoring"
    if getattr(p, "res_w", None) is not None:
        # the ResBlock compression (token-wise) on as many tokens as the sample has queries, fwd + bwd
        cb = p.h_cu_blk.long()
        rows = torch.cat([torch.arange(int(cb[i]), int(cb[i + 1])) for i in qbs])
        for s in ("k", "v"):
            x = getattr(p, "h_" + s)[rows].reshape(rows.numel(), -1)
            oracle.compress_vjp(x, torch.ones(x.shape), p.res_w[s])
        flops += 24.0 * rows.numel() * p.hidden ** 2
        what += " and the ResBlock K/V compression of as many tokens"
    dt = time.perf_counter() - t0
    return dict(value=flops / dt / 1e12, unit="TFLOP/s", cores=torch.get_num_threads(), kind="port",
                sample=f"{len(qbs)} of {p.nb} query blocks ({tokens} of {p.N} queries), {what}, fp32 torch on "
                       f"{torch.get_num_threads()} host threads",
                seconds=dt)


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, cfg):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    p = Problem(cfg, args.seed, "cpu", pin=False)  # host tensors only
    # a third of the baseline's sample per step and two query blocks per warm-up, so that the default
    # 3 + 10 steps end within a few minutes on the host
    per_step = max(4, args.cpu_qblocks // 3)
    for _ in range(args.warmup):
        cpu_sample(p, 2, args.seed)
    vals, secs = [], []
    for i in range(args.steps):
        r = cpu_sample(p, per_step, args.seed + 1 + i)
        vals.append(r["value"])
        secs.append(r["seconds"])
    v = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(secs),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-sphere SDF shell voxels, Morton octree blocks)",
        "config": workload_config(cfg, p, ws),
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": r["cores"], "kind": "port", "sample": r["sample"]},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line, default=_json_default), flush=True)


def workload_config(cfg, p, world=1):
    return {"parallelism": f"ulysses sequence parallel over {world} GPUs (strong scaling)" if world > 1
            else "single GPU","workload": f"three-branch sparse attention fwd+bwd, N={cfg['n']} voxel tokens, H={cfg['heads']}, "
                        f"d={cfg['head_dim']}, top-{cfg['topk']} per query block, window {cfg['window']}",
            "tokens": cfg["n"], "heads": cfg["heads"], "head_dim": cfg["head_dim"], "blocks": p.nb,
            "block_len": [min(p.lens), max(p.lens)], "topk": cfg["topk"], "window": cfg["window"],
            "gate": cfg["gate"], "selection": "per query block, bit-exact fp32 score, own block forced",
            "l2": f"inputs larger than L2 (q/k/v {cfg['n'] * cfg['heads'] * cfg['head_dim'] * 2 / 1e6:.0f} MB each), no flush",
            "grid_res": cfg.get("res")}


def kernel_flops(name, pairs, H, D, N, nb):
    """Algorithmic FLOPs of one launch of a profiled kernel (pairs summed
    over heads): forward 4d, dQ pass 6d (QK^T, dO V^T, dS K), dK/dV pass 8d
    (K Q^T, V dO^T, P^T dO, dS^T Q) per attended pair."""
    table = {"select": pairs["select"], "range": pairs["compressed"], "sliding": pairs["sliding"]}
    for kind, mult in (("attn_fwd_", 4), ("attn_dq_", 6), ("attn_dkdv_", 8)):
        if name.startswith(kind):
            return mult * D * table[name[len(kind):]], "tensor"
    return None, None


def run_ours(args, cfg):
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime

        # NCCL's version banner goes to stdout, where the one JSON result line belongs
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    from lsrm_sparse import _lib, ops, ulysses

    lib_launches = _lib.launch_count
    if ws > 1:
        # Ulysses sequence parallelism: every rank builds the same whole
        # problem on the host and keeps its token shard on the device
        from lsrm_sparse import ulysses

        if cfg.get("compression", "mean") != "mean":
            raise SystemExit("the sequence-parallel bench runs the block-mean compression only")

        full = Problem(cfg, args.seed, "cpu", pin=True)
        plan = ulysses.ShardPlan(full.h_cu_blk.tolist(), ws, rank)
        p = ShardedProblem(full, plan, dev)
        step = forward_backward_sp
    else:
        p = Problem(cfg, args.seed, dev)
        step = forward_backward
    cap = {}
    step(p, capture=cap)
    zero_grads(p)
    err = ops.read_errors()
    if err:
        raise RuntimeError(f"device error bits 0x{err:x} in the first step")
    pairs = count_pairs(p, cap["block_topk"])
    # this rank's own work (all heads on one GPU; H / N heads of the whole sequence under Ulysses)
    rank_pairs = dict(pairs)
    if ws > 1:
        rank_pairs["compressed"] = pairs["compressed"] // ws
        rank_pairs["sliding"] = pairs["sliding"] // ws
        # each rank selected for its own heads: the whole job's pairs are the sum
        t = torch.tensor([float(pairs["select"])], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t)
        pairs["select"] = int(t.item())
    flops_attn = 14.0 * p.D * (pairs["select"] + pairs["compressed"] + pairs["sliding"])
    # ResBlock compression (cfg3): two C x C Linears per K and V, forward 2 FLOPs per MAC, backward twice that
    flops_comp = 24.0 * p.N * p.hidden ** 2 if getattr(p, "res_w", None) is not None else 0.0
    flops_step = flops_attn + flops_comp
    for _ in range(max(args.warmup - 1, 0)):
        step(p)
        zero_grads(p)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    # ---- the step as a CUDA graph (checked against the eager step's gradients) ----
    graph, graph_launches, graph_note = None, 0, "eager (--eager)"
    if not args.eager:
        ok = 1
        try:
            ref = [None if g is None else g.clone() for g in _eager_grads(step, p)]
            graph, graph_launches = capture_step(step, p, lib_launches)
            graph.replay()
            torch.cuda.synchronize()
            same = all((a is None and b is None) or (a is not None and b is not None and torch.equal(a, b))
                       for a, b in zip(ref, grads_of(p)))
            if not same:
                raise RuntimeError("graph replay gradients differ from the eager step's")
            del ref
            graph_note = "CUDA graph of the whole step (forward + backward), replayed once per step; its " \
                         "gradients equal the eager step's bit for bit"
        except Exception as e:  # a call on the path refused the capture: time the eager step
            print(f"CUDA graph capture not used ({e}); timing the eager step", file=sys.stderr, flush=True)
            graph, ok, graph_note = None, 0, f"eager (graph capture failed: {str(e)[:120]})"
        if ws > 1:  # every rank replays or none does
            t = torch.tensor([ok], dtype=torch.int32, device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            if int(t.item()) == 0 and graph is not None:
                graph, graph_note = None, "eager (graph capture failed on another rank)"
        if graph is None:
            zero_grads(p)
        for _ in range(2 if graph is not None else 0):  # warm replays
            graph.replay()

    # ---- timed pass (device time, CUDA events on the compute stream) ----
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = lib_launches()
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(p)
                zero_grads(p)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = lib_launches() - n0 + graph_launches * (args.steps if graph is not None else 0)
    _check_device_errors(ops)
    barrier()
    if graph is not None:
        zero_grads(p)  # the eager passes below allocate their own gradients
    if rank == 0:
        print(f"device memory: {torch.cuda.max_memory_allocated(dev) / 2**30:.2f} GiB allocated at peak",
              file=sys.stderr, flush=True)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = ms
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_max = float(t.item())
    value = flops_step / (ms_max * 1e-3) / 1e12  # whole job: one problem (N=1) or one sharded problem (N>1)

    # ---- profiled pass: per-kernel device time (events on the launching stream) ----
    _lib.profile_enable(True)
    xtimer = ulysses.time_exchanges(True) if ws > 1 else None
    for _ in range(args.steps):
        step(p)
        zero_grads(p)
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    _lib.profile_enable(False)
    exchange = None
    if xtimer is not None:
        xs = xtimer.stats()
        ulysses.time_exchanges(False)
        # the busiest rank's exchange time; bytes are this rank's per direction
        t = torch.tensor([xs["ms"]], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        a2a_ms = float(t.item()) / args.steps
        out_b = xs["bytes_out"] / args.steps
        exchange = {"a2a_ms_per_step": a2a_ms, "calls_per_step": xs["calls"] / args.steps,
                    "bytes_out_per_step": out_b, "bytes_in_per_step": xs["bytes_in"] / args.steps,
                    "a2a_gbs": out_b / (a2a_ms * 1e-3) / 1e9 if a2a_ms > 0 else None,
                    "link_gbs": 900.0, "link_note": "NVLink 5 nominal per direction per GPU (measured peer copy "
                                                    "on this pool: 770)",
                    "share_of_step": a2a_ms / ms_max,
                    "how": "CUDA events on the compute stream around every all_to_all_single of the step (forward "
                           "and backward: q, k, v, gate logits, output); bytes = what leaves this rank"}
    peaks, peak_kind = load_peaks()
    total_prof = sum(v[0] for v in prof.values())
    kernels = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] / args.steps,
                   "share": v[0] / total_prof if total_prof else None} for k, v in sorted(prof.items())}
    attn = {k: v for k, v in prof.items() if kernel_flops(k, rank_pairs, p.H, p.D, p.N, p.nb)[0] is not None}
    dom = max(attn.items(), key=lambda kv: kv[1][0])[0] if attn else None
    roofline = None
    if dom is not None:
        # one GPU's kernel: this rank's own pairs over this rank's launch time, against one GPU's peak
        fl, bound = kernel_flops(dom, rank_pairs, p.H, p.D, p.N, p.nb)
        avg_ms = prof[dom][0] / prof[dom][1]
        achieved = fl / (avg_ms * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        roofline = {"kernel": dom, "bound": bound, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic_for(dom, cfg.get("name") if ws == 1 else None),
                    "peak_source": f"bf16_tflops_sustained of {peak_kind} (kernel timed inside a long step)",
                    "scope": "one GPU (rank 0): its own pairs and launch time" if ws > 1 else "one GPU"}
    slowest = max(prof.items(), key=lambda kv: kv[1][0])[0] if prof else None

    # ---- end to end through the public API: H2D inputs, D2H loss ----
    e2e = None
    if not args.no_e2e:
        e_steps = max(3, min(args.steps, 20))
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        copy_stream = torch.cuda.Stream(device=dev)

        partial = isinstance(p, Problem)  # single GPU: x and g are awaited where the step first uses them
        names = {2: "qkv", 3: "x", 4: "g"}

        def fetch():
            # this step's inputs, pinned host -> device on the copy stream: block
            # tables, q, k, v first (the first kernels use them), then x and g
            hs = p.host_inputs()
            order = list(range(5, len(hs))) + [0, 1, 2, 3, 4] if partial else list(range(len(hs)))
            ts = [None] * len(hs)
            evs = {}
            with torch.cuda.stream(copy_stream):
                for j in order:
                    ts[j] = hs[j].to(dev, non_blocking=True)
                    if partial and j in names:
                        evs[names[j]] = torch.cuda.Event()
                        evs[names[j]].record(copy_stream)
                evs["all"] = torch.cuda.Event()
                evs["all"].record(copy_stream)
            return ts, evs

        def take(nx):
            ts, evs = nx
            if partial:
                stream.wait_event(evs["qkv"])
                p.ready = {"x": evs["x"], "g": evs["g"]}
            else:
                stream.wait_event(evs["all"])
            for t in ts:
                t.record_stream(stream)
            p.adopt(ts)

        # untimed round trips first: the allocator then holds the buffers of
        # two steps' inputs (the prefetch keeps two alive) next to the CUDA
        # graph's private pool; the first eager steps after the capture run
        # 3-5x slower while it grows (measured on one B200: 128, 87, 87, 118,
        # 75 ms, then 26 ms per step)
        for _ in range(max(6, args.warmup)):
            take(fetch())
            nxt_w = fetch()
            loss = step(p, want_loss=True)
            float(loss.item())
            zero_grads(p)
            del nxt_w
        torch.cuda.synchronize()
        step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(e_steps + 1)]
        # each step's loss goes device -> pinned host on the compute stream; the
        # host reads it one step later, so it never stalls the GPU between steps
        loss_host = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
        loss_ev = [torch.cuda.Event() for _ in range(2)]
        losses = []
        e0.record(stream)
        nxt = fetch()
        for i in range(e_steps):
            take(nxt)
            if i + 1 < e_steps:
                nxt = fetch()  # the next step's copy overlaps this step's compute
            loss = step(p, want_loss=True)
            loss_host[i & 1].copy_(loss.detach().float(), non_blocking=True)  # device -> host: the step's result
            loss_ev[i & 1].record(stream)
            zero_grads(p)
            step_ev[i + 1].record(stream)
            if i >= 1:
                loss_ev[(i - 1) & 1].synchronize()
                losses.append(float(loss_host[(i - 1) & 1]))
        e1.record(stream)
        loss_ev[(e_steps - 1) & 1].synchronize()
        losses.append(float(loss_host[(e_steps - 1) & 1]))
        torch.cuda.synchronize()
        p.ready = None
        assert len(losses) == e_steps and all(math.isfinite(x) for x in losses), "non-finite loss in the e2e run"
        e_ms = e0.elapsed_time(e1) / e_steps
        per_step = [e0.elapsed_time(step_ev[1])] + [step_ev[i].elapsed_time(step_ev[i + 1])
                                                   for i in range(1, e_steps)]
        if rank == 0:
            print("e2e per-step ms: " + " ".join(f"{x:.1f}" for x in per_step), file=sys.stderr, flush=True)
        if ws > 1:
            t = torch.tensor([e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": flops_step / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": p.h2d_bytes(), "d2h_bytes_per_step": 4,
               "note": "every step copies its inputs from pinned host memory (copy stream, overlapped with the "
                       "previous step's compute) and copies its loss back to pinned host memory (read by the "
                       "host one step later)"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_sample(p, args.cpu_qblocks, args.seed)
        cpu.pop("seconds", None)

    # a graph holding NCCL calls is released before the process group goes
    graph = None
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic: seeded random-sphere SDF shell ({p.shell} shell voxels, subsampled), Morton octree "
                "blocks; q/k/v N(0,1), grad N(0,0.1)",
        "config": workload_config(cfg, p, ws),
        "tokens_per_s": p.N / (ms_max * 1e-3),
        "flops_per_step": flops_step,
        "attention_tflops": flops_attn / (ms_max * 1e-3) / 1e12,
        "compression_flops_per_step": flops_comp,
        "pairs_per_step": pairs,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": int(launches),
        "timed_step": graph_note,
        "clocks": clk.summary(),
        "exchange": exchange,
        "kernels": kernels,
        "slowest_kernel": slowest,
    }
    print(json.dumps(line, default=_json_default), flush=True)


def _json_default(o):
    if hasattr(o, "item"):
        return o.item()
    return str(o)


def traffic_for(kernel, workload):
    """DRAM bytes per launch of `kernel` from the committed ncu summary of
    this very workload on one GPU, if one exists (profiles/traffic.json:
    {config name: {kernel: bytes_per_launch}}); None for any other workload
    (another config, overridden sizes, or one rank's share under N > 1)."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if workload and os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(workload, {}).get(kernel)
    return None


# ---------------------------------------------------------------------------
# --path volume_output: VolTransformer.prepare_volume_output (the decoder's
# output formatting, models_sparse/voldecoder.py:196-268)
# ---------------------------------------------------------------------------

VOLUME_CFG = dict(n=131072, res=256, upsample=2, channels=32)  # cfg2's voxel shell; the VolUpsampler default of 32


def volume_problem(seed):
    from lsrm_sparse import synth

    c = VOLUME_CFG
    vox, shell = synth.sdf_shell_voxels(c["res"], c["n"], seed)  # [n, 3] x, y, z, Morton order
    n = vox.shape[0]
    vidx = torch.zeros(n, 4, dtype=torch.int32)
    vidx[:, 1], vidx[:, 2], vidx[:, 3] = (torch.from_numpy(vox[:, j].copy()) for j in (2, 1, 0))
    g = torch.Generator().manual_seed(seed)
    vol = torch.randn(n, c["channels"] * c["upsample"] ** 3, generator=g).bfloat16()
    return vol, vidx, shell


def volume_bytes(n):
    """Algorithmic HBM bytes of one call: the -1 fill of the index volume,
    the feature transpose (read + write), the index reads (boundary and
    scatter passes) and one 4-byte index write per sub-voxel."""
    c = VOLUME_CFG
    S, R = c["upsample"] ** 3, c["res"] * c["upsample"]
    return R ** 3 * 4 + 2 * n * c["channels"] * S * 2 + 2 * n * 16 + n * S * 4


def volume_cpu_sample(vol, vidx, n_tok):
    import oracle

    c = VOLUME_CFG
    t0 = time.perf_counter()
    oracle.prepare_volume_output(vol[:n_tok].float().numpy(), vidx[:n_tok].numpy(), c["channels"], c["upsample"],
                                 c["res"], batch_size=1)
    dt = time.perf_counter() - t0
    return dict(value=volume_bytes(n_tok) / dt / 1e9, unit="GB/s", cores=1, kind="port",
                sample=f"{n_tok} of {vidx.shape[0]} tokens (full {c['res'] * c['upsample']}^3 index volume), numpy "
                       f"oracle on one host thread", seconds=dt)


def run_volume_output(args):
    ws, rank, local = dist_env()
    if rank != 0:  # single-GPU path: the other ranks have nothing to do
        return
    c = VOLUME_CFG
    vol_h, vidx_h, shell = volume_problem(args.seed)
    n = vidx_h.shape[0]
    base = {"metric": "prepare_volume_output HBM throughput (algorithmic bytes / time)", "unit": "GB/s",
            "higher_is_better": True,
            "config": {"workload": f"prepare_volume_output, {n} voxel tokens of a {c['res']}^3 SDF shell, upsample "
                                   f"x{c['upsample']}, {c['channels']} channels bf16, batch 1",
                       "l2": "the 537 MB index volume written every call is larger than L2"}}
    if args.impl == "reference":
        sample = 2048
        for _ in range(min(args.warmup, 1)):
            volume_cpu_sample(vol_h, vidx_h, sample)
        vals = [volume_cpu_sample(vol_h, vidx_h, sample) for _ in range(args.steps)]
        v = statistics.median(r["value"] for r in vals)
        cb = dict(vals[0])
        cb["value"] = v
        cb.pop("seconds", None)
        line = dict(base, impl="reference", value=v, n_gpus=ws, steps=args.steps, warmup=args.warmup,
                    ms_per_step=statistics.median(r["seconds"] for r in vals) * 1e3, scaling="weak",
                    vs_baseline=None, dtype="u8", data="synthetic", cpu_baseline=cb,
                    e2e={"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return
    from lsrm_sparse import _lib
    from lsrm_sparse import ops
    from lsrm_sparse import volume as V

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    vol_h, vidx_h = vol_h.pin_memory(), vidx_h.pin_memory()
    vol, vidx = vol_h.to(dev), vidx_h.to(dev)
    prior = torch.zeros(1, device=dev)
    call = lambda v, i: V.prepare_volume_output(v, i, prior, c["channels"], c["upsample"], c["res"], batch_size=1)
    for _ in range(args.warmup):
        call(vol, vidx)
    _check_device_errors(ops)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            call(vol, vidx)
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = volume_bytes(n)
    value = nbytes / (ms * 1e-3) / 1e9
    peaks, kind = load_peaks()
    # end to end: the call's inputs from pinned host memory, its boundaries back
    cu_h = torch.empty(2, dtype=torch.int32).pin_memory()
    vol_d, vidx_d = torch.empty_like(vol), torch.empty_like(vidx)
    out = call(vol, vidx)  # the loop keeps one call's outputs alive during the next: let the allocator hold two sets
    out = call(vol, vidx)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        vol_d.copy_(vol_h, non_blocking=True)
        vidx_d.copy_(vidx_h, non_blocking=True)
        out = call(vol_d, vidx_d)
        cu_h.copy_(out["cu_seqlens"], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    assert ops.read_errors() == 0 and int(cu_h[1]) == n * c["upsample"] ** 3
    e_ms = e0.elapsed_time(e1) / args.steps
    cpu = None
    if not args.no_cpu:
        cpu = volume_cpu_sample(vol_h, vidx_h, 2048)
        cpu.pop("seconds", None)
    line = dict(base, value=value, n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms, scaling="weak",
                vs_baseline=None, dtype="u8",
                data=f"synthetic: seeded random-sphere SDF shell ({shell} shell voxels, subsampled), features N(0,1)",
                roofline={"kernel": "volume_output", "bound": "hbm", "achieved": value, "peak": peaks["hbm_gbs"],
                          "unit": "GB/s", "frac": value / peaks["hbm_gbs"], "traffic": None,
                          "peak_source": f"hbm_gbs of {kind}"},
                cpu_baseline=cpu,
                e2e={"value": nbytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e_ms,
                     "h2d_bytes_per_step": int(vol_h.numel() * 2 + vidx_h.numel() * 4), "d2h_bytes_per_step": 8},
                gpu_launches=int(launches), clocks=clk.summary())
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# --path volume_geo_topk: the geometric volume-to-volume block selection of
# build_volume_to_volume_attn (misc/sparse_utils.py:1203-1279)
# ---------------------------------------------------------------------------

GEO_CFG = dict(res=64, block_size=8, topk=8, bbox_radius=0.5, batch=2)  # the reference's defaults


def geo_problem(seed):
    from lsrm_sparse import synth

    c = GEO_CFG
    parts = []
    for b in range(c["batch"]):
        vox, _ = synth.sdf_shell_voxels(c["res"], 1 << 30, seed + b)  # every shell voxel
        t = torch.zeros(vox.shape[0], 4, dtype=torch.int32)
        t[:, 0] = b
        t[:, 1], t[:, 2], t[:, 3] = (torch.from_numpy(vox[:, j].copy()) for j in (2, 1, 0))
        parts.append(t)
    return torch.cat(parts)


def run_volume_geo(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    import types

    c = GEO_CFG
    coords_h = geo_problem(args.seed)
    n = coords_h.shape[0]
    base = {"metric": "geometric volume-to-volume block selection (tokens/s)", "unit": "tokens/s",
            "higher_is_better": True,
            "config": {"workload": f"build_volume_to_volume_attn top-{c['topk']}: {n} voxel tokens of {c['batch']} SDF "
                                   f"shells, {c['res']}^3 volume, {c['block_size']}^3 blocks",
                       "l2": "inputs fit in L2; the selection is bound by distance evaluations, not memory"}}
    from lsrm_sparse import blocks

    if args.impl == "reference":
        import oracle

        cs, cb, srt = blocks_cpu_separation(coords_h)
        sample = 2000
        rows = np.linspace(0, n - 1, sample).astype(np.int64)
        secs = []
        for _ in range(max(1, args.steps)):
            t0 = time.perf_counter()
            oracle.volume_block_topk(srt, cs, cb, c["batch"], c["res"], c["bbox_radius"], c["topk"], rows=rows)
            secs.append(time.perf_counter() - t0)
        v = sample / statistics.median(secs)
        cb_line = dict(value=v, unit="tokens/s", cores=1, kind="port",
                       sample=f"{sample} of {n} tokens (evenly spaced), numpy oracle on one host thread (block centres "
                              f"of the whole set included)")
        print(json.dumps(dict(base, impl="reference", value=v, n_gpus=ws, steps=args.steps, warmup=args.warmup,
                              ms_per_step=statistics.median(secs) * 1e3, scaling="weak", vs_baseline=None,
                              dtype="f32", data="synthetic", cpu_baseline=cb_line,
                              e2e={"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                   "d2h_bytes_per_step": 0})), flush=True)
        return
    from lsrm_sparse import _lib, ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    coords = coords_h.to(dev)
    keys = blocks.volume_sort_keys(coords, c["res"], c["block_size"])
    coords = coords[torch.argsort(keys, stable=True)].contiguous()
    bs = c["block_size"]
    cu_sb, cu_blk, _ = blocks.block_separation(coords, 3, [bs] * 3, c["batch"], [c["res"]] * 3)
    nb = int(cu_sb[-1])
    call = lambda: blocks.volume_block_topk(coords, cu_sb, cu_blk, c["batch"], c["res"], c["bbox_radius"], c["topk"])
    for _ in range(args.warmup):
        call()
    _check_device_errors(ops)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    value = n / (ms * 1e-3)
    # distance evaluations: each token against every block of its batch element
    blocks_per_elem = (cu_sb[1:] - cu_sb[:-1]).cpu().tolist()
    counts = torch.bincount(coords_h[:, 0].long(), minlength=c["batch"]).tolist()
    evals = sum(a * b for a, b in zip(counts, blocks_per_elem))
    hbm_bytes = n * 16 * 2 + n * c["topk"] * 4 + nb * 12  # coordinates (two passes), selections, centres
    peaks, kind = load_peaks()
    # end to end through the public call: block-sorted coordinates from pinned host
    # memory, separation + selection, the first selection row read back
    args_ns = types.SimpleNamespace(block_size=bs, volume_res=c["res"], use_3d_aware_attn=True,
                                    topk_volume=c["topk"], bbox_radius=c["bbox_radius"])
    sorted_h = coords.cpu().pin_memory()
    row_h = torch.empty(c["topk"], dtype=torch.int32).pin_memory()
    blocks.build_volume_to_volume_attn(sorted_h.to(dev), args_ns)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        res = blocks.build_volume_to_volume_attn(sorted_h.to(dev, non_blocking=True), args_ns)
        row_h.copy_(res["block_topk"][0, 0], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1) / args.steps
    cpu = None
    if not args.no_cpu:
        import oracle

        rows = np.linspace(0, n - 1, 2000).astype(np.int64)
        t0 = time.perf_counter()
        oracle.volume_block_topk(coords.cpu().numpy(), cu_sb.cpu().numpy(), cu_blk.cpu().numpy(), c["batch"], c["res"],
                                 c["bbox_radius"], c["topk"], rows=rows)
        dt = time.perf_counter() - t0
        cpu = dict(value=2000 / dt, unit="tokens/s", cores=1, kind="port",
                   sample=f"2000 of {n} tokens (evenly spaced), numpy oracle on one host thread (block centres of "
                          f"the whole set included)")
    print(json.dumps(dict(
        base, value=value, n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms, scaling="weak",
        vs_baseline=None, dtype="f32", data=f"synthetic: {c['batch']} seeded random-sphere SDF shells, {nb} blocks",
        distance_evals_per_s=evals / (ms * 1e-3),
        roofline={"kernel": "volume_block_topk", "bound": "hbm", "achieved": hbm_bytes / (ms * 1e-3) / 1e9,
                  "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": hbm_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                  "traffic": None, "peak_source": f"hbm_gbs of {kind}",
                  "note": "memory is not the bound: the kernel evaluates every (token, block) distance of a batch "
                          "element on the fp32 pipe (distance_evals_per_s)"},
        cpu_baseline=cpu,
        e2e={"value": n / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
             "h2d_bytes_per_step": int(sorted_h.numel() * 4), "d2h_bytes_per_step": c["topk"] * 4},
        gpu_launches=int(launches), clocks=clk.summary())), flush=True)


def blocks_cpu_separation(coords_h):
    """Block order and separation of the geometric workload with the oracle
    (for the CPU baseline, which needs the whole set's block centres)."""
    import oracle

    c = GEO_CFG
    keys = oracle.volume_sort_keys(coords_h.numpy(), c["res"], c["block_size"])
    order = np.argsort(keys, kind="stable")
    srt = coords_h.numpy()[order]
    bs = c["block_size"]
    cs, cb = oracle.block_separation(srt, 3, [bs] * 3, c["batch"], [c["res"]] * 3)
    return cs, cb, srt


# ---------------------------------------------------------------------------
# --path head_layernorm_pack: per-head LayerNorm32 fused with the Ulysses pack
# (models_sparse/utils.py:239-270 normalisation before the exchange)
# ---------------------------------------------------------------------------

HLN_CFG = dict(n=131072, heads=16, head_dim=64, world=8)  # cfg2's q, packed for 8 ranks


def run_head_layernorm(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    c = HLN_CFG
    n, H, D, W = c["n"], c["heads"], c["head_dim"], c["world"]
    g = torch.Generator().manual_seed(args.seed)
    x_h = torch.randn(n, H, D, generator=g).bfloat16()
    gy_h = torch.randn(W, n, H // W, D, generator=g).bfloat16()
    elem = n * H * D * 2
    base = {"metric": "per-head LayerNorm + Ulysses pack, forward + backward HBM throughput", "unit": "GB/s",
            "higher_is_better": True,
            "config": {"workload": f"head_layernorm_pack fwd + bwd of [{n}, {H}, {D}] bf16 for {W} ranks",
                       "l2": "every tensor (268 MB) is larger than L2"}}
    nbytes = 2 * elem + 3 * elem  # forward: read x, write packed; backward: read x and grad, write dx

    def cpu_sample(reps):
        torch.set_num_threads(os.cpu_count() or 1)
        xs, gs = x_h[:8192], gy_h[:, :8192]
        secs = []
        for _ in range(max(1, reps)):
            t0 = time.perf_counter()
            xr = xs.float().requires_grad_()
            y = F_layer_norm(xr, D)
            y.to(torch.bfloat16).view(8192, W, H // W, D).permute(1, 0, 2, 3).contiguous()
            y.backward(gs.permute(1, 0, 2, 3).reshape(8192, H, D).float())
            secs.append(time.perf_counter() - t0)
        v = nbytes * 8192 / n / statistics.median(secs) / 1e9
        return dict(value=v, unit="GB/s", cores=torch.get_num_threads(), kind="port",
                    sample=f"8192 of {n} tokens: torch fp32 layer_norm + pack + autograd backward on the host"), secs

    if args.impl == "reference":
        cb, secs = cpu_sample(args.steps)
        v = cb["value"]
        print(json.dumps(dict(base, impl="reference", value=v, n_gpus=ws, steps=args.steps, warmup=args.warmup,
                              ms_per_step=statistics.median(secs) * 1e3, scaling="weak", vs_baseline=None,
                              dtype="bf16", data="synthetic", cpu_baseline=cb,
                              e2e={"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                   "d2h_bytes_per_step": 0})), flush=True)
        return
    from lsrm_sparse import _lib, ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    x, gy = x_h.to(dev), gy_h.to(dev)

    def step():
        ops.head_layernorm_pack(x, W)
        ops.head_layernorm_pack_bwd(x, gy)

    def unfused():  # the reference's order: LayerNorm32 as its own pass, then the pack
        y = F_layer_norm(x.float(), D).to(torch.bfloat16)
        ops.ulysses_pack(y, W)

    for _ in range(args.warmup):
        step()
        unfused()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    e0.record(stream)
    for _ in range(args.steps):
        unfused()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_unfused_fwd = e0.elapsed_time(e1) / args.steps
    value = nbytes / (ms * 1e-3) / 1e9
    peaks, kind = load_peaks()
    x_p, gy_p = x_h.pin_memory(), gy_h.pin_memory()
    x_d, gy_d = torch.empty_like(x), torch.empty_like(gy)
    out_h = torch.empty(8, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        x_d.copy_(x_p, non_blocking=True)
        gy_d.copy_(gy_p, non_blocking=True)
        dx = ops.head_layernorm_pack_bwd(x_d, gy_d)
        ops.head_layernorm_pack(x_d, W)
        out_h.copy_(dx[0, 0, :8], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps(dict(
        base, value=value, n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms, scaling="weak",
        vs_baseline=None, dtype="bf16", data="synthetic: x N(0,1), packed gradient N(0,1)",
        unfused_forward_ms=ms_unfused_fwd,
        roofline={"kernel": "head_layernorm_pack(+bwd)", "bound": "hbm", "achieved": value, "peak": peaks["hbm_gbs"],
                  "unit": "GB/s", "frac": value / peaks["hbm_gbs"], "traffic": None,
                  "peak_source": f"hbm_gbs of {kind}"},
        cpu_baseline=None if args.no_cpu else cpu_sample(3)[0],
        e2e={"value": nbytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e_ms,
             "h2d_bytes_per_step": 2 * elem, "d2h_bytes_per_step": 16},
        gpu_launches=int(launches), clocks=clk.summary())), flush=True)


# ---------------------------------------------------------------------------
# --path view_block_topk: the volume-to-image block selection of
# build_volume_to_image_attn (misc/sparse_utils.py:991-1200)
# ---------------------------------------------------------------------------

# test_rgb.sh's image settings (16 views of 768^2, patch 8, block 8, window 3x3,
# 4 blocks per view) with the surface points at half resolution (the reference
# renders them at input_image_res[1] // 2), and cfg2's 131072 voxels as queries
VIEW_CFG = dict(views=16, image_res=768, patch_size=8, block_size=8, surface_res=384, attn_winsize=3,
                topk_multiimage=4, n=131072, res=256, bbox_radius=0.5)


def view_problem(seed):
    from lsrm_sparse import synth

    c = VIEW_CFG
    vox, _ = synth.sdf_shell_voxels(c["res"], c["n"], seed)
    coords = np.zeros((len(vox), 4), np.int32)
    coords[:, 1], coords[:, 2], coords[:, 3] = vox[:, 2], vox[:, 1], vox[:, 0]
    centres, radii = synth.scene_spheres(seed)
    sc = synth.view_scene(centres, radii, 1, c["views"], c["image_res"], c["surface_res"], seed + 1)
    im = synth.image_tokens(sc["mask_input"], c["patch_size"], c["block_size"])
    return coords, im, sc


def run_view_maps(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    import types

    c = VIEW_CFG
    coords_h, im_h, sc = view_problem(args.seed)
    n, M = coords_h.shape[0], c["views"]
    win, topk = c["attn_winsize"] ** 2, c["topk_multiimage"] * M
    ps, bs, S, H = c["patch_size"], c["block_size"], c["surface_res"], c["image_res"]
    nbi = (H // (ps * bs)) ** 2
    P = (S // (H // (ps * bs))) ** 2
    base = {"metric": "volume-to-image block selection (voxel queries/s)", "unit": "tokens/s",
            "higher_is_better": True,
            "config": {"workload": f"build_volume_to_image_attn: {n} voxel queries (cfg2 shell) x {M} views of "
                                   f"{H}^2 px (patch {ps}, block {bs}: {nbi} blocks of {P} surface points per view), "
                                   f"window {win}, top-{topk}",
                       "l2": "the packed surface points (<= 38 MB) stay in L2; the selection is bound by distance "
                             "evaluations, not memory"}}
    sample = 512
    rows = np.linspace(0, n - 1, sample).astype(np.int64)

    def cpu_sample(reps):
        import oracle

        w2c_o, th_o, _ = oracle.camera_terms(sc["cameras"])
        pts_o = oracle.voxel_points(coords_h[rows], c["res"], c["bbox_radius"])
        secs = []
        for _ in range(max(1, reps)):
            t0 = time.perf_counter()
            oracle.view_block_topk(pts_o, coords_h[rows, 0], sc["mask_input"][:, :, 0], sc["surface_points"],
                                   sc["surface_masks"], w2c_o, th_o, ps, bs, win, topk, 2 * c["bbox_radius"])
            secs.append(time.perf_counter() - t0)
        v = sample / statistics.median(secs)
        return dict(value=v, unit="tokens/s", cores=1, kind="port",
                    sample=f"{sample} of {n} voxel queries (evenly spaced), numpy oracle on one host thread "
                           f"(every view's block preparation included)"), secs

    if args.impl == "reference":
        cb, secs = cpu_sample(args.steps)
        v = cb["value"]
        print(json.dumps(dict(base, impl="reference", value=v, n_gpus=ws, steps=args.steps, warmup=args.warmup,
                              ms_per_step=statistics.median(secs) * 1e3, scaling="weak", vs_baseline=None,
                              dtype="f32", data="synthetic", cpu_baseline=cb,
                              e2e={"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                   "d2h_bytes_per_step": 0})), flush=True)
        return
    from lsrm_sparse import _lib, blocks, ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    host = {"cameras_input": torch.from_numpy(sc["cameras"]), "mask_input": torch.from_numpy(sc["mask_input"])}
    dense_h = {"surface_points_input": torch.from_numpy(sc["surface_points"]),
               "masks_input": torch.from_numpy(sc["surface_masks"])}
    coords = torch.from_numpy(coords_h).to(dev)
    batch = {k: v.to(dev) for k, v in host.items()}
    dense = {k: v.to(dev) for k, v in dense_h.items()}
    w2c, th, _ = blocks.camera_terms(batch, dev)
    mi = batch["mask_input"][:, :, 0]

    def call():
        pts = blocks.voxel_points(coords, c["res"], c["bbox_radius"])
        return blocks.view_block_topk_raw(pts, coords, mi, dense["surface_points_input"], dense["masks_input"], w2c,
                                          th, None, ps, bs, win, topk, 2 * c["bbox_radius"])

    for _ in range(args.warmup):
        out = call()
    _check_device_errors(ops)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    value = n / (ms * 1e-3)
    valid = (out >= 0).sum(1).float().mean().item()
    # the reference's distance evaluations: every query against all points of its window blocks
    sel = sc["mask_input"][0, :, 0].reshape(M, H // (ps * bs), ps * bs, H // (ps * bs), ps * bs).any((2, 4))
    C = int(np.minimum(sel.reshape(M, -1).sum(1), win).sum())
    ref_evals = n * C * P
    hbm_bytes = (M * S * S * 16 + M * H * H * 4 + n * (16 + 12) + n * topk * 4)
    peaks, kind = load_peaks()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    clock_hz = 1965e6
    issue_evals = sms * 4 * 32 * clock_hz / 10  # 10 warp instructions per 32 point evaluations

    e2e = None
    if not args.no_e2e:
        args_ns = types.SimpleNamespace(block_size=bs, patch_size=ps, input_image_res=[H // 2, H],
                                        attn_winsize=c["attn_winsize"], topk_multiimage=c["topk_multiimage"],
                                        image_num_per_batch=M, bbox_radius=c["bbox_radius"], volume_res=c["res"],
                                        use_3d_aware_attn=True)
        pin = {"vol": torch.from_numpy(coords_h).pin_memory(), "im": torch.from_numpy(im_h).pin_memory()}
        pin.update({k: v.pin_memory() for k, v in host.items()})
        pin.update({k: v.pin_memory() for k, v in dense_h.items()})
        row_h = torch.empty(topk, dtype=torch.int32).pin_memory()

        def e2e_call():
            g = {k: v.to(dev, non_blocking=True) for k, v in pin.items()}
            b_ = {"cameras_input": g["cameras_input"], "mask_input": g["mask_input"]}
            d_ = {"surface_points_input": g["surface_points_input"], "masks_input": g["masks_input"]}
            res = blocks.build_volume_to_image_attn(g["im"], g["vol"], b_, d_, args_ns)
            row_h.copy_(res["block_topk"][0, 0], non_blocking=True)

        for _ in range(2):
            e2e_call()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_call()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / args.steps
        e2e = {"value": n / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": int(sum(v.numel() * v.element_size() for v in pin.values())),
               "d2h_bytes_per_step": topk * 4}
    print(json.dumps(dict(
        base, value=value, n_gpus=1, steps=args.steps, warmup=args.warmup, ms_per_step=ms, scaling="weak",
        vs_baseline=None, dtype="f32",
        data=f"synthetic: seeded random-sphere scene, {M} posed views ray-cast at {H}^2 and {S}^2, "
             f"{C} window candidates per query, {valid:.1f} blocks kept per query on average",
        ref_distance_evals_per_s=ref_evals / (ms * 1e-3),
        roofline={"kernel": "view_block_topk", "bound": "hbm", "achieved": hbm_bytes / (ms * 1e-3) / 1e9,
                  "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": hbm_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                  "traffic": None, "peak_source": f"hbm_gbs of {kind}",
                  "note": "memory is not the bound: distance evaluations on the fp32 pipe are (compute)"},
        compute={"ref_distance_evals_per_s": ref_evals / (ms * 1e-3), "issue_ceiling_evals_per_s": issue_evals,
                 "ref_evals_over_ceiling": ref_evals / (ms * 1e-3) / issue_evals,
                 "note": "the reference's evaluations (every point of every window block) against the issue rate "
                         "of scalar code at 10 warp instructions per 32 evaluations; above 1 because the kernel "
                         "evaluates only valid points, skips tiles whose bounding box cannot lower a minimum and "
                         "uses packed fp32 pairs"},
        cpu_baseline=None if args.no_cpu else cpu_sample(1)[0], e2e=e2e,
        gpu_launches=int(launches), clocks=clk.summary())), flush=True)


# ---------------------------------------------------------------------------
# --path decoder: a stack of BlockMix layers (models_sparse/utils.py:575-640)
# over voxel and image tokens with the 3D-aware maps, forward + backward +
# optimizer step (the sparse decoder's training step without its embedding
# and upsampler)
# ---------------------------------------------------------------------------

# cfg4's decoder (24 layers, hidden 1024, 16 heads, MLP 4x, multi-head: 16 key/value heads; the
# head-independent 3D-aware maps are repeated once per key/value head) and image side (8 views x 1024
# tokens); the remaining settings are the reference's argument defaults
DEC_CFG = dict(layers=24, dim=1024, q_heads=16, kv_heads=16, mlp_ratio=4.0, n_vol=524288, volume_res=512, views=8,
               image_res=256, patch_size=8, block_size=8, surface_res=128, topk_volume=8, topk_multiimage=2,
               attn_winsize=2, bbox_radius=0.5)


def decoder_problem(seed, n_vol, dev):
    import types

    from lsrm_sparse import blocks, synth

    c = DEC_CFG
    vox, shell = synth.sdf_shell_voxels(c["volume_res"], n_vol, seed)
    vol = np.zeros((len(vox), 4), np.int32)
    vol[:, 1], vol[:, 2], vol[:, 3] = vox[:, 2], vox[:, 1], vox[:, 0]
    volc = torch.from_numpy(vol).to(dev)
    volc = volc[torch.argsort(blocks.volume_sort_keys(volc, c["volume_res"], c["block_size"]), stable=True)]
    centres, radii = synth.scene_spheres(seed)
    sc = synth.view_scene(centres, radii, 1, c["views"], c["image_res"], c["surface_res"], seed + 1)
    sc["mask_input"][:] = 1.0  # every patch is a token: 8 x 1024 image tokens
    imc = torch.from_numpy(synth.image_tokens(sc["mask_input"], c["patch_size"], c["block_size"])).to(dev)
    args = types.SimpleNamespace(block_size=c["block_size"], volume_res=c["volume_res"], use_3d_aware_attn=True,
                                 topk_volume=c["topk_volume"], bbox_radius=c["bbox_radius"],
                                 attn_winsize=c["attn_winsize"], topk_multiimage=c["topk_multiimage"],
                                 image_num_per_batch=c["views"], input_image_res=[c["image_res"] // 2, c["image_res"]],
                                 patch_size=c["patch_size"])
    batch = {"mask_input": torch.from_numpy(sc["mask_input"]).to(dev),
             "cameras_input": torch.from_numpy(sc["cameras"]).to(dev)}
    dense = {"surface_points_input": torch.from_numpy(sc["surface_points"]).to(dev),
             "masks_input": torch.from_numpy(sc["surface_masks"]).to(dev)}
    maps = blocks.build_3D_aware_attn(imc.contiguous(), volc.contiguous(), batch, dense, args)  # first call: loads
    torch.cuda.synchronize()
    t0 = time.perf_counter()  # the steady-state construction time, as every training step pays it
    maps = blocks.build_3D_aware_attn(imc.contiguous(), volc.contiguous(), batch, dense, args)
    for m in maps.values():  # one copy of the head-independent selection per key/value head
        m["block_topk"] = m["block_topk"][:1].expand(c["kv_heads"], -1, -1).contiguous()
    torch.cuda.synchronize()
    map_ms = (time.perf_counter() - t0) * 1e3
    maps["_vol_index"], maps["_im_index"] = volc.contiguous(), imc.contiguous()  # the whole decoder's inputs
    return maps, volc.shape[0], imc.shape[0], shell, map_ms


def run_decoder(args):
    ws, rank, local = dist_env()
    if args.impl == "reference" and rank != 0:
        return
    if args.decoder_heads:  # other head geometries (hidden size unchanged, so head_dim = dim / Q)
        hq, hkv = (int(x) for x in args.decoder_heads.split(","))
        DEC_CFG.update(q_heads=hq, kv_heads=hkv)
    c = DEC_CFG
    n_req = args.decoder_tokens or c["n_vol"]
    base = {"metric": "sparse decoder training step (voxel tokens/s)", "unit": "tokens/s", "higher_is_better": True}
    if args.impl == "reference":
        print(json.dumps(dict(base, impl="reference", unavailable="the reference decoder needs its Triton kernels "
                              "and flash-attn on the GPU; its CPU path (Triton interpreter, fp16 only) takes ~24 s "
                              "for one 256-token attention call, so a decoder step is out of reach")), flush=True)
        return
    from lsrm_sparse import _lib, ops, ulysses
    from lsrm_sparse.decoder import BlockMix

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import datetime

        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    # every rank builds the whole problem (maps over all tokens, as each rank needs them for its heads)
    maps, nx, ny, shell, map_ms = decoder_problem(args.seed, n_req, dev)
    torch.manual_seed(args.seed)  # the same weights on every rank
    n_layers = args.decoder_layers or c["layers"]
    full = args.decoder_model == "full"
    if full:  # the whole decoder; its forward distributes and collects the tokens itself
        from lsrm_sparse.decoder import VolTransformer

        skips = tuple(i for i in (17, 11, 4) if i < n_layers)
        layers = VolTransformer(vol_res=c["volume_res"], upsample_scale=2, embed_dim=c["dim"], output_dim=32,
                                depth=n_layers, num_q_heads=c["q_heads"], num_kv_heads=c["kv_heads"],
                                mlp_ratio=c["mlp_ratio"], skip_links=skips, topk_volume=c["topk_volume"],
                                topk_multiimage=c["topk_multiimage"], use_decomposed_embed=True,
                                use_sequence_parallel=ws > 1,
                                fused_qkv=False if args.unfused_qkv else None).to(dev).to(torch.bfloat16)
    else:
        layers = torch.nn.ModuleList(
            BlockMix(c["dim"], num_q_heads=c["q_heads"], num_kv_heads=c["kv_heads"], mlp_ratio=c["mlp_ratio"],
                     topk_volume=c["topk_volume"], topk_multiimage=c["topk_multiimage"], use_sequence_parallel=ws > 1,
                     fused_qkv=False if args.unfused_qkv else None)
            for _ in range(n_layers)
        ).to(dev).to(torch.bfloat16)
    opt = torch.optim.AdamW(layers.parameters(), lr=1e-5, fused=True)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    x_in = torch.randn(nx, c["dim"], device=dev, dtype=torch.bfloat16, generator=gen)
    y_in = torch.randn(ny, c["dim"], device=dev, dtype=torch.bfloat16, generator=gen)
    if full:
        # x_in stands for the prior volume features (only the fuse_all_layers variant reads them); the
        # decoder embeds the voxel tokens itself
        vol_index, im_index = maps.pop("_vol_index"), maps.pop("_im_index")
        prior_volume = torch.zeros(1, 32, 4, 4, 4, device=dev)
        params = list(layers.parameters())
    else:
        maps.pop("_vol_index"), maps.pop("_im_index")
    if full:
        pass
    elif ws > 1:
        # sequence parallel: this rank's whole blocks of both token sets (the reference's distribute step)
        (x_in,), (y_in,), cu_x, cu_y, maps = ulysses.seq_parallel_token_blocks([x_in], [y_in], maps, "distribute")
        x_in, y_in = x_in.contiguous(), y_in.contiguous()
        params = list(layers.parameters())
    else:
        cu_x = torch.tensor([0, nx], dtype=torch.int32, device=dev)
        cu_y = torch.tensor([0, ny], dtype=torch.int32, device=dev)
    import torch.utils.checkpoint as cp

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        if full:  # embedding, layers (one checkpoint each, cp_freq = 1), upsampler, output formatting
            out, _ = layers(y, [y], im_index, x, None, vol_index, prior_volume, None, maps, c["views"])
            loss = out["sparse_feat"].float().square().mean()  # the same collected volume on every rank
        else:
            for blk in layers:  # one checkpoint per block (the reference's cp_freq = 1)
                x, y, _ = cp.checkpoint(blk, x, cu_x, y, cu_y, maps, c["views"], use_reentrant=False)
            # the loss of the whole token set: every rank's share over the global counts
            loss = x.float().square().sum() / nx + y.float().square().sum() / ny
        loss.backward()
        if ws > 1:  # weights are replicated: sum the ranks' gradients in one flat exchange
            grads = [p.grad for p in params]
            flat = torch._utils._flatten_dense_tensors(grads)
            torch.distributed.all_reduce(flat)
            for g_, f_ in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
                g_.copy_(f_)
        opt.step()
        return loss.detach()

    for _ in range(args.warmup):
        step(x_in, y_in)
    torch.cuda.synchronize()
    _check_device_errors(ops)
    mem_gb = torch.cuda.max_memory_allocated(dev) / 2 ** 30
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.launch_count()
    if ws > 1:
        torch.distributed.barrier()
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step(x_in, y_in)
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    exchange = None
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        xt = ulysses.time_exchanges(True)  # one more step with the exchanges timed
        step(x_in, y_in)
        xs = xt.stats()
        ulysses.time_exchanges(False)
        t = torch.tensor([xs["ms"]], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        exchange = {"a2a_ms_per_step": float(t.item()), "calls_per_step": xs["calls"],
                    "bytes_out_per_step": xs["bytes_out"], "share_of_step": float(t.item()) / ms,
                    "a2a_gbs": xs["bytes_out"] / (float(t.item()) * 1e-3) / 1e9 if t.item() > 0 else None,
                    "link_gbs": 900.0}
    # per-kernel device time of this library's launches in one more step (CUDA events on the launching
    # stream); the rest of the step is library GEMMs, elementwise glue and (N > 1) the exchanges
    _lib.profile_enable(True)
    step(x_in, y_in)
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    _lib.profile_enable(False)
    kernels = {k: {"ms_per_step": v[0], "launches_per_step": v[1], "share_of_step": v[0] / ms}
               for k, v in sorted(prof.items(), key=lambda kv: -kv[1][0])}
    if args.torch_profile:  # per-kernel device time of one more step, as a table on stderr
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            step(x_in, y_in)
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=70),
              file=sys.stderr, flush=True)
    e2e = None
    if not args.no_e2e:
        xh, yh = x_in.cpu().pin_memory(), y_in.cpu().pin_memory()  # this rank's tokens
        loss_h = torch.empty((), dtype=torch.float32).pin_memory()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            loss_h.copy_(step(xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True)), non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / args.steps
        if ws > 1:
            t = torch.tensor([e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": nx / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": (x_in.shape[0] + y_in.shape[0]) * c["dim"] * 2, "d2h_bytes_per_step": 4}
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        if rank != 0:
            return
    print(json.dumps(dict(
        base, value=nx / (ms * 1e-3), n_gpus=ws, steps=args.steps, warmup=args.warmup, ms_per_step=ms,
        scaling="strong", vs_baseline=None, dtype="bf16", exchange=exchange,
        config={"parallelism": f"Ulysses sequence parallel over {ws} GPUs (whole blocks per rank, all-to-all "
                               "around the attention cores, gradients all-reduced)" if ws > 1 else "single GPU",
                "model": "VolTransformer: decomposed position embedding, the layers and 3 one-sided skip blocks, "
                         "LayerNorm, upsampler (x2, 32 channels), output formatting" if full else "BlockMix stack",
                "qkv": "three Linears (library GEMMs), then the fused per-head LayerNorm" if args.unfused_qkv
                       else "one GEMM per token set with the per-head LayerNorm in its epilogue",
                "workload": f"{n_layers} BlockMix layers, hidden {c['dim']}, {c['q_heads']} query / "
                            f"{c['kv_heads']} key-value heads, MLP {c['mlp_ratio']}x; {nx} voxel tokens "
                            f"({c['volume_res']}^3 shell, {c['block_size']}^3 blocks) + {ny} image tokens "
                            f"({c['views']} views x 1024); 3D-aware maps (top-{c['topk_volume']} volume blocks, "
                            f"{c['attn_winsize']}^2 window, top-{c['topk_multiimage'] * c['views']} image blocks); "
                            f"one checkpoint per block; AdamW step",
                "l2": "activations are far larger than L2"},
        data=f"synthetic: seeded random-sphere shell ({shell} voxels before subsampling), N(0,1) token features, "
             f"random-init weights",
        attn_map_ms=map_ms, peak_mem_gib=mem_gb, cpu_baseline=None, e2e=e2e, gpu_launches=int(launches),
        clocks=clk.summary(), kernels=kernels,
        kernels_ms_per_step=sum(v["ms_per_step"] for v in kernels.values()))), flush=True)


# ---------------------------------------------------------------------------
# --path qkv_norm: CrossAttention's q / k / v projections with the per-head
# LayerNorm32 of q and k (models_sparse/utils.py:114-127, 239-270) at the
# decoder's token count: one fused GEMM against three Linears + the fused norm
# ---------------------------------------------------------------------------


def run_qkv_norm(args):
    ws, rank, local = dist_env()
    n, C, Hq, Hkv = 131072, 1024, 16, 16
    D = C // Hq
    base = {"metric": "q/k/v projection + per-head LayerNorm forward+backward (TFLOP/s of the GEMMs)",
            "unit": "TFLOP/s", "higher_is_better": True}
    if args.impl == "reference" or rank != 0:
        if rank == 0:
            print(json.dumps(dict(base, impl="reference", unavailable="the reference runs these as torch "
                                  "Linears + LayerNorm32; this path's baseline is the library-GEMM leg below")))
        return
    from lsrm_sparse import _lib, ops
    from lsrm_sparse import functional as F
    from lsrm_sparse.ulysses import head_layernorm

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.manual_seed(args.seed)
    lins = [torch.nn.Linear(C, n_, bias=False).to(dev).bfloat16() for n_ in (C, Hkv * D, Hkv * D)]
    x = torch.randn(n, C, device=dev, dtype=torch.bfloat16, requires_grad=True)
    gs = [torch.randn(n, m, device=dev, dtype=torch.bfloat16) for m in (C, Hkv * D, Hkv * D, Hkv * D)]
    N = C + 2 * Hkv * D
    flops_fwd = 2.0 * n * C * N
    flops = 3 * flops_fwd  # forward + input and weight gradients

    def fused():
        (_, q), (k, kn), (v, _) = F.qkv_norm(x, lins, [(False, True), (True, True), (True, False)], D)
        torch.autograd.backward([q, k, kn, v], gs)

    def unfused():
        q, k, v = (lin(x) for lin in lins)
        qn = head_layernorm(q.view(n, Hq, D)).view(n, -1)
        kn = head_layernorm(k.view(n, Hkv, D)).view(n, -1)
        torch.autograd.backward([qn, k, kn, v], gs)

    res = {}
    stream = torch.cuda.current_stream()
    with ClockSampler(local) as clk:
        for name, fn in (("fused", fused), ("library_gemms", unfused)):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            res[name] = {"ms_per_step": ms, "tflops": flops / (ms * 1e-3) / 1e12}
    _check_device_errors(ops)
    # the fused forward kernel alone (CUDA events on the launching stream, this library's profiler)
    _lib.profile_enable(True)
    for _ in range(args.steps):
        F.qkv_norm(x.detach(), lins, [(False, True), (True, True), (True, False)], D)
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    _lib.profile_enable(False)
    ms_k, cnt = prof.get("qkv_norm_gemm", (0.0, 1))
    k_ms = ms_k / max(cnt, 1)
    peaks, peak_kind = load_peaks()
    peak = peaks.get("bf16_tflops", 0)
    achieved = flops_fwd / (k_ms * 1e-3) / 1e12 if k_ms else None
    print(json.dumps(dict(
        base, value=res["fused"]["tflops"], n_gpus=1, steps=args.steps, warmup=args.warmup,
        ms_per_step=res["fused"]["ms_per_step"], scaling="weak", vs_baseline=None, dtype="bf16",
        data="synthetic: N(0,1) tokens, random-init Linears",
        config={"workload": f"{n} tokens, hidden {C}, {Hq} q / {Hkv} kv heads of {D}: q, k, v projections "
                            f"(N = {N}), LayerNorm32 of q and k per head, forward + backward",
                "l2": "inputs larger than L2"},
        library_gemms=res["library_gemms"], fused=res["fused"],
        roofline={"kernel": "qkv_norm_gemm", "bound": "tensor", "achieved": achieved, "peak": peak,
                  "unit": "TFLOP/s", "frac": achieved / peak if achieved and peak else None, "traffic": None,
                  "peak_source": f"bf16_tflops (burst) of {peak_kind}: the forward kernel timed alone",
                  "ms_per_launch": k_ms},
        cpu_baseline=None, e2e=None, gpu_launches=None, clocks=clk.summary())), flush=True)


def F_layer_norm(x, D):
    return torch.nn.functional.layer_norm(x, (D,), eps=1e-5)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--seed", type=int, default=0)
    # overrides of the chosen attention config (the BASELINE scaling sweep's axes)
    ap.add_argument("--tokens", type=int, default=0, help="voxel tokens N (with --grid-res: the shell's grid)")
    ap.add_argument("--grid-res", type=int, default=0, help="resolution of the random-sphere SDF grid")
    ap.add_argument("--blk-range", default="", help="octree block sizes MIN,MAX")
    ap.add_argument("--topk", type=int, default=0, help="selected blocks per query block")
    ap.add_argument("--window", type=int, default=0, help="sliding window")
    ap.add_argument("--cpu-qblocks", type=int, default=24)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--eager", action="store_true", help="time the eager step instead of its CUDA graph")
    ap.add_argument("--path", choices=["attention", "volume_output", "volume_geo_topk", "head_layernorm_pack",
                                       "view_block_topk", "decoder", "qkv_norm"],
                    default="attention",
                    help="attention: the three-branch sparse-attention step (the headline); volume_output: the "
                         "decoder's output formatting (prepare_volume_output); volume_geo_topk: the geometric "
                         "volume-to-volume block selection (build_volume_to_volume_attn); head_layernorm_pack: the "
                         "per-head LayerNorm fused with the Ulysses pack; view_block_topk: the volume-to-image "
                         "block selection (build_volume_to_image_attn); decoder: a 24-layer BlockMix "
                         "training step (decoder tokens/s)")
    ap.add_argument("--decoder-tokens", type=int, default=0, help="voxel tokens of --path decoder (default cfg4's)")
    ap.add_argument("--decoder-layers", type=int, default=0, help="layers of --path decoder (default 24)")
    ap.add_argument("--decoder-heads", default="", help="Q,KV heads of --path decoder (default 16,16; the "
                    "reference's production model uses 32,2 at hidden 1024, i.e. head_dim 32)")
    ap.add_argument("--torch-profile", action="store_true",
                    help="--path decoder: print torch.profiler's per-kernel table of one extra step on stderr")
    ap.add_argument("--unfused-qkv", action="store_true",
                    help="--path decoder: q / k / v projections as three Linears (library GEMMs) and the fused "
                         "per-head LayerNorm, instead of one GEMM with the norm in its epilogue")
    ap.add_argument("--decoder-model", choices=["blocks", "full"], default="blocks",
                    help="--path decoder: the BlockMix stack alone, or the whole VolTransformer (position "
                         "embedding, layers + skip blocks, norm, upsampler, output formatting)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = dict(CONFIGS[args.config], name=args.config)
    for key, val in (("n", args.tokens), ("res", args.grid_res), ("topk", args.topk), ("window", args.window)):
        if val:
            cfg[key] = val
            cfg["name"] = None  # no longer the named workload
    if args.blk_range:
        cfg["blk_min"], cfg["blk_max"] = (int(x) for x in args.blk_range.split(","))
        cfg["name"] = None
    if args.path == "volume_output":
        run_volume_output(args)
    elif args.path == "volume_geo_topk":
        run_volume_geo(args)
    elif args.path == "head_layernorm_pack":
        run_head_layernorm(args)
    elif args.path == "view_block_topk":
        run_view_maps(args)
    elif args.path == "decoder":
        run_decoder(args)
    elif args.path == "qkv_norm":
        run_qkv_norm(args)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
