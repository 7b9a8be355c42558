"""The timed step as a CUDA graph.

``bench.capture_step`` captures ``bench.forward_backward`` (the public
three-branch op, the gate Linear and the backward of all of it) at config 1.
A replay must give the eager step's gradients bit for bit, and a replay after
new query values are copied into the same buffer must give the eager
gradients of those new values (the graph reads the live input buffers)."""

import pytest
import torch

import bench
from lsrm_sparse import _lib, ops

pytestmark = pytest.mark.gpu


def test_graph_replay_equals_eager_step():
    p = bench.Problem(bench.CONFIGS["cfg1"], 0, torch.device("cuda"))
    ref = [g.clone() for g in bench._eager_grads(bench.forward_backward, p)]
    graph, launches = bench.capture_step(bench.forward_backward, p, _lib.launch_count)
    assert launches >= 10  # the step's own kernels are in the graph
    graph.replay()
    torch.cuda.synchronize()
    assert ops.read_errors() == 0
    for i, (a, b) in enumerate(zip(ref, bench.grads_of(p))):
        assert torch.equal(a, b), f"gradient {i} differs between the eager step and the replay"

    g = torch.Generator(device="cuda").manual_seed(7)
    with torch.no_grad():
        p.q.copy_((torch.randn(p.q.shape, generator=g, device="cuda") * 0.5).to(p.q.dtype))
    graph.replay()
    torch.cuda.synchronize()
    got = [t.clone() for t in bench.grads_of(p)]
    assert not torch.equal(got[0], ref[0])
    eager = bench._eager_grads(bench.forward_backward, p)
    for i, (a, b) in enumerate(zip(eager, got)):
        assert torch.equal(a, b), f"gradient {i} differs after new inputs"
    del graph
    torch.cuda.synchronize()
