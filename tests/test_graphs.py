"""CUDA-graph capture of a training step through the drop-in modules: the
fused forward and backward (and the standalone encoding) replay in a captured
graph with new inputs and give the eager results bit for bit (the kernels are
deterministic), which serves the launch-bound small configurations."""
from __future__ import annotations

import copy

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _embeddings(dev):
    from piecewiselinearembeddings_optimized_b200 import workloads
    from rtdl_num_embeddings_cuda import CudaPiecewiseLinearEmbeddings

    wl = workloads.make_workload("c1", n=1024)
    m = CudaPiecewiseLinearEmbeddings([torch.from_numpy(b) for b in wl.bins], wl.d, activation=True,
                                      version="B").to(dev)
    return wl, m


def test_graph_replay_of_training_step_matches_eager(cuda_device):
    wl, m = _embeddings(cuda_device)
    rng = np.random.default_rng(0)
    x = torch.from_numpy(wl.x).to(cuda_device)
    g = torch.randn(wl.n, wl.f, wl.d, device=cuda_device)
    params = list(m.parameters())

    def step():
        y = m(x)
        y.backward(g)
        return y

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):  # warm-up outside the capture (allocator pools, attributes)
            step()
    torch.cuda.current_stream().wait_stream(side)
    for p in params:
        p.grad.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_static = step()

    ref_m = copy.deepcopy(m)  # eager twin with the same parameters (the captured grads stay in place)
    for trial in range(2):  # new inputs each replay
        x.copy_(torch.from_numpy(rng.standard_normal(wl.x.shape).astype(np.float32)))
        g.normal_()
        for p in params:
            p.grad.zero_()
        graph.replay()
        torch.cuda.synchronize()
        ref_m.zero_grad(set_to_none=True)
        ref_y = ref_m(x)
        ref_y.backward(g)
        assert torch.equal(y_static, ref_y), f"replay {trial}: output differs from eager"
        for a, b in zip(params, ref_m.parameters()):
            assert torch.equal(a.grad, b.grad), f"replay {trial}: gradient differs from eager"
    del graph


def test_graph_replay_of_encoding(cuda_device):
    from piecewiselinearembeddings_optimized_b200 import workloads
    from rtdl_num_embeddings_cuda import CudaPiecewiseLinearEncoding

    wl = workloads.make_workload("c2", n=512)
    enc = CudaPiecewiseLinearEncoding([torch.from_numpy(b) for b in wl.bins]).to(cuda_device)
    x = torch.from_numpy(wl.x).to(cuda_device)
    enc(x)  # warm-up
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = enc(x)
    x.mul_(0.5)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, enc(x))
    del graph
