"""CUDA-graph capture of a forward + backward step.

The operators launch on the current stream, allocate only through the caching allocator and
never synchronise, so a step captured with torch.cuda.graph and replayed on new data gives
bit-identical results to the eager step (the launch-overhead answer for small batches).
"""

import pytest
import torch

import flash_hypercons as fh

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [4, 8, 16, 32])
def test_graph_replay_matches_eager(dtype, n):
    gen = torch.Generator(device="cuda").manual_seed(n)
    batch = 4099
    static_a = (torch.randn(batch, n, n, device="cuda", generator=gen) * 0.5).to(dtype).requires_grad_()
    static_g = torch.randn(batch, n, n, device="cuda", generator=gen).to(dtype)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):  # warm-up outside the capture (allocator pools, launch-shape caches)
            y = fh.matrix_exp(static_a)
            torch.autograd.grad(y, static_a, static_g)
    torch.cuda.current_stream().wait_stream(side)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_static = fh.matrix_exp(static_a)
        (grad_static,) = torch.autograd.grad(y_static, static_a, static_g)

    for seed in (1, 2):
        gen.manual_seed(100 * n + seed)
        new_a = (torch.randn(batch, n, n, device="cuda", generator=gen) * (0.5 * seed)).to(dtype)
        new_g = torch.randn(batch, n, n, device="cuda", generator=gen).to(dtype)
        with torch.no_grad():
            static_a.copy_(new_a)
        static_g.copy_(new_g)
        graph.replay()
        x = new_a.clone().requires_grad_()
        y = fh.matrix_exp(x)
        (grad,) = torch.autograd.grad(y, x, new_g)
        torch.cuda.synchronize()
        assert torch.equal(y_static, y)
        assert torch.equal(grad_static, grad)
    del graph
