"""prefill and decode inside a captured CUDA graph: a serving loop captures
one step and replays it with new inputs written into the same tensors,
paying no per-call launch cost on the host. Replays must equal eager calls
bit for bit (same kernels, same inputs). A first eager call on the stream
sets up the device and the decode scratch, which capture cannot allocate."""

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("h,h_kv,d", [(12, 12, 64), (14, 2, 64), (8, 8, 128)])
def test_decode_graph_replay_equals_eager(dtype, h, h_kv, d):
    torch.manual_seed(h + d)
    b, s = 6, 3000
    q = torch.randn(b, h, 1, d, device="cuda").to(dtype)
    k = torch.randn(b, h_kv, s, d, device="cuda").to(dtype)
    v = torch.randn(b, h_kv, s, d, device="cuda").to(dtype)
    lens = torch.tensor([3000, 1, 0, 1500, 2999, 64], dtype=torch.int32,
                        device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        flashattn_cuda.decode(q, k, v, lens, d ** -0.5)  # warm-up, eager
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out = flashattn_cuda.decode(q, k, v, lens, d ** -0.5)
    torch.cuda.current_stream().wait_stream(side)
    for step in range(4):
        q.copy_(torch.randn_like(q, dtype=torch.float32).to(dtype))
        lens.copy_(torch.tensor([3000 - step, step, 0, 1500 + step, 2999, 64],
                                dtype=torch.int32))
        graph.replay()
        want = flashattn_cuda.decode(q, k, v, lens, d ** -0.5)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert flashattn_cuda.take_device_error() == 0


def test_prefill_graph_replay_equals_eager():
    torch.manual_seed(5)
    q, k, v = (torch.randn(2, 14, 1000, 64, device="cuda").half()
               for _ in range(3))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        flashattn_cuda.prefill(q, k, v, True, 0.125)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out = flashattn_cuda.prefill(q, k, v, True, 0.125)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        q.copy_(torch.randn_like(q))
        graph.replay()
        want = flashattn_cuda.prefill(q, k, v, True, 0.125)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert flashattn_cuda.take_device_error() == 0
