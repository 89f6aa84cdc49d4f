"""The ops trace under torch.compile(fullgraph=True) and replay inside a CUDA graph (reference
tests/test_torch_compile.py), which needs the fake kernels and a decode path with no host sync."""

import pytest
import torch

import flash_lab

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("impl", ["sm100", "mma_pipelined"])
def test_attention_compiles_without_graph_breaks(impl):
    torch._dynamo.reset()

    def block(q, k, v):
        out, lse = flash_lab.attention(q, k, v, causal=True, impl=impl, return_lse=True)
        return out * 2 + 1, lse.exp()

    q = torch.randn(2, 96, 4, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(2, 96, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(2, 96, 2, 128, device="cuda", dtype=torch.bfloat16)
    compiled = torch.compile(block, fullgraph=True)
    for got, want in zip(compiled(q, k, v), block(q, k, v), strict=True):
        torch.testing.assert_close(got, want)


@pytest.mark.parametrize("impl", ["decode_inplace", "splitkv"])
def test_decode_compiles_without_graph_breaks(impl):
    torch._dynamo.reset()

    def step(q, k_cache, v_cache, seq_lens):
        return flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl) * 2

    q = torch.randn(3, 1, 8, 128, device="cuda", dtype=torch.bfloat16)
    k_cache = torch.randn(3, 500, 2, 128, device="cuda", dtype=torch.bfloat16)
    v_cache = torch.randn(3, 500, 2, 128, device="cuda", dtype=torch.bfloat16)
    seq_lens = torch.tensor([500, 7, 260], device="cuda", dtype=torch.int32)
    compiled = torch.compile(step, fullgraph=True)
    torch.testing.assert_close(compiled(q, k_cache, v_cache, seq_lens),
                               step(q, k_cache, v_cache, seq_lens))


def test_decode_replays_in_a_cuda_graph():
    q = torch.randn(2, 1, 16, 128, device="cuda", dtype=torch.bfloat16)
    k_cache = torch.randn(2, 4096, 4, 128, device="cuda", dtype=torch.bfloat16)
    v_cache = torch.randn(2, 4096, 4, 128, device="cuda", dtype=torch.bfloat16)
    seq_lens = torch.tensor([4096, 100], device="cuda", dtype=torch.int32)
    flash_lab.decode(q, k_cache, v_cache, seq_lens)   # warm-up outside capture
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            out = flash_lab.decode(q, k_cache, v_cache, seq_lens)
    torch.cuda.current_stream().wait_stream(stream)
    for lens in ([4096, 100], [17, 3000]):
        seq_lens.copy_(torch.tensor(lens, device="cuda", dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, flash_lab.decode(q, k_cache, v_cache, seq_lens),
                                   rtol=0, atol=0)
