"""The library's launches inside a captured CUDA graph (how a serving loop replays a fixed-shape encoder).

Every entry point is stream-ordered and never synchronises the host, so it can be captured: a graph holding
the windowed and global attention layers (bf16 and f16), the fused GEMMs and the LayerNorm of a block must
replay to the same bits as the eager calls. While a stream captures, the bf16 global layers replay the
per-layer choice they had (no measurement is taken inside a graph)."""
import numpy as np
import pytest

from tests.helpers import make_inputs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def to_dev(a, dt, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_attention_layers_replay_from_a_cuda_graph(samrs, cuda, dt):
    sets = []
    for h, bh, seed in ((14, 40, 1), (64, 4, 2)):
        q, kt, v, t = make_inputs(h, h, bh, 80, seed=seed, table_std=0.5)
        sets.append((h, [to_dev(x, dt, cuda) for x in (q, kt, v, t)]))
    eager = [samrs.attention_relpos(*args, h, h, 80 ** -0.5) for h, args in sets]
    torch.cuda.synchronize()
    outs = [torch.empty_like(e) for e in eager]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on the capture stream (first-call set-up happens outside the graph)
        for (h, args), o in zip(sets, outs):
            samrs.attention_relpos(*args, h, h, 80 ** -0.5, out=o)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (h, args), o in zip(sets, outs):
            samrs.attention_relpos(*args, h, h, 80 ** -0.5, out=o)
    for o in outs:
        o.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert samrs.device_status() == 0
    for e, o in zip(eager, outs):
        assert torch.equal(e, o)
    del g


@pytest.mark.parametrize("window", [14, 0])
def test_block_replays_from_a_cuda_graph(samrs, cuda, window):
    """One ViT-B block (LayerNorm, qkv GEMM into the attention layout, attention, head merge, proj + residual,
    LayerNorm, MLP GEMMs), f16, windowed and global, captured whole: the replay matches the eager call."""
    from tests.test_gpu_block import block_params, rnd
    g = torch.Generator(device=cuda).manual_seed(21 + window)
    p = block_params(768, 12, window, g, cuda, "f16")
    x = rnd((1, 64, 64, 768), "f16", cuda, g)
    blk = samrs.Block(p, 12, window)
    eager = blk.forward(x)
    torch.cuda.synchronize()
    static_x = x.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blk.forward(static_x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_y = blk.forward(static_x)
    graph.replay()
    torch.cuda.synchronize()
    assert samrs.device_status() == 0
    assert torch.equal(static_y, eager)
    del graph
