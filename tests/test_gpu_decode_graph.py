"""The decode step as a CUDA graph (``QuestDecoder.graph``): its output equals the
eager step's bit for bit (same kernels on the same inputs), before and after the
cache grows between replays (the graph holds the cache's buffer addresses), for the
single-CTA and the chunked selection forms."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("chunks", [None, 3])
def test_graph_step_matches_eager(cuda, chunks, monkeypatch):
    from linattn_b200 import PagedKVCache, QuestDecoder

    # strict mode synchronises after every call, which a graph capture cannot hold
    monkeypatch.setenv("LINATTN_B200_STRICT", "0")
    gen = torch.Generator().manual_seed(21)
    b, hq, hkv, d, p, max_pages = 4, 16, 4, 128, 64, 40
    lens = [2000, 1500, 64 * 30, 777]
    cache = PagedKVCache(b, hkv, d, p, max_pages, dtype=torch.bfloat16, device="cuda")
    k = torch.randn(b, hkv, max(lens), d, generator=gen).to(torch.bfloat16)
    v = torch.randn(b, hkv, max(lens), d, generator=gen).to(torch.bfloat16)
    cache.fill(k.to(cuda), v.to(cuda), lens)
    dec = QuestDecoder(cache, hq, 12, sink_pages=1, select_chunks=chunks)
    g = dec.graph()
    for step in range(3):
        q = torch.randn(b, hq, 1, d, generator=gen).to(torch.bfloat16)
        eager = dec.step(q.to(cuda)).cpu()
        got = g.run(q)
        torch.cuda.synchronize()
        assert torch.equal(got, eager)
        kn = torch.randn(b, hkv, 1, d, generator=gen).to(torch.bfloat16).to(cuda)
        cache.append(kn, kn)
