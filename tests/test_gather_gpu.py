"""Gather kernel (gather.cu, via the C ABI): byte-identical slot contents.

Port of the reference's tests/test_gather.py plus the raw (uncompressed) path
from pinned host memory, the skip list, odd sizes (scalar path) and CTA counts.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def rand(g, *shape, device=DEV):
    return torch.randint(-(2**31), 2**31 - 1, shape, dtype=torch.int32, device=device, generator=g)


@pytest.mark.parametrize("ctas", [1, 4, 16, 64])
def test_gather_copies_rows_and_scales(ctas):
    """The reference test_gather.py case (compressed RAM rows -> staging, cache rows -> slab)."""
    from vllm_expert_pager.gather import gather_rows

    E, S = 8, 4
    WORDS, PITCH, SCALE_WORDS = (8192, 4096), (6144, 3072), (32, 16)
    g = torch.Generator(device=DEV).manual_seed(0)
    src = [rand(g, 16, p) for p in PITCH]
    cache = [rand(g, S, w) for w in WORDS]
    dst = [torch.zeros((S, w), dtype=torch.int32, device=DEV) for w in WORDS]
    stg = [torch.zeros((S, p), dtype=torch.int32, device=DEV) for p in PITCH]
    scale = [rand(g, E, w) for w in SCALE_WORDS]
    scale_dst = [torch.zeros((S, w), dtype=torch.int32, device=DEV) for w in SCALE_WORDS]
    todo = torch.tensor([3, 5, -1, -1], dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    dst_row[3], dst_row[5] = 1, 2
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    cache_row[5] = 0
    src_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    src_row[3] = 7
    gather_rows(todo, dst_row, cache_row, src_row, 2, src, cache, dst, stg, scale, scale_dst,
                ctas=ctas)
    torch.cuda.synchronize()
    for i in range(2):
        assert torch.equal(stg[i][0], src[i][9])
        assert torch.equal(dst[i][2], cache[i][0])
        assert torch.equal(scale_dst[i][1], scale[i][3])
        assert torch.equal(scale_dst[i][2], scale[i][5])
        assert not dst[i][0].any() and not dst[i][1].any() and not dst[i][3].any()
        assert not stg[i][1:].any()
        assert not scale_dst[i][0].any() and not scale_dst[i][3].any()


@pytest.mark.parametrize("words", [(262144, 131072), (1029, 517)])
def test_raw_rows_from_pinned_memory(words):
    """Uncompressed RAM rows in pinned host memory go straight into the slab (16-byte and odd sizes)."""
    from vllm_expert_pager import native
    from vllm_expert_pager.store import PinnedBuffer

    E, S, R = 32, 6, 32
    g = torch.Generator().manual_seed(1)
    bufs = [PinnedBuffer(R * w * 4, DEV) for w in words]
    src = [b.cpu[: R * w * 4].view(torch.int32).view(R, w) for b, w in zip(bufs, words)]
    for s in src:
        s.copy_(torch.randint(-(2**31), 2**31 - 1, s.shape, dtype=torch.int32, generator=g))
    views = [b.cuda[: R * w * 4].view(torch.int32).view(R, w) for b, w in zip(bufs, words)]
    cache = [torch.zeros((S, w), dtype=torch.int32, device=DEV) for w in words]
    dst = [torch.zeros((S, w), dtype=torch.int32, device=DEV) for w in words]
    scale = [torch.arange(E * 8, dtype=torch.int32, device=DEV).view(E, 8) * (i + 1)
             for i in range(2)]
    scale_dst = [torch.zeros((S, 8), dtype=torch.int32, device=DEV) for _ in range(2)]
    todo = torch.tensor([7, 30, -1, 2, 11, -1], dtype=torch.int64, device=DEV)
    skip = torch.tensor([11, -1, -1, -1, -1, -1], dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    for e, r in ((7, 4), (30, 0), (2, 5), (11, 1)):
        dst_row[e] = r
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    src_row = (torch.arange(E, device=DEV) * 7) % R
    for source in (src, views):
        for d in dst + scale_dst:
            d.zero_()
        # skip without fetch (a C-ABI-only form): the copy leaves out expert 11
        native.check(native.lib().xp_gather_rows(
            todo.data_ptr(), 6, dst_row.data_ptr(), cache_row.data_ptr(), src_row.data_ptr(), 0,
            _ptr(source[0]), cache[0].data_ptr(), dst[0].data_ptr(), None, words[0], words[0],
            _ptr(source[1]), cache[1].data_ptr(), dst[1].data_ptr(), None, words[1], words[1],
            scale[0].data_ptr(), scale_dst[0].data_ptr(), 8,
            scale[1].data_ptr(), scale_dst[1].data_ptr(), 8,
            skip.data_ptr(), 0, 0, 8, 0, None, None, None, 0, 0, 0, 0,
            torch.cuda.current_stream().cuda_stream), "gather")
        torch.cuda.synchronize()
        for i in range(2):
            for e, r in ((7, 4), (30, 0), (2, 5)):
                assert torch.equal(dst[i][r].cpu(), src[i][(e * 7) % R]), (e, i)
                assert torch.equal(scale_dst[i][r], scale[i][e])
            assert not dst[i][1].any() and not dst[i][2].any() and not dst[i][3].any()
    for b in bufs:
        b.free()


def _ptr(t):
    from vllm_expert_pager.gather import _src_ptr

    return _src_ptr(t)


def test_gather_replays_in_a_cuda_graph():
    """Index arrays change between replays; each replay copies the rows they name."""
    from vllm_expert_pager.gather import gather_rows

    E, S, W = 16, 4, 8192
    g = torch.Generator(device=DEV).manual_seed(2)
    src = [rand(g, E, W), rand(g, E, W // 2)]
    cache = [torch.zeros((S, W), dtype=torch.int32, device=DEV),
             torch.zeros((S, W // 2), dtype=torch.int32, device=DEV)]
    dst = [torch.zeros_like(c) for c in cache]
    scale = [rand(g, E, 4), rand(g, E, 4)]
    scale_dst = [torch.zeros((S, 4), dtype=torch.int32, device=DEV) for _ in range(2)]
    todo = torch.full((S,), -1, dtype=torch.int64, device=DEV)
    dst_row = torch.zeros((E,), dtype=torch.int64, device=DEV)
    cache_row = torch.full((E,), -1, dtype=torch.int64, device=DEV)
    src_row = torch.arange(E, dtype=torch.int64, device=DEV)
    args = (todo, dst_row, cache_row, src_row, 0, src, cache, dst, None, scale, scale_dst)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gather_rows(*args)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            gather_rows(*args)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    for _ in range(10):
        experts = rng.permutation(E)[:S]
        todo.copy_(torch.from_numpy(experts))
        order = np.zeros(E, dtype=np.int64)
        order[experts] = np.arange(S)
        dst_row.copy_(torch.from_numpy(order))
        graph.replay()
        torch.cuda.synchronize()
        for e in experts:
            r = int(dst_row[e])
            for i in range(2):
                assert torch.equal(dst[i][r], src[i][e])
                assert torch.equal(scale_dst[i][r], scale[i][e])
