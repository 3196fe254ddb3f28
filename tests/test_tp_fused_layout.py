"""Host-side layout of the fused TP GEMM + all-reduce regions (no GPU): offsets, alignment, growth."""

import torch

from prism_cp_b200.parallel import tp_fused


class _FakeHeap:
    created = []

    def __init__(self, group, nbytes, device):
        self.nbytes = nbytes
        self.bases = [1 << 40, 2 << 40]       # two ranks' mapped heap bases
        self.closed = False
        _FakeHeap.created.append(self)

    def close(self):
        self.closed = True


def test_regions_are_aligned_disjoint_and_grow(monkeypatch):
    calls = []

    class _Lib:
        def gemm_allreduce(self, a, b, out, a_mn, b_mn, regions, me, max_tiles, ld, seq, status):
            calls.append((regions.clone(), me, max_tiles, ld, seq, tuple(out.shape)))

    monkeypatch.setattr(tp_fused, "SymmetricHeap", _FakeHeap)
    monkeypatch.setattr(tp_fused, "lib", lambda: _Lib())
    monkeypatch.setattr(tp_fused, "status", lambda dev: None)
    monkeypatch.setattr(tp_fused.dist, "get_world_size", lambda group=None: 2)
    monkeypatch.setattr(tp_fused.dist, "get_rank", lambda group=None: 1)
    monkeypatch.setattr(tp_fused.dist, "barrier", lambda group=None: None)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: type("S", (), {"synchronize": lambda self: None})())
    f = tp_fused.FusedAllReduceGemm(object(), torch.device("cpu"))
    a = torch.zeros(1000, 64, dtype=torch.bfloat16)
    b = torch.zeros(520, 64, dtype=torch.bfloat16)
    f(a, b)
    regions, me, max_tiles, ld, seq, shape = calls[-1]
    assert me == 1 and seq == 1 and ld == 520 and shape == (1000, 520)
    tiles = (-(-1000 // 128)) * (-(-520 // 256))
    assert max_tiles >= tiles
    staging, outbuf, part, res = regions.tolist()
    for r in range(2):
        base = _FakeHeap.created[-1].bases[r]
        assert part[r] == base and res[r] == base + 2 * max_tiles * 8          # flags first
        assert staging[r] % 256 == 0 and outbuf[r] % 256 == 0
        assert staging[r] >= res[r] + max_tiles * 8                           # flags do not overlap data
        R = -(-(-(-1000 // 128)) // 2)
        assert outbuf[r] - staging[r] >= 2 * R * 128 * ld * 2                 # t staging slots
        assert outbuf[r] + 8 * 128 * ld * 2 <= base + _FakeHeap.created[-1].nbytes
    # a larger call grows the heap collectively and keeps counting sequence numbers
    first = _FakeHeap.created[-1]
    f(torch.zeros(8192, 64, dtype=torch.bfloat16), torch.zeros(4096, 64, dtype=torch.bfloat16))
    assert first.closed and _FakeHeap.created[-1] is not first
    assert calls[-1][4] == 2
    # a smaller call reuses the grown heap
    grown = _FakeHeap.created[-1]
    f(a, b)
    assert _FakeHeap.created[-1] is grown and calls[-1][4] == 3
