"""Host side of the P2P reshard: the block tables the gather kernel follows (CPU, no GPU).

The test stages every rank's outgoing rows the way ``P2PTransport.exchange`` does, replays the
gather kernel's copies block by block from the compiled tables, and requires the result to equal the
destination layout computed directly from the interval route.
"""

import pytest
import torch

from prism_cp_b200.parallel.symm import _CompiledP2PRoute, staging_offsets
from prism_cp_b200.planner.joint.ir import Group, Layout, route, spans


def _rows(layout, lengths, world):
    """Per rank: the (sample, position) of every local row, in local order."""
    out = []
    for row in spans(layout, lengths, world):
        local = []
        for s, begin, off, count in row:
            local += [(s, begin + j) for j in range(count)]
        out.append(local)
    return out


@pytest.mark.parametrize("world,lengths,src_mode,dst_mode,rows_per_block", [
    (2, {0: 4096, 1: 1024}, "contiguous", "zigzag", 64),
    (4, {0: 8192, 1: 2048, 2: 2048}, "contiguous", "zigzag", 64),
    (4, {0: 8192, 1: 2048, 2: 2048}, "zigzag", "contiguous", 100),
    (8, {i: 4096 for i in range(8)}, "contiguous", "zigzag", 64),
])
def test_gather_tables_reproduce_the_route(world, lengths, src_mode, dst_mode, rows_per_block):
    group = (Group(tuple(range(world)), tuple(sorted(lengths))),)
    src, dst = Layout(group, src_mode), Layout(group, dst_mode)
    edges = route(src, dst, lengths, world)
    src_rows, dst_rows = _rows(src, lengths, world), _rows(dst, lengths, world)
    # a row's content is its (sample, position) identity
    x = [torch.tensor([[s, p] for s, p in r], dtype=torch.int64).reshape(-1, 2) for r in src_rows]
    table = staging_offsets(edges, world)
    compiled = [_CompiledP2PRoute(edges, r, 16, rows_per_block, torch.device("cpu"), table) for r in range(world)]
    # each sender stages its outgoing rows in the order its send_index gives
    stage = [x[r][compiled[r].send_index] for r in range(world)]
    for r in range(world):
        c = compiled[r]
        out = torch.full((c.rows_out, 2), -1, dtype=torch.int64)
        for b in range(c.block_route.numel()):
            s, src_off, dst_off, n = (int(v) for v in c.routes[int(c.block_route[b])])
            r0 = int(c.block_row0[b])
            r1 = min(n, r0 + rows_per_block)
            a, d = src_off // 16 + r0, dst_off // 16 + r0
            assert (out[d:d + r1 - r0] == -1).all(), "a destination row was written twice"
            out[d:d + r1 - r0] = stage[s][a:a + r1 - r0]
        want = torch.tensor([[s, p] for s, p in dst_rows[r]], dtype=torch.int64).reshape(-1, 2)
        assert torch.equal(out, want), r
    # the largest staging area any rank needs is what the heap must hold per half
    sent = [sum(n for s, _, _, _, n in edges if s == r) for r in range(world)]
    assert max(sent) == max(int(c.send_index.numel()) for c in compiled)


def test_staging_heap_grows_only_when_a_route_needs_more(monkeypatch):
    """The transport's heap is allocated on first use and regrown, after a barrier of the group, only
    when a route's largest staging area exceeds half of it (the same decision on every rank)."""
    from prism_cp_b200.parallel import symm

    made, barriers, closed = [], [], []

    class FakeHeap:
        def __init__(self, group, nbytes, device):
            self.group, self.nbytes, self.device = group, nbytes, device
            made.append(nbytes)

        def close(self):
            closed.append(self.nbytes)

    monkeypatch.setattr(symm, "SymmetricHeap", FakeHeap)
    monkeypatch.setattr(symm.dist, "barrier", lambda group=None: barriers.append(group))
    t = symm.P2PTransport(group="team", device=torch.device("cpu"), min_bytes=1 << 20)
    t._ensure(1000)
    assert made == [1 << 20] and not barriers and t.half == 1 << 19
    t._ensure(1 << 19)                      # fits in half: no new heap
    assert made == [1 << 20]
    t._ensure((1 << 19) + 1)                # does not fit: barrier, close, twice the need
    assert barriers == ["team"] and closed == [1 << 20] and made[-1] == 2 * ((1 << 19) + 1)
    t.close()
    assert t.heap is None
