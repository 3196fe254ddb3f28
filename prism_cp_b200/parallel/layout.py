"""This rank's view of one ownership layout of one microbatch.

``LocalLayout`` is what a mixer sees: the local tokens (spans of samples in
local order), their true sequence positions (for RoPE), and three operations
that hide the context-parallel communication of the layer:

* ``attention(q, k, v)`` - causal GQA attention over the CP team (zigzag ring
  when cp > 1, the local varlen kernel when cp == 1);
* ``conv(x, w)``         - causal short conv with the 3-token halo fetched from
  the previous rank of the team for a sample continuing from it;
* ``delta_rule(...)``    - the chunked gated delta rule with the recurrent state
  of a continuing sample carried across the team (contiguous layouts).

Teams are pre-created for every aligned dyadic rank interval once (the
reference pre-creates the same groups at init, joint_cp/adapter.py:83-99), so a
new per-layer CP degree never re-initialises process groups.
"""

from __future__ import annotations

import os

import torch
import torch.utils.checkpoint

from ..ops.attention import AttentionMeta, flash_attention
from ..ops.elementwise import causal_conv1d_silu
from ..ops.gdn import ChunkLayout, chunk_gated_delta_rule, fused_gated_delta_rule, fused_supported
from ..planner.joint.ir import Layout, spans


# "peer" (default): the team's K/V (Q/dO in the backward) are staged in symmetric memory, pulled
# over NVLink by one P2P gather kernel and read by the tcgen05 kernels in global positions; it
# applies to layouts whose sequences split into whole 128-token chunks (measured 2.3 % faster per
# 1.3B step than the ring at CP = 2). Other layouts, and "ring", use the NCCL point-to-point ring
# with LSE merges. Override with PRISM_CP_ATTENTION.
CP_ATTENTION = {"impl": os.environ.get("PRISM_CP_ATTENTION", "peer")}


class LocalLayout:
    def __init__(self, layout: Layout, lengths: dict, world: int, rank: int, device, teams=None):
        self.layout, self.mode, self.world, self.rank = layout, layout.mode, world, rank
        self.lengths = lengths
        group = layout.group_of(rank)
        self.group_ranks = group.ranks
        self.cp = len(group.ranks)
        self.index = group.ranks.index(rank)
        self.samples = group.samples
        self.spans = spans(layout, lengths, world)[rank]
        self.tokens = sum(c for _, _, _, c in self.spans)
        self.device = device
        self.team = teams.team(group.ranks) if (teams is not None and self.cp > 1) else None
        self.world_group = getattr(teams, "world_group", None)
        # point-to-point peers are addressed by global rank
        to_global = getattr(teams, "global_rank", None)
        self.global_ranks = tuple(to_global(r) for r in group.ranks) if to_global is not None else group.ranks
        pos = []
        for _, begin, _, count in self.spans:
            pos.extend(range(begin, begin + count))
        self.positions = torch.tensor(pos, dtype=torch.int32, device=device)
        seg_lens = tuple(c for _, _, _, c in self.spans)
        cu = [0]
        for c in seg_lens:
            cu.append(cu[-1] + c)
        self.cu_segments = torch.tensor(cu, dtype=torch.int32, device=device)
        self.segment_lengths = seg_lens
        self._attn_meta = None
        self._chunk_layout = None
        self._cp_attn = None
        self._gdn_cp = None

    # ------------------------------------------------------------ attention
    def attention(self, q, k, v):
        if self.cp == 1:
            if self._attn_meta is None:
                lens = tuple(self.lengths[s] for s in self.samples)
                self._attn_meta = AttentionMeta(lens, lens, True, q.device)
            out, _ = flash_attention(q, k, v, self._attn_meta)
            return out
        if self.mode != "zigzag":
            raise ValueError("GQA context parallelism requires a zigzag layout")
        if self._cp_attn is None:
            from . import peer_attention
            if q.is_cuda and CP_ATTENTION["impl"] == "peer" and peer_attention.supported(self):
                self._cp_attn = peer_attention.PeerAttention(self)
            else:
                from .cp_attention import ZigzagRing
                self._cp_attn = ZigzagRing(self)
        return self._cp_attn(q, k, v)

    # ------------------------------------------------------------ GDN pieces
    def conv(self, x, weight):
        if self.cp == 1:
            return causal_conv1d_silu(x, weight, self.cu_segments)
        from .gdn_cp import conv_with_halo
        return conv_with_halo(self, x, weight)

    def chunk_layout(self) -> ChunkLayout:
        if self._chunk_layout is None:
            self._chunk_layout = ChunkLayout(self.segment_lengths, self.device)
        return self._chunk_layout

    def delta_rule(self, q, k, v, g, beta):
        if self.cp == 1:
            layout = self.chunk_layout()
            if fused_supported(q, v):
                return fused_gated_delta_rule(q, k, v, g, beta, layout)[0]
            if q.is_cuda and torch.is_grad_enabled():
                # the fp32 chunk intermediates are recomputed in the backward
                # (only the bf16 inputs stay alive between forward and backward)
                return torch.utils.checkpoint.checkpoint(
                    lambda *a: chunk_gated_delta_rule(*a, layout)[0], q, k, v, g, beta, use_reentrant=False)
            o, _ = chunk_gated_delta_rule(q, k, v, g, beta, layout)
            return o
        if self.mode != "contiguous":
            raise ValueError("GDN context parallelism requires a contiguous layout")
        from .gdn_cp import delta_rule_cp
        return delta_rule_cp(self, q, k, v, g, beta)

    # ------------------------------------------------------------ MLP placement
    def enter(self, x, source: "LocalLayout"):
        from .transport import move
        return move(x, source, self)

    def leave(self, y, target: "LocalLayout"):
        from .transport import move
        return move(y, self, target)


def single_rank_layout(lengths: dict, mode: str = "zigzag"):
    """Layout with every sample on rank 0 (CP = 1, world = 1)."""
    from ..planner.joint.ir import Group
    return Layout((Group((0,), tuple(sorted(lengths))),), mode)
