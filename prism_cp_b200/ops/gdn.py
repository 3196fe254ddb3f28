"""Chunked gated delta rule (the Gated-DeltaNet recurrence).

Per head, with log-decay ``g_t <= 0``, ``beta_t`` in (0, 1) and state ``S`` of shape
``[dk, dv]`` (outputs ``o_t = S_t^T q_t``)::

    S_t = exp(g_t) (I - beta_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T

This is the recurrence of Yang et al. (Gated Delta Networks, 2024), the same op
as FLA's ``chunk_gated_delta_rule`` that the reference trains through
(oracle: ``experiments/performance_model/module_bench.py:148-160``). It is
evaluated in chunks of 64 tokens in the WY form: with in-chunk cumulative decay
``G`` and ``L_ij = beta_i exp(G_i - G_j) k_i.k_j`` (i > j)::

    Delta = (I + L)^-1 (beta V) - (I + L)^-1 (beta e^G K) S_c   = U - W S_c
    S_{c+1} = e^{G_last} S_c + (e^{G_last - G} K)^T Delta
    O = (e^G Q) S_c + tril(Q K^T * e^{G_i - G_j}) Delta

The chunk-parallel algebra runs as batched tensor products; the sequential
state pass is ``_StatePass`` (CUDA kernels in ``csrc/gdn_state.cu``, a chunk
loop on CPU). Sequences are padded to whole chunks with ``beta = g = 0``
tokens, which leave the state untouched. ``initial_state`` / ``final_state``
carry the recurrent state across context-parallel ranks.
"""

from __future__ import annotations

import os

import torch

from ._lib import is_cuda, lib, status

CHUNK = 64


# ---------------------------------------------------------------- state pass
def _state_pass_reference(W, U, Kd, gamma, S0, seq_chunks):
    Nc, H, C, DK = W.shape
    DV = U.shape[-1]
    nseq = len(seq_chunks) - 1
    Delta = torch.empty_like(U)
    S_all = torch.empty((Nc, H, DK, DV), dtype=W.dtype, device=W.device)
    S_final = torch.empty((nseq, H, DK, DV), dtype=W.dtype, device=W.device)
    for s in range(nseq):
        S = S0[s].clone() if S0 is not None else torch.zeros((H, DK, DV), dtype=W.dtype, device=W.device)
        for c in range(seq_chunks[s], seq_chunks[s + 1]):
            S_all[c] = S
            d = U[c] - W[c] @ S
            Delta[c] = d
            S = gamma[c][:, None, None] * S + Kd[c].transpose(-1, -2) @ d
        S_final[s] = S
    return Delta, S_all, S_final


def _state_pass_backward_reference(W, dDelta_ext, Kd, gamma, dS_ext, dS_final, seq_chunks):
    Nc, H, C, DK = W.shape
    DV = dDelta_ext.shape[-1]
    nseq = len(seq_chunks) - 1
    dDelta = torch.empty_like(dDelta_ext)
    G_next = torch.empty((Nc, H, DK, DV), dtype=W.dtype, device=W.device)
    dS0 = torch.empty((nseq, H, DK, DV), dtype=W.dtype, device=W.device)
    for s in range(nseq):
        G = dS_final[s].clone() if dS_final is not None else torch.zeros((H, DK, DV), dtype=W.dtype,
                                                                          device=W.device)
        for c in range(seq_chunks[s + 1] - 1, seq_chunks[s] - 1, -1):
            G_next[c] = G
            dd = dDelta_ext[c] + Kd[c] @ G
            dDelta[c] = dd
            G = dS_ext[c] + gamma[c][:, None, None] * G - W[c].transpose(-1, -2) @ dd
        dS0[s] = G
    return dDelta, G_next, dS0


class _StatePass(torch.autograd.Function):
    @staticmethod
    def forward(ctx, W, U, Kd, gamma, S0, seq_chunks, seq_chunks_dev):
        W, U, Kd, gamma = (t.contiguous() for t in (W, U, Kd, gamma))
        if W.is_cuda:
            Nc, H, C, DK = W.shape
            DV = U.shape[-1]
            nseq = len(seq_chunks) - 1
            Delta = torch.empty_like(U)
            S_all = torch.empty((Nc, H, DK, DV), dtype=torch.float32, device=W.device)
            S_final = torch.empty((nseq, H, DK, DV), dtype=torch.float32, device=W.device)
            lib().gdn_state_fwd(W, U, Kd, gamma, S0.contiguous() if S0 is not None else None,
                                seq_chunks_dev, Delta, S_all, S_final)
        else:
            Delta, S_all, S_final = _state_pass_reference(W, U, Kd, gamma, S0, seq_chunks)
        ctx.save_for_backward(W, Kd, gamma, S_all, Delta)
        ctx.seq_chunks, ctx.seq_chunks_dev = seq_chunks, seq_chunks_dev
        ctx.has_s0 = S0 is not None
        return Delta, S_all, S_final

    @staticmethod
    def backward(ctx, dDelta_ext, dS_ext, dS_final):
        W, Kd, gamma, S_all, Delta = ctx.saved_tensors
        if dDelta_ext is None:
            dDelta_ext = torch.zeros_like(Delta)
        if dS_ext is None:
            dS_ext = torch.zeros_like(S_all)
        dDelta_ext, dS_ext = dDelta_ext.contiguous(), dS_ext.contiguous()
        if W.is_cuda:
            dDelta = torch.empty_like(dDelta_ext)
            G_next = torch.empty_like(S_all)
            dS0 = torch.empty((len(ctx.seq_chunks) - 1,) + S_all.shape[1:], dtype=torch.float32, device=W.device)
            lib().gdn_state_bwd(W, dDelta_ext, Kd, gamma, dS_ext,
                                dS_final.contiguous() if dS_final is not None else None,
                                ctx.seq_chunks_dev, dDelta, G_next, dS0)
        else:
            dDelta, G_next, dS0 = _state_pass_backward_reference(W, dDelta_ext, Kd, gamma, dS_ext, dS_final,
                                                                 ctx.seq_chunks)
        # chunk-local gradients: dU = dDelta, dW = -dDelta S^T, dKd = Delta G^T, dgamma = <S, G>
        dU = dDelta
        dW = -(dDelta @ S_all.transpose(-1, -2))
        dKd = Delta @ G_next.transpose(-1, -2)
        dgamma = (S_all * G_next).sum(dim=(-1, -2))
        return dW, dU, dKd, dgamma, (dS0 if ctx.has_s0 else None), None, None


# ---------------------------------------------------------------- packing helpers
class ChunkLayout:
    """Maps packed varlen tokens to whole 64-token chunks (per sequence padding)."""

    def __init__(self, lengths: tuple[int, ...], device):
        self.lengths = tuple(int(n) for n in lengths)
        chunks = [(n + CHUNK - 1) // CHUNK for n in self.lengths]
        self.seq_chunks = [0]
        for c in chunks:
            self.seq_chunks.append(self.seq_chunks[-1] + c)
        self.num_chunks = self.seq_chunks[-1]
        index = []
        offset = 0
        for n, c in zip(self.lengths, chunks):
            base = len(index)
            index.extend(range(offset, offset + n))
            index.extend([-1] * (c * CHUNK - n))
            offset += n
        idx = torch.tensor(index, dtype=torch.int64)
        self.valid = idx >= 0
        self.padded_to_token = idx.clamp(min=0).to(device)
        self.valid_dev = self.valid.to(device)
        self.token_to_padded = torch.nonzero(self.valid).flatten().to(device)
        self.aligned = bool(self.valid.all())
        self.seq_chunks_dev = torch.tensor(self.seq_chunks, dtype=torch.int32, device=device)
        tok0, valid_rows = [], []
        offset = 0
        for n, c in zip(self.lengths, chunks):
            for j in range(c):
                tok0.append(offset + j * CHUNK)
                valid_rows.append(min(CHUNK, n - j * CHUNK))
            offset += n
        self.tok0_dev = torch.tensor(tok0, dtype=torch.int32, device=device)
        self.len_dev = torch.tensor(valid_rows, dtype=torch.int32, device=device)

    def pad(self, x: torch.Tensor) -> torch.Tensor:
        """[T, ...] -> [Nc, C, ...] with zeros in padded slots."""
        if self.aligned:
            return x.reshape(self.num_chunks, CHUNK, *x.shape[1:])
        out = x.new_zeros((self.num_chunks * CHUNK,) + tuple(x.shape[1:]))
        out = out.index_copy(0, self.token_to_padded, x)
        return out.reshape(self.num_chunks, CHUNK, *x.shape[1:])

    def unpad(self, y: torch.Tensor) -> torch.Tensor:
        flat = y.reshape(self.num_chunks * CHUNK, *y.shape[2:])
        if self.aligned:
            return flat
        return flat.index_select(0, self.token_to_padded)


def chunk_prep(q, k, v, g, beta, layout: ChunkLayout, scale: float | None = None) -> dict:
    """Chunk-parallel part: everything that does not depend on the initial state."""
    T, H, DK = q.shape
    scale = DK ** -0.5 if scale is None else scale
    f32 = torch.float32
    Q = layout.pad(q.to(f32)).permute(0, 2, 1, 3) * scale     # [Nc, H, C, dk]
    K = layout.pad(k.to(f32)).permute(0, 2, 1, 3)
    V = layout.pad(v.to(f32)).permute(0, 2, 1, 3)
    gl = layout.pad(g.to(f32)).permute(0, 2, 1)                # [Nc, H, C]
    bt = layout.pad(beta.to(f32)).permute(0, 2, 1)
    G = gl.cumsum(-1)
    diff = G[..., :, None] - G[..., None, :]                   # G_i - G_j
    lower = torch.ones((CHUNK, CHUNK), dtype=torch.bool, device=q.device).tril()
    decay = torch.where(lower, diff, torch.zeros_like(diff)).exp() * lower
    strict = decay * (~torch.eye(CHUNK, dtype=torch.bool, device=q.device))
    A = torch.eye(CHUNK, dtype=f32, device=q.device) + bt[..., :, None] * (K @ K.transpose(-1, -2)) * strict
    rhs = torch.cat([bt[..., None] * G.exp()[..., None] * K, bt[..., None] * V], dim=-1)
    sol = torch.linalg.solve_triangular(A, rhs, upper=False, unitriangular=True)
    G_last = G[..., -1:]
    return {"Q": Q, "K": K, "G": G, "decay": decay, "W": sol[..., :DK], "U": sol[..., DK:],
            "Kd": (G_last - G).exp()[..., None] * K, "gamma": G_last[..., 0].exp(), "layout": layout,
            "dtype": v.dtype}


def chunk_state(prep: dict, initial_state: torch.Tensor | None = None):
    """Sequential state pass: returns (Delta, S_all, S_final)."""
    layout = prep["layout"]
    return _StatePass.apply(prep["W"], prep["U"], prep["Kd"], prep["gamma"], initial_state, layout.seq_chunks,
                            layout.seq_chunks_dev)


def chunk_output(prep: dict, Delta, S_all):
    Q, K, G = prep["Q"], prep["K"], prep["G"]
    QK = (Q @ K.transpose(-1, -2)) * prep["decay"]
    O = (G.exp()[..., None] * Q) @ S_all + QK @ Delta          # [Nc, H, C, dv]
    return prep["layout"].unpad(O.permute(0, 2, 1, 3)).to(prep["dtype"])


def chunk_transition(prep: dict, seq: int) -> torch.Tensor:
    """[H, dk, dk] linear map from the initial to the final state of sequence
    ``seq`` (the recurrence with zero values, started from the identity)."""
    layout = prep["layout"]
    c0, c1 = layout.seq_chunks[seq], layout.seq_chunks[seq + 1]
    W, Kd, gamma = prep["W"][c0:c1], prep["Kd"][c0:c1], prep["gamma"][c0:c1]
    H, DK = W.shape[1], W.shape[-1]
    eye = torch.eye(DK, dtype=W.dtype, device=W.device).expand(1, H, DK, DK).contiguous()
    zeros = torch.zeros(W.shape[:-1] + (DK,), dtype=W.dtype, device=W.device)
    local = [0, c1 - c0]
    dev = torch.tensor(local, dtype=torch.int32, device=W.device)
    _, _, M = _StatePass.apply(W, zeros, Kd, gamma, eye, local, dev)
    return M[0]


def chunk_gated_delta_rule(q, k, v, g, beta, layout: ChunkLayout, scale: float | None = None,
                           initial_state: torch.Tensor | None = None):
    """Return ``(o, final_state)``.

    q, k: [T, H, dk]; v: [T, H, dv]; g (log decay), beta: [T, H];
    initial_state / final_state: [nseq, H, dk, dv] fp32.
    """
    prep = chunk_prep(q, k, v, g, beta, layout, scale)
    Delta, S_all, S_final = chunk_state(prep, initial_state)
    return chunk_output(prep, Delta, S_all), S_final


# ---------------------------------------------------------------- fused sm_100a path
def fused_supported(q: torch.Tensor, v: torch.Tensor) -> bool:
    """Shapes the fused kernels of ``csrc/gdn_chunk.cu`` take: dk = 128, dv in {128, 256}."""
    return is_cuda(q) and q.shape[-1] == 128 and v.shape[-1] in (128, 256) and q.shape[0] >= CHUNK


_SIDE = {}


SIDE_STREAM = os.environ.get("PRISM_GDN_SIDE_STREAM", "1") == "1"
# keep the forward's prep outputs, per-chunk states and Delta rows for the backward (about 2 GB per
# GDN layer per 32K tokens at 16 heads x dv 256) instead of recomputing them
SAVE_INTERMEDIATES = os.environ.get("PRISM_GDN_SAVE", "1") == "1"


def _side_stream(device) -> torch.cuda.Stream:
    s = _SIDE.get(device.index)
    if s is None:
        s = _SIDE[device.index] = torch.cuda.Stream(device=device)
    return s


class _FusedChunkRule(torch.autograd.Function):
    """Chunked gated delta rule on the fused kernels.

    Forward: prep (WY form, decays, Aqk, and the k.k / s q.k / T blocks the
    backward needs) and one tcgen05 state pass that also produces the output and
    writes the per-chunk states and Delta rows. These are kept for the backward,
    which runs the reverse state pass and the chunk-local backward (dv
    contractions on tcgen05, WY/decay terms on CUDA cores). With
    ``PRISM_GDN_SAVE=0`` only the inputs are kept and the backward recomputes
    the prep and the states (the recompute on a second stream, side by side
    with the reverse pass). Same recurrence as ``chunk_gated_delta_rule``.
    """

    @staticmethod
    def forward(ctx, q, k, v, g, beta, layout, scale, S0, keep_intermediates):
        L = lib()
        bf = torch.bfloat16
        qb, kb, vb = (t.to(bf).contiguous() for t in (q, k, v))
        gf, bt = g.float().contiguous(), beta.float().contiguous()
        st = status(q.device)
        keep = keep_intermediates and any(ctx.needs_input_grad[:5])
        Wn, U, Kd, Qg, Aqk, gam, Gc, aux = L.gdn_chunk_prep(qb, kb, vb, gf, bt, layout.tok0_dev, layout.len_dev,
                                                            scale, keep, st)
        T, H, DV = vb.shape
        o = torch.empty_like(vb)
        S_final = torch.empty((len(layout.lengths), H, qb.shape[-1], DV), dtype=torch.float32, device=q.device)
        s0 = S0.float().contiguous() if S0 is not None else None
        states = rows = None
        if keep:
            Nc = Wn.shape[0]
            states = torch.empty((Nc, H, DV, 128), dtype=torch.bfloat16, device=q.device)
            rows = torch.empty((Nc, H, DV, CHUNK), dtype=torch.bfloat16, device=q.device)
        L.gdn_chunk_fwd(Wn, U, Kd, Qg, Aqk, gam, layout.tok0_dev, layout.len_dev, layout.seq_chunks_dev, s0, o,
                        S_final, states, rows, st)
        if keep:
            ctx.save_for_backward(qb, kb, vb, gf, bt, s0, Wn, U, Kd, Qg, Aqk, gam, Gc, aux, states, rows)
        else:
            ctx.save_for_backward(qb, kb, vb, gf, bt, s0)
        ctx.kept = keep
        ctx.layout, ctx.scale, ctx.has_s0 = layout, scale, S0 is not None
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, g.dtype, beta.dtype)
        return o.to(v.dtype), S_final

    @staticmethod
    def backward(ctx, do, dS_final):
        L = lib()
        lay = ctx.layout
        saved = ctx.saved_tensors  # unpacked once (activation checkpointing allows a single unpack)
        main = torch.cuda.current_stream(saved[0].device)
        side = main
        if ctx.kept:
            qb, kb, vb, gf, bt, s0, Wn, U, Kd, Qg, Aqk, gam, Gc, aux, states, rows = saved
            st = status(qb.device)
        else:
            qb, kb, vb, gf, bt, s0 = saved
            st = status(qb.device)
            Wn, U, Kd, Qg, Aqk, gam, Gc, aux = L.gdn_chunk_prep(qb, kb, vb, gf, bt, lay.tok0_dev, lay.len_dev,
                                                                ctx.scale, True, st)
            Nc, H = Wn.shape[0], Wn.shape[1]
            DV = vb.shape[-1]
            states = torch.empty((Nc, H, DV, 128), dtype=torch.bfloat16, device=qb.device)
            rows = torch.empty((Nc, H, DV, CHUNK), dtype=torch.bfloat16, device=qb.device)
            # the recomputed forward states and the reverse pass are independent sequential
            # scans over a few dozen SMs each: run them side by side on two streams
            side = _side_stream(qb.device) if SIDE_STREAM else main
            side.wait_stream(main)
            with torch.cuda.stream(side):
                L.gdn_chunk_fwd(Wn, U, Kd, Qg, Aqk, gam, lay.tok0_dev, lay.len_dev, lay.seq_chunks_dev, s0, None,
                                None, states, rows, st)
            for t in (Wn, U, Kd, Qg, Aqk, gam, states, rows) + ((s0,) if s0 is not None else ()):
                t.record_stream(side)
        dstates, drows = torch.empty_like(states), torch.empty_like(rows)
        dS0 = torch.empty_like(s0) if ctx.has_s0 else None
        if do is None:
            do = torch.zeros_like(vb)
        dob = do.to(torch.bfloat16).contiguous()
        dsf = dS_final.float().contiguous() if dS_final is not None else None
        L.gdn_chunk_bwd_state(Wn, Kd, Qg, Aqk, gam, dob, lay.tok0_dev, lay.len_dev, lay.seq_chunks_dev, dsf, dS0,
                              dstates, drows, st)
        main.wait_stream(side)
        dq, dk, dv, dg, dbeta = L.gdn_chunk_bwd_local(qb, kb, vb, gf, bt, lay.tok0_dev, lay.len_dev, Gc, aux, states,
                                                      dstates, rows, drows, dob, ctx.scale, st, [])
        tq, tk, tv, tg, tb = ctx.dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), dg.to(tg), dbeta.to(tb), None, None, dS0, None


class _FusedAffineRule(torch.autograd.Function):
    """The zero-start recurrence of every segment plus the linear part of the first segment, on one prep.

    Outputs ``(o, S_final, L, M)``: ``o`` and ``S_final`` as ``_FusedChunkRule`` with no initial state;
    ``L`` [n0, H, dk] and ``M`` [H, dk, dk] are the outputs and the final state of the first segment's
    recurrence with zero values started from the identity (o_t += L_t S_in and S_out += M S_in for an
    incoming state S_in). Both state passes read the same prep (W, Kd, Qg, Aqk, decays do not depend
    on the values); the identity pass runs on a second stream next to the main one, forward and
    backward, and its dv contractions are added to the main pass's before the one local backward.
    """

    @staticmethod
    def forward(ctx, q, k, v, g, beta, layout, first, scale):
        L_ = lib()
        bf = torch.bfloat16
        qb, kb, vb = (t.to(bf).contiguous() for t in (q, k, v))
        gf, bt = g.float().contiguous(), beta.float().contiguous()
        st = status(q.device)
        Wn, U, Kd, Qg, Aqk, gam, Gc, aux = L_.gdn_chunk_prep(qb, kb, vb, gf, bt, layout.tok0_dev, layout.len_dev,
                                                             scale, True, st)
        T, H, DV = vb.shape
        DK = qb.shape[-1]
        Nc, nc0, n0 = Wn.shape[0], first.num_chunks, first.lengths[0]
        dev = q.device
        o = torch.empty_like(vb)
        S_final = torch.empty((len(layout.lengths), H, DK, DV), dtype=torch.float32, device=dev)
        states = torch.empty((Nc, H, DV, DK), dtype=bf, device=dev)
        rows = torch.empty((Nc, H, DV, CHUNK), dtype=bf, device=dev)
        main = torch.cuda.current_stream(dev)
        side = _side_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            eye = torch.eye(DK, dtype=torch.float32, device=dev).expand(1, H, DK, DK).contiguous()
            U0 = torch.zeros((nc0, H, CHUNK, DK), dtype=bf, device=dev)
            Lo = torch.empty((n0, H, DK), dtype=bf, device=dev)
            M = torch.empty((1, H, DK, DK), dtype=torch.float32, device=dev)
            states2 = torch.empty((nc0, H, DK, DK), dtype=bf, device=dev)
            rows2 = torch.empty((nc0, H, DK, CHUNK), dtype=bf, device=dev)
            L_.gdn_chunk_fwd(Wn[:nc0], U0, Kd[:nc0], Qg[:nc0], Aqk[:nc0], gam[:nc0], first.tok0_dev, first.len_dev,
                             first.seq_chunks_dev, eye, Lo, M, states2, rows2, st)
        L_.gdn_chunk_fwd(Wn, U, Kd, Qg, Aqk, gam, layout.tok0_dev, layout.len_dev, layout.seq_chunks_dev, None, o,
                         S_final, states, rows, st)
        main.wait_stream(side)
        for t in (Wn, Kd, Qg, Aqk, gam):
            t.record_stream(side)
        for t in (Lo, M, states2, rows2):
            t.record_stream(main)
        ctx.save_for_backward(qb, kb, vb, gf, bt, Wn, Kd, Qg, Aqk, gam, Gc, aux, states, rows, states2, rows2)
        ctx.layout, ctx.first, ctx.scale = layout, first, scale
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, g.dtype, beta.dtype)
        return o.to(v.dtype), S_final, Lo, M[0]

    @staticmethod
    def backward(ctx, do, dS_final, dLo, dM):
        L_ = lib()
        lay, first = ctx.layout, ctx.first
        (qb, kb, vb, gf, bt, Wn, Kd, Qg, Aqk, gam, Gc, aux, states, rows, states2, rows2) = ctx.saved_tensors
        st = status(qb.device)
        dev = qb.device
        nc0 = first.num_chunks
        bf = torch.bfloat16
        dob = (do if do is not None else torch.zeros_like(vb)).to(bf).contiguous()
        dsf = dS_final.float().contiguous() if dS_final is not None else None
        dL = (dLo if dLo is not None else torch.zeros((first.lengths[0],) + tuple(qb.shape[1:]),
                                                      dtype=bf, device=dev)).to(bf).contiguous()
        dMf = dM.float().contiguous()[None] if dM is not None else None
        main = torch.cuda.current_stream(dev)
        side = _side_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            dstates2, drows2 = torch.empty_like(states2), torch.empty_like(rows2)
            L_.gdn_chunk_bwd_state(Wn[:nc0], Kd[:nc0], Qg[:nc0], Aqk[:nc0], gam[:nc0], dL, first.tok0_dev,
                                   first.len_dev, first.seq_chunks_dev, dMf, None, dstates2, drows2, st)
        dstates, drows = torch.empty_like(states), torch.empty_like(rows)
        L_.gdn_chunk_bwd_state(Wn, Kd, Qg, Aqk, gam, dob, lay.tok0_dev, lay.len_dev, lay.seq_chunks_dev, dsf, None,
                               dstates, drows, st)
        main.wait_stream(side)
        for t in (dstates2, drows2):
            t.record_stream(main)
        for t in (Wn, Kd, Qg, Aqk, gam, states2, dL) + ((dMf,) if dMf is not None else ()):
            t.record_stream(side)
        dq, dk, dv, dg, dbeta = L_.gdn_chunk_bwd_local(qb, kb, vb, gf, bt, lay.tok0_dev, lay.len_dev, Gc, aux,
                                                       states, dstates, rows, drows, dob, ctx.scale, st,
                                                       [states2, dstates2, rows2, drows2, dL])
        tq, tk, tv, tg, tb = ctx.dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), dg.to(tg), dbeta.to(tb), None, None, None


def fused_affine_delta_rule(q, k, v, g, beta, layout: ChunkLayout, first: ChunkLayout,
                            scale: float | None = None):
    """``(o, S_final, L, M)``: the zero-start rule over ``layout`` and the identity-started, zero-value
    rule over its first segment (``first`` = the layout of that segment alone), sharing one prep."""
    if not (fused_supported(q, v) and first.lengths[0] >= CHUNK and first.lengths[0] == layout.lengths[0]):
        raise ValueError("fused affine rule needs the fused kernels and a first segment of at least one chunk")
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    return _FusedAffineRule.apply(q, k, v, g, beta, layout, first, scale)


def fused_gated_delta_rule(q, k, v, g, beta, layout: ChunkLayout, scale: float | None = None,
                           initial_state: torch.Tensor | None = None, keep_intermediates: bool | None = None):
    """``(o, final_state)`` of the chunked gated delta rule on the fused sm_100a kernels.

    ``keep_intermediates`` (default: on unless ``PRISM_GDN_SAVE=0``) keeps the forward's prep
    outputs and per-chunk states for the backward; False keeps only the inputs and recomputes the
    prep and the states in the backward (less memory for passes whose outputs are small)."""
    if not fused_supported(q, v):
        raise ValueError("fused gated delta rule needs CUDA tensors with dk = 128 and dv in {128, 256}")
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    keep = SAVE_INTERMEDIATES if keep_intermediates is None else bool(keep_intermediates)
    return _FusedChunkRule.apply(q, k, v, g, beta, layout, scale, initial_state, keep)


def naive_gated_delta_rule(q, k, v, g, beta, lengths, scale=None, initial_state=None):
    """Token-by-token fp64 oracle of the same recurrence (tests only)."""
    T, H, DK = q.shape
    DV = v.shape[-1]
    scale = DK ** -0.5 if scale is None else scale
    out = torch.zeros((T, H, DV), dtype=torch.float64)
    finals = []
    off = 0
    for s, n in enumerate(lengths):
        S = (initial_state[s].double().clone() if initial_state is not None
             else torch.zeros((H, DK, DV), dtype=torch.float64))
        for t in range(off, off + n):
            kt, vt, qt = k[t].double(), v[t].double(), q[t].double() * scale
            a = g[t].double().exp()[:, None, None]
            b = beta[t].double()
            S = a * S
            pred = torch.einsum("hk,hkv->hv", kt, S)
            S = S + torch.einsum("hk,hv->hkv", kt, b[:, None] * (vt - pred))
            out[t] = torch.einsum("hk,hkv->hv", qt, S)
        finals.append(S)
        off += n
    return out, torch.stack(finals)
