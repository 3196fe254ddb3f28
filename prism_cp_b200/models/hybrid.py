"""Native PyTorch hybrid Gated-DeltaNet : GQA decoder (no Megatron dependency).

Layer structure (pre-norm, residual, TP = PP = 1 inside a stage):
  * GQA mixer: RMSNorm -> fused QKV GEMM -> RoPE(q, k) -> causal varlen GQA
    attention (ring over the CP team when CP > 1) -> output GEMM.
  * GDN mixer: RMSNorm -> fused in-projection GEMM (q, k, v, z, beta, decay) ->
    causal conv1d(4) + SiLU on q/k/v (halo from the previous CP rank) -> L2 norm
    of q/k -> chunked gated delta rule (state carried across CP ranks) ->
    gated RMSNorm with silu(z) -> output GEMM.
  * MLP: RMSNorm -> fc1 GEMM -> SwiGLU -> fc2 GEMM.
Untied embedding and output head; the head is fused with cross-entropy.

Every mixer receives a ``LocalLayout`` (``parallel/layout.py``) that describes
this rank's tokens for the layer's ownership layout and performs the layer's
context-parallel communication, so the same module runs CP = 1 (one GPU) and
any per-layer CP degree chosen by the planner.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.cross_entropy import head_cross_entropy
from ..ops.elementwise import causal_conv1d_silu, rope, swiglu
from ..ops.norms import gated_rms_norm, l2_norm, rms_norm
from ..ops.split import split_columns
from ..parallel.tensor import column_linear, row_linear, shard_cols, shard_rows
from .config import HybridConfig


def _normal(shape, std, dtype, device, generator, shard=None):
    """Full-size init from the shared generator (same stream for every TP/PP split), then the shard."""
    t = torch.empty(shape, dtype=torch.float32, device="cpu")
    t.normal_(0.0, std, generator=generator)
    if shard is not None:
        t = shard(t)
    return nn.Parameter(t.contiguous().to(device=device, dtype=dtype))


def _replicated(t) -> nn.Parameter:
    """A parameter every TP rank holds in full (its gradient is identical on all of them)."""
    p = t if isinstance(t, nn.Parameter) else nn.Parameter(t)
    p.tp_replicated = True
    return p


def _tp_size(tp) -> int:
    return tp.tp if (tp is not None and tp.enabled) else 1


class MLP(nn.Module):
    def __init__(self, cfg: HybridConfig, dtype, device, gen, tp=None):
        super().__init__()
        h, f = cfg.hidden_size, cfg.ffn_hidden_size
        out_std = cfg.init_method_std / math.sqrt(2.0 * cfg.num_layers)
        self.tp = tp
        self.norm = _replicated(torch.ones(h, dtype=dtype, device=device))
        self.fc1 = _normal((2 * f, h), cfg.init_method_std, dtype, device, gen, lambda t: shard_rows(t, (f, f), tp))
        self.fc2 = _normal((h, f), out_std, dtype, device, gen, lambda t: shard_cols(t, tp))
        self.eps = cfg.norm_epsilon

    def forward(self, x):
        y = rms_norm(x, self.norm, self.eps)
        return row_linear(swiglu(column_linear(y, self.fc1, self.tp)), self.fc2, self.tp)


class GQAMixer(nn.Module):
    def __init__(self, cfg: HybridConfig, dtype, device, gen, tp=None):
        super().__init__()
        h = cfg.hidden_size
        t = _tp_size(tp)
        hq, hkv, d = cfg.num_attention_heads, cfg.num_query_groups, cfg.kv_channels
        if hq % t or hkv % t:
            raise ValueError("attention heads must split evenly over the tensor-parallel group")
        self.hq, self.hkv, self.d = hq // t, hkv // t, d
        self.tp = tp
        out_std = cfg.init_method_std / math.sqrt(2.0 * cfg.num_layers)
        self.norm = _replicated(torch.ones(h, dtype=dtype, device=device))
        self.qkv = _normal((cfg.qkv_dim, h), cfg.init_method_std, dtype, device, gen,
                           lambda w: shard_rows(w, (hq * d, hkv * d, hkv * d), tp))
        self.proj = _normal((h, hq * d), out_std, dtype, device, gen, lambda w: shard_cols(w, tp))
        self.eps, self.base = cfg.norm_epsilon, cfg.rotary_base

    def forward(self, x, ctx):
        T = x.shape[0]
        y = rms_norm(x, self.norm, self.eps)
        qkv = column_linear(y, self.qkv, self.tp)
        qd, kd = self.hq * self.d, self.hkv * self.d
        qs, ks, vs = split_columns(qkv, (qd, kd, kd))
        q = rope(qs, ctx.positions, self.hq, self.d, self.base).view(T, self.hq, self.d)
        k = rope(ks, ctx.positions, self.hkv, self.d, self.base).view(T, self.hkv, self.d)
        v = vs.view(T, self.hkv, self.d)
        o = ctx.attention(q, k, v)
        return row_linear(o.reshape(T, qd), self.proj, self.tp)


class GDNMixer(nn.Module):
    def __init__(self, cfg: HybridConfig, dtype, device, gen, tp=None):
        super().__init__()
        h = cfg.hidden_size
        t = _tp_size(tp)
        H = cfg.linear_num_key_heads
        if H % t:
            raise ValueError("GDN heads must split evenly over the tensor-parallel group")
        self.tp = tp
        self.H, self.dk, self.dv = H // t, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        qk, vd = cfg.gdn_qk_dim, cfg.gdn_v_dim
        self.qk_dim, self.v_dim = qk // t, vd // t
        out_std = cfg.init_method_std / math.sqrt(2.0 * cfg.num_layers)
        conv_ch = 2 * qk + vd
        self.norm = _replicated(torch.ones(h, dtype=dtype, device=device))
        def in_shard(w):
            if t == 1:
                return w
            local = shard_rows(w, (qk, qk, vd, vd, H, H), tp)
            pad = (-local.shape[0]) % 8  # 16-byte aligned output rows
            return torch.cat([local, local.new_zeros((pad, h))]) if pad else local
        self.in_proj = _normal((cfg.gdn_in_proj, h), cfg.init_method_std, dtype, device, gen, in_shard)
        bound = 1.0 / math.sqrt(cfg.linear_conv_kernel_dim)
        conv = torch.empty((conv_ch, cfg.linear_conv_kernel_dim)).uniform_(-bound, bound, generator=gen)
        self.conv = nn.Parameter(shard_rows(conv, (qk, qk, vd), tp).contiguous().to(device=device, dtype=dtype))
        a = torch.empty(H).uniform_(1.0, 16.0, generator=gen)
        dt = torch.exp(torch.empty(H).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
        self.A_log = nn.Parameter(shard_rows(a.log(), (H,), tp).contiguous().to(device=device, dtype=torch.float32))
        self.dt_bias = nn.Parameter(shard_rows(dt + torch.log(-torch.expm1(-dt)), (H,), tp).contiguous().to(
            device=device, dtype=torch.float32))
        self.out_norm = _replicated(torch.ones(self.dv, dtype=dtype, device=device))
        self.proj = _normal((h, vd), out_std, dtype, device, gen, lambda w: shard_cols(w, tp))
        self.eps = cfg.norm_epsilon

    def forward(self, x, ctx):
        T = x.shape[0]
        y = rms_norm(x, self.norm, self.eps)
        p = column_linear(y, self.in_proj, self.tp)
        c_end = 2 * self.qk_dim + self.v_dim
        conv_in, z, b, a = split_columns(p, (c_end, self.v_dim, self.H, self.H))
        qkv = ctx.conv(conv_in, self.conv)
        qs, ks, vs = split_columns(qkv, (self.qk_dim, self.qk_dim, self.v_dim))
        q = l2_norm(qs, self.H).view(T, self.H, self.dk)
        k = l2_norm(ks, self.H).view(T, self.H, self.dk)
        v = vs.view(T, self.H, self.dv)
        b, a = b.float(), a.float()
        beta = torch.sigmoid(b)
        g = -self.A_log.exp() * F.softplus(a + self.dt_bias)
        o = ctx.delta_rule(q, k, v, g, beta)
        o = gated_rms_norm(o.reshape(T, self.v_dim), z, self.out_norm, self.H, self.eps)
        return row_linear(o, self.proj, self.tp)


class HybridLayer(nn.Module):
    def __init__(self, cfg: HybridConfig, symbol: str, dtype, device, gen, tp=None):
        super().__init__()
        self.symbol = symbol
        self.mixer = (GQAMixer if symbol == "*" else GDNMixer)(cfg, dtype, device, gen, tp)
        self.mlp = MLP(cfg, dtype, device, gen, tp)

    def forward(self, x, ctx, mlp_ctx=None):
        x = x + self.mixer(x, ctx)
        if mlp_ctx is None or mlp_ctx is ctx:
            return x + self.mlp(x)
        # joint plans may run the MLP in a different ownership layout
        moved = mlp_ctx.enter(x, ctx)
        return x + mlp_ctx.leave(self.mlp(moved), ctx)


class HybridModel(nn.Module):
    def __init__(self, cfg: HybridConfig, dtype=torch.bfloat16, device="cpu", seed: int = 0,
                 layers: range | None = None, pre_process: bool = True, post_process: bool = True, tp=None):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        gen = torch.Generator(device="cpu")
        gen.manual_seed(seed)
        pattern = cfg.pattern
        # Parameters are created for every layer in order so that a pipeline
        # stage owning ``layers`` gets bitwise the same weights as the full model.
        self.layer_ids = list(layers if layers is not None else range(cfg.num_layers))
        self.pre_process, self.post_process = pre_process, post_process
        emb = _replicated(_normal((cfg.vocab_size, cfg.hidden_size), cfg.init_method_std, dtype, device, gen))
        self.embedding = emb if pre_process else None
        built = nn.ModuleList()
        for i, symbol in enumerate(pattern):
            layer = HybridLayer(cfg, symbol, dtype, device, gen, tp)
            if i in self.layer_ids:
                built.append(layer)
        self.layers = built
        self.final_norm = _replicated(torch.ones(cfg.hidden_size, dtype=dtype, device=device))
        head = _replicated(_normal((cfg.vocab_size, cfg.hidden_size), cfg.init_method_std, dtype, device, gen))
        self.head = head if post_process else None
        if not post_process:
            self.final_norm = None

    @property
    def pattern(self) -> str:
        return "".join(layer.symbol for layer in self.layers)

    def embed(self, tokens):
        return F.embedding(tokens, self.embedding)

    def run_layers(self, x, contexts, mlp_contexts=None):
        for i, layer in enumerate(self.layers):
            x = layer(x, contexts[i], None if mlp_contexts is None else mlp_contexts[i])
        return x

    def loss(self, x, labels, token_weight):
        y = rms_norm(x, self.final_norm, self.cfg.norm_epsilon)
        return head_cross_entropy(y, self.head, labels, token_weight)

    def forward(self, tokens, labels, token_weight, contexts, mlp_contexts=None):
        x = self.embed(tokens)
        x = self.run_layers(x, contexts, mlp_contexts)
        return self.loss(x, labels, token_weight)
