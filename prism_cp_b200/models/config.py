"""Hybrid Gated-DeltaNet : GQA decoder configurations.

The layer pattern uses the reference's symbols: ``G`` = Gated-DeltaNet layer,
``*`` = grouped-query softmax attention layer; every layer is followed by a
dense SwiGLU MLP (reference pattern ``GGG*GGG*``, README.md:3). Field names
mirror the Megatron flags the reference launcher passes
(scripts/run_manual_gdn_cp_case.sh:312-394).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass(frozen=True)
class HybridConfig:
    num_layers: int
    hidden_size: int
    ffn_hidden_size: int
    vocab_size: int
    num_attention_heads: int
    num_query_groups: int
    kv_channels: int
    linear_num_key_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int = 4
    linear_attention_freq: int = 4   # one GQA layer after every (freq-1) GDN layers
    chunk_size: int = 64
    rotary_base: float = 10000.0
    norm_epsilon: float = 1e-6
    init_method_std: float = 0.02
    name: str = "custom"

    def __post_init__(self):
        if self.num_attention_heads % self.num_query_groups:
            raise ValueError("query heads must be a multiple of query groups")
        if self.linear_conv_kernel_dim != 4:
            raise ValueError("the short convolution kernel is fixed at 4")
        if self.linear_attention_freq < 1:
            raise ValueError("linear_attention_freq must be positive")

    @property
    def pattern(self) -> str:
        f = self.linear_attention_freq
        return "".join("*" if (i + 1) % f == 0 else "G" for i in range(self.num_layers))

    @property
    def gdn_qk_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def gdn_v_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_value_head_dim

    @property
    def gdn_in_proj(self) -> int:
        # q, k (qk dim each), v, output gate z (v dim each), beta and decay logits (heads
        # each), rounded up to a multiple of 8 columns so every row starts 16-byte aligned
        width = 2 * self.gdn_qk_dim + 2 * self.gdn_v_dim + 2 * self.linear_num_key_heads
        return (width + 7) // 8 * 8

    @property
    def qkv_dim(self) -> int:
        return (self.num_attention_heads + 2 * self.num_query_groups) * self.kv_channels

    def parameter_count(self) -> int:
        h, f, v = self.hidden_size, self.ffn_hidden_size, self.vocab_size
        gqa = h * self.qkv_dim + self.num_attention_heads * self.kv_channels * h + h
        conv_ch = 2 * self.gdn_qk_dim + self.gdn_v_dim
        gdn = (h * self.gdn_in_proj + conv_ch * 4 + self.gdn_v_dim * h + self.linear_value_head_dim
               + 2 * self.linear_num_key_heads + h)
        mlp = h * 2 * f + f * h + h
        per = {"G": gdn, "*": gqa}
        return 2 * v * h + h + sum(per[c] + mlp for c in self.pattern)

    def flops_per_token(self, mean_causal_context: float) -> float:
        """Training (F+B) matmul FLOPs per token; attention uses the mean causal context."""
        h, f = self.hidden_size, self.ffn_hidden_size
        dense = 0
        for c in self.pattern:
            if c == "*":
                dense += h * self.qkv_dim + self.num_attention_heads * self.kv_channels * h
            else:
                dense += h * self.gdn_in_proj + self.gdn_v_dim * h
            dense += 3 * h * f
        dense += h * self.vocab_size
        total = 6.0 * dense
        n_gqa = self.pattern.count("*")
        # QK^T and PV: 2 * 2 * ctx * d * Hq forward, x3 for F+B
        total += n_gqa * 3 * 4 * mean_causal_context * self.kv_channels * self.num_attention_heads
        # GDN chunk algebra: ~ (4 dk dv + 2 C (dk + dv)) per head forward, x3 F+B
        dk, dv, C = self.linear_key_head_dim, self.linear_value_head_dim, self.chunk_size
        total += self.pattern.count("G") * 3 * 2 * self.linear_num_key_heads * (4 * dk * dv + 2 * C * (dk + dv))
        return total

    def to_dict(self):
        return asdict(self)


def hybrid_1p3b() -> HybridConfig:
    """1.3B hybrid: 24 layers (18 GDN + 6 GQA), hidden 2048, vocab 32000,
    GQA 16q/4kv x 128, GDN 16 heads x (k 128, v 256). FFN 3584 (SwiGLU) brings
    the total to ~1.33e9 parameters with untied embeddings."""
    return HybridConfig(num_layers=24, hidden_size=2048, ffn_hidden_size=3584, vocab_size=32000,
                        num_attention_heads=16, num_query_groups=4, kv_channels=128,
                        linear_num_key_heads=16, linear_key_head_dim=128, linear_value_head_dim=256,
                        name="hybrid-1.3b")


def hybrid_7b() -> HybridConfig:
    """7B hybrid: 32 layers at 3:1, hidden 4096, vocab 32000, GQA 32q/8kv x 128,
    GDN 32 heads x (k 128, v 256), FFN 11008."""
    return HybridConfig(num_layers=32, hidden_size=4096, ffn_hidden_size=11008, vocab_size=32000,
                        num_attention_heads=32, num_query_groups=8, kv_channels=128,
                        linear_num_key_heads=32, linear_key_head_dim=128, linear_value_head_dim=256,
                        name="hybrid-7b")


def hybrid_reference_8l() -> HybridConfig:
    """The reference's own measurement model: 8 layers GGG*GGG*, hidden 4096,
    FFN 16384, vocab 32768, Q32/KV8/d128, GDN 16 x 128 (joint_cp/model.py:19-26)."""
    return HybridConfig(num_layers=8, hidden_size=4096, ffn_hidden_size=16384, vocab_size=32768,
                        num_attention_heads=32, num_query_groups=8, kv_channels=128,
                        linear_num_key_heads=16, linear_key_head_dim=128, linear_value_head_dim=128,
                        name="reference-8l")


def hybrid_tiny() -> HybridConfig:
    """4 layers (3 GDN + 1 GQA), hidden 256, vocab 4096, GQA 4q/2kv x 64,
    GDN 4 heads x 64 (CPU/gloo plumbing model)."""
    return HybridConfig(num_layers=4, hidden_size=256, ffn_hidden_size=512, vocab_size=4096,
                        num_attention_heads=4, num_query_groups=2, kv_channels=64,
                        linear_num_key_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
                        name="hybrid-tiny")


PRESETS = {
    "hybrid-1.3b": hybrid_1p3b,
    "hybrid-7b": hybrid_7b,
    "reference-8l": hybrid_reference_8l,
    "hybrid-tiny": hybrid_tiny,
}
