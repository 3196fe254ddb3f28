"""Megatron-style command-line flags of the training entry point.

The flag names are the ones the reference's launch recipe passes to
``pretrain_gpt.py`` (scripts/run_manual_gdn_cp_case.sh:312-394), so an existing
command line carries over. Flags that select Megatron internals with no
counterpart here (attention backend, TE kernels, fusion switches) are
accepted and recorded; flags that request an unsupported combination are
rejected with a clear message.
"""

from __future__ import annotations

import argparse

from ..models.config import HybridConfig


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="prism_cp_b200 hybrid GDN:GQA training", allow_abbrev=False)
    m = p.add_argument_group("model")
    m.add_argument("--num-layers", type=int, default=24)
    m.add_argument("--hidden-size", type=int, default=2048)
    m.add_argument("--ffn-hidden-size", type=int, default=3584)
    m.add_argument("--num-attention-heads", type=int, default=16)
    m.add_argument("--num-query-groups", type=int, default=4)
    m.add_argument("--kv-channels", type=int, default=128)
    m.add_argument("--group-query-attention", action="store_true")
    m.add_argument("--experimental-attention-variant", default="gdn", choices=("gdn",))
    m.add_argument("--linear-attention-freq", type=int, default=4)
    m.add_argument("--linear-key-head-dim", type=int, default=128)
    m.add_argument("--linear-value-head-dim", type=int, default=256)
    m.add_argument("--linear-num-key-heads", type=int, default=16)
    m.add_argument("--linear-num-value-heads", type=int, default=16)
    m.add_argument("--linear-conv-kernel-dim", type=int, default=4)
    m.add_argument("--linear-cp-mode", default="chunkwise", choices=("chunkwise",))
    m.add_argument("--vocab-size", type=int, default=32000)
    m.add_argument("--normalization", default="RMSNorm", choices=("RMSNorm",))
    m.add_argument("--position-embedding-type", default="rope", choices=("rope",))
    m.add_argument("--rotary-base", type=float, default=10000.0)
    m.add_argument("--swiglu", action="store_true", default=True)
    m.add_argument("--disable-bias-linear", action="store_true", default=True)
    m.add_argument("--untie-embeddings-and-output-weights", action="store_true", default=True)
    m.add_argument("--init-method-std", type=float, default=0.02)
    m.add_argument("--norm-epsilon", type=float, default=1e-6)
    c = p.add_argument_group("context parallelism")
    c.add_argument("--context-parallel-size", type=int, default=None)
    c.add_argument("--cp-partition-mode", default="zigzag", choices=("zigzag",))
    c.add_argument("--cp-comm-type", default="p2p", choices=("p2p",))
    c.add_argument("--dynamic-context-parallel", action="store_true")
    c.add_argument("--min-dynamic-context-parallel-size", type=int, default=1)
    c.add_argument("--sequence-packing-scheduler", default="default_dynamic_cp",
                   choices=("default_dynamic_cp", "joint", "fixed", "online"))
    c.add_argument("--gdn-preserve-parent-contiguous", action="store_true")
    c.add_argument("--max-seqlen-per-dp-cp-rank", type=int, default=32768)
    c.add_argument("--joint-replay", default=None, help="replay.json from the joint planner")
    c.add_argument("--tensor-model-parallel-size", type=int, default=1)
    c.add_argument("--pipeline-model-parallel-size", type=int, default=1)
    d = p.add_argument_group("data")
    d.add_argument("--micro-batch-size", type=int, default=1)
    d.add_argument("--global-batch-size", type=int, default=8)
    d.add_argument("--seq-length", type=int, default=32768)
    d.add_argument("--use-varlen-dataset", action="store_true")
    d.add_argument("--mock-data", action="store_true", default=True)
    d.add_argument("--varlen-mock-dataset-config-json", default=None)
    d.add_argument("--packet-manifest", default=None, help="joint_cp_inputs_v1 manifest")
    d.add_argument("--seed", type=int, default=1234)
    t = p.add_argument_group("training")
    t.add_argument("--bf16", action="store_true", default=True)
    t.add_argument("--optimizer", default="adam", choices=("adam",))
    t.add_argument("--lr", type=float, default=3e-4)
    t.add_argument("--min-lr", type=float, default=3e-5)
    t.add_argument("--lr-decay-style", default="cosine", choices=("cosine", "linear", "constant"))
    t.add_argument("--lr-warmup-iters", type=int, default=0)
    t.add_argument("--lr-decay-iters", type=int, default=None)
    t.add_argument("--weight-decay", type=float, default=0.1)
    t.add_argument("--clip-grad", type=float, default=1.0)
    t.add_argument("--adam-beta1", type=float, default=0.9)
    t.add_argument("--adam-beta2", type=float, default=0.95)
    t.add_argument("--use-distributed-optimizer", action="store_true", default=True)
    t.add_argument("--calculate-per-token-loss", action="store_true", default=True)
    t.add_argument("--overlap-grad-reduce", action="store_true")
    t.add_argument("--overlap-param-gather", action="store_true")
    t.add_argument("--ddp-bucket-size", type=int, default=None)
    t.add_argument("--train-iters", type=int, default=10)
    t.add_argument("--recompute-granularity", default=None, choices=(None, "full", "selective"))
    t.add_argument("--recompute-tokens", type=int, default=None,
                   help="recompute the layers of microbatches holding more than this many tokens on a rank "
                        "(--recompute-granularity full: every microbatch)")
    t.add_argument("--distributed-backend", default="nccl", choices=("nccl", "gloo"))
    t.add_argument("--distributed-timeout-minutes", type=int, default=30)
    k = p.add_argument_group("checkpoint and logging")
    k.add_argument("--ckpt-format", default="torch_dist", choices=("torch_dist",))
    k.add_argument("--save", default=None)
    k.add_argument("--load", default=None)
    k.add_argument("--save-interval", type=int, default=None)
    k.add_argument("--log-interval", type=int, default=1)
    k.add_argument("--records", default=None, help="directory for steps_rank*.jsonl")
    k.add_argument("--profile", action="store_true")
    k.add_argument("--profile-step-start", type=int, default=3)
    k.add_argument("--profile-step-end", type=int, default=4)
    k.add_argument("--profile-ranks", type=int, nargs="*", default=[0])
    k.add_argument("--nvtx-ranges", action="store_true")
    k.add_argument("--device", default="cuda", choices=("cuda", "cpu"))
    return p


def validate(args) -> None:
    if args.tensor_model_parallel_size != 1 and args.pipeline_model_parallel_size != 1:
        raise SystemExit("tensor and pipeline parallelism cannot be combined in one run")
    if args.recompute_granularity not in (None, "full", "selective"):
        raise SystemExit("unknown recompute granularity")
    if args.linear_num_value_heads != args.linear_num_key_heads:
        raise SystemExit("GDN value heads must equal key heads")
    if args.num_attention_heads % args.num_query_groups:
        raise SystemExit("attention heads must be a multiple of query groups")


def model_config(args) -> HybridConfig:
    return HybridConfig(num_layers=args.num_layers, hidden_size=args.hidden_size,
                        ffn_hidden_size=args.ffn_hidden_size, vocab_size=args.vocab_size,
                        num_attention_heads=args.num_attention_heads, num_query_groups=args.num_query_groups,
                        kv_channels=args.kv_channels, linear_num_key_heads=args.linear_num_key_heads,
                        linear_key_head_dim=args.linear_key_head_dim,
                        linear_value_head_dim=args.linear_value_head_dim,
                        linear_conv_kernel_dim=args.linear_conv_kernel_dim,
                        linear_attention_freq=args.linear_attention_freq, rotary_base=args.rotary_base,
                        norm_epsilon=args.norm_epsilon, init_method_std=args.init_method_std, name="cli")
