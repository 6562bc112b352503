"""Command-line surface: the reference's flag names, defaults and cross-flag validation.

One argparse namespace carries cluster, training, rollout, algorithm, data, evaluation,
fault-tolerance, router, tracking, debug and CI options. Flags that configure the reference's
external engines keep working: Megatron-style model/optimizer flags map onto this trainer, and
every `--sglang-<name>` flag is accepted and forwarded to the in-process rollout engine
(unknown engine options are recorded and ignored).

Reference: miles/utils/arguments.py (groups :41-1624, parse_args :1691, validation :1805-2096),
backends/sglang_utils/arguments.py (--sglang-* mirroring), megatron_utils/arguments.py.
"""
from __future__ import annotations

import argparse
import os
from typing import Callable

import yaml

from miles_b200.utils.misc import load_function


def _str2bool(v):
    if isinstance(v, bool):
        return v
    return str(v).lower() in ("1", "true", "yes", "y")


def add_cluster_args(p):
    g = p.add_argument_group("cluster")
    g.add_argument("--actor-num-nodes", type=int, default=1)
    g.add_argument("--actor-num-gpus-per-node", type=int, default=8)
    g.add_argument("--critic-num-nodes", type=int, default=None)
    g.add_argument("--critic-num-gpus-per-node", type=int, default=None)
    g.add_argument("--rollout-num-gpus", type=int, default=None)
    g.add_argument("--rollout-num-gpus-per-engine", type=int, default=1)
    g.add_argument("--num-gpus-per-node", type=int, default=8)
    g.add_argument("--colocate", action="store_true", default=False)
    g.add_argument("--offload", action="store_true", default=False)
    g.add_argument("--offload-train", action="store_true", default=None)
    g.add_argument("--offload-rollout", action="store_true", default=None)
    g.add_argument("--offload-rollout-level", nargs="+", default=["kv_cache", "weight", "cuda_graph"])
    g.add_argument("--distributed-backend", default="nccl")
    g.add_argument("--distributed-timeout-minutes", type=int, default=10)
    g.add_argument("--train-env-vars", type=str, default="{}")
    g.add_argument("--train-memory-margin-bytes", type=int, default=1 << 30)


def add_train_args(p):
    g = p.add_argument_group("train")
    g.add_argument("--train-backend", choices=["megatron", "fsdp", "b200"], default="b200",
                   help="all values run this framework's trainer; kept for script compatibility")
    g.add_argument("--qkv-format", choices=["thd", "bshd"], default="thd")
    g.add_argument("--true-on-policy-mode", action="store_true", default=False)
    g.add_argument("--megatron-to-hf-mode", choices=["raw", "bridge"], default="raw")
    g.add_argument("--custom-model-provider-path", default=None)
    g.add_argument("--recompute-loss-function", action="store_true", default=False)
    g.add_argument("--log-probs-chunk-size", type=int, default=-1)
    g.add_argument("--allgather-cp", action="store_true", default=False)
    g.add_argument("--model-name", default=None, help="model preset (e.g. qwen3-30b-a3b)")
    # model / optimizer (Megatron-compatible names)
    g.add_argument("--tensor-model-parallel-size", type=int, default=1)
    g.add_argument("--pipeline-model-parallel-size", type=int, default=1)
    g.add_argument("--virtual-pipeline-model-parallel-size", type=int, default=None,
                   help="model chunks per pipeline rank (interleaved 1F1B schedule)")
    g.add_argument("--decoder-first-pipeline-num-layers", type=int, default=None,
                   help="layers on the first pipeline stage (the rest split evenly)")
    g.add_argument("--decoder-last-pipeline-num-layers", type=int, default=None,
                   help="layers on the last pipeline stage")
    g.add_argument("--context-parallel-size", type=int, default=1)
    g.add_argument("--expert-model-parallel-size", type=int, default=1)
    g.add_argument("--expert-tensor-parallel-size", type=int, default=None,
                   help="TP ranks that split each routed expert: 1 (whole experts, each TP rank "
                        "routes its share of the tokens) or the TP size (default)")
    g.add_argument("--sequence-parallel", action="store_true", default=False)
    g.add_argument("--vocab-parallel-logprob", action="store_true", default=False,
                   help="under TP, split the LM-head logits of the trainer's log-probs over the TP ranks")
    g.add_argument("--lr", type=float, default=1e-6)
    g.add_argument("--min-lr", type=float, default=0.0)
    g.add_argument("--lr-decay-style", default="constant",
                   choices=["constant", "linear", "cosine", "inverse-square-root"])
    g.add_argument("--lr-warmup-init", type=float, default=0.0)
    g.add_argument("--lr-warmup-iters", type=int, default=0)
    g.add_argument("--lr-warmup-fraction", type=float, default=None)
    g.add_argument("--lr-decay-iters", type=int, default=None)
    g.add_argument("--weight-decay", type=float, default=0.1)
    g.add_argument("--adam-beta1", type=float, default=0.9)
    g.add_argument("--adam-beta2", type=float, default=0.98)
    g.add_argument("--adam-eps", type=float, default=1e-8)
    g.add_argument("--clip-grad", type=float, default=1.0)
    g.add_argument("--optimizer-cpu-offload", action="store_true", default=False)
    g.add_argument("--accumulate-allreduce-grads-in-fp32", action="store_true", default=False)
    g.add_argument("--micro-batch-size", type=int, default=1)
    g.add_argument("--global-batch-size", type=int, default=None)
    g.add_argument("--seq-length", type=int, default=4096)
    g.add_argument("--bf16", action="store_true", default=True)
    g.add_argument("--recompute-granularity", default="full")
    g.add_argument("--recompute-method", default="uniform")
    g.add_argument("--recompute-num-layers", type=int, default=1)
    g.add_argument("--seed", type=int, default=1234)
    g.add_argument("--load", default=None)
    g.add_argument("--save", default=None)
    g.add_argument("--save-interval", type=int, default=None)
    g.add_argument("--async-save", action="store_true", default=False)
    g.add_argument("--no-save-optim", action="store_true", default=False)
    g.add_argument("--no-load-optim", action="store_true", default=False)
    g.add_argument("--reset-optimizer-states", action="store_true", default=False)
    g.add_argument("--low-memory-resume", action="store_true", default=False)
    g.add_argument("--critic-load", default=None)
    g.add_argument("--critic-save", default=None)
    g.add_argument("--critic-lr", type=float, default=None)
    g.add_argument("--critic-lr-warmup-iters", type=int, default=0)
    g.add_argument("--num-critic-only-steps", type=int, default=0)
    g.add_argument("--padded-vocab-size", type=int, default=None)


def add_rollout_args(p):
    g = p.add_argument_group("rollout")
    g.add_argument("--hf-checkpoint", default=None)
    g.add_argument("--model-path", dest="hf_checkpoint_alias", default=None, help=argparse.SUPPRESS)
    g.add_argument("--rollout-function-path", default="miles_b200.rollout.default.generate_rollout")
    g.add_argument("--rollout-temperature", type=float, default=1.0)
    g.add_argument("--rollout-top-p", type=float, default=1.0)
    g.add_argument("--rollout-top-k", type=int, default=-1)
    g.add_argument("--rollout-max-context-len", type=int, default=None)
    g.add_argument("--rollout-max-prompt-len", type=int, default=None)
    g.add_argument("--rollout-max-response-len", type=int, default=1024)
    g.add_argument("--rollout-skip-special-tokens", action="store_true", default=False)
    g.add_argument("--rollout-stop", nargs="+", default=None)
    g.add_argument("--rollout-stop-token-ids", type=int, nargs="+", default=None)
    g.add_argument("--rollout-shuffle", action="store_true", default=False)
    g.add_argument("--rollout-seed", type=int, default=42)
    g.add_argument("--over-sampling-batch-size", type=int, default=None)
    g.add_argument("--dynamic-sampling-filter-path", default=None)
    g.add_argument("--partial-rollout", action="store_true", default=False)
    g.add_argument("--mask-offpolicy-in-partial-rollout", action="store_true", default=False)
    g.add_argument("--max-weight-staleness", type=int, default=None)
    g.add_argument("--custom-generate-function-path", default=None)
    g.add_argument("--update-weight-buffer-size", type=int, default=512 * 1024 ** 2)
    g.add_argument("--update-weights-interval", type=int, default=1)
    g.add_argument("--pause-generation-mode", choices=["abort", "retract", "in_place"], default="abort")
    g.add_argument("--keep-old-actor", action="store_true", default=False)
    g.add_argument("--rollout-external", action="store_true", default=False)
    g.add_argument("--rollout-external-engine-addrs", nargs="+", default=None)
    g.add_argument("--update-weight-transfer-mode", choices=["broadcast", "p2p"], default="broadcast")
    g.add_argument("--update-weight-transport", choices=["auto", "peer", "nccl"], default="auto",
                   help="trainer -> engine refit: kernels storing into the engines' IPC-mapped "
                        "staging over NVLink (peer), or NCCL broadcast")
    g.add_argument("--grad-reduce", choices=["nccl", "peer"], default="nccl",
                   help="data-parallel gradient reduce-scatter: NCCL, or the fused peer-memory "
                        "kernel (sum + cast + shard norm in one pass over a resident symmetric "
                        "gradient buffer; the buffer is not released during rollout)")
    g.add_argument("--fp8-format", choices=["e4m3", "hybrid"], default=None,
                   help="block-scaled fp8 forward GEMMs in training and rollout (e4m3 only)")
    g.add_argument("--fp8-recipe", choices=["blockwise", "mxfp8", "delayed", "tensorwise"],
                   default="blockwise", help="fp8 scaling recipe (blockwise: 1x128 activation "
                   "and 128x128 weight scales)")
    g.add_argument("--update-weight-quant", choices=["none", "fp8"], default="none",
                   help="quantise weights at refit (fp8: 128x128 block-scaled e4m3 broadcast)")
    g.add_argument("--fully-async", action="store_true", default=False,
                   help="train_async.py: keep generation running continuously on the rollout GPUs")
    g.add_argument("--p2p-transfer-num-workers", type=int, default=4)
    g.add_argument("--p2p-transfer-timeout", type=float, default=300.0)
    g.add_argument("--rollout-task-type", default=None)
    g.add_argument("--rollout-buffer-url", default=None)
    g.add_argument("--fetch-trajectory-retry-times", type=int, default=-1)
    g.add_argument("--min-batch-collection-ratio", type=float, default=1.0)
    g.add_argument("--use-distributed-post", action="store_true", default=False)
    g.add_argument("--rollout-max-batch", type=int, default=256,
                   help="maximum concurrently decoded sequences per engine")
    g.add_argument("--no-cuda-graph", action="store_true", default=False)


def add_ft_args(p):
    g = p.add_argument_group("fault tolerance")
    g.add_argument("--use-fault-tolerance", action="store_true", default=False)
    g.add_argument("--rollout-health-check-interval", type=float, default=30.0)
    g.add_argument("--rollout-health-check-timeout", type=float, default=30.0)
    g.add_argument("--rollout-health-check-first-wait", type=float, default=0.0)


def add_data_args(p):
    g = p.add_argument_group("data")
    g.add_argument("--num-rollout", type=int, default=None)
    g.add_argument("--num-epoch", type=int, default=None)
    g.add_argument("--disable-rollout-global-dataset", action="store_true", default=False)
    g.add_argument("--data-source-path", default="miles_b200.rollout.data_source.RolloutDataSourceWithBuffer")
    g.add_argument("--prompt-data", default=None)
    g.add_argument("--apply-chat-template", action="store_true", default=False)
    g.add_argument("--apply-chat-template-kwargs", type=str, default="{}")
    g.add_argument("--chat-template-path", default=None)
    g.add_argument("--input-key", default="input")
    g.add_argument("--label-key", default=None)
    g.add_argument("--metadata-key", default="metadata")
    g.add_argument("--tool-key", default=None)
    g.add_argument("--multimodal-keys", type=str, default=None)
    g.add_argument("--rollout-batch-size", type=int, default=None)
    g.add_argument("--n-samples-per-prompt", type=int, default=1)
    g.add_argument("--num-steps-per-rollout", type=int, default=None)
    g.add_argument("--balance-data", action="store_true", default=False)
    g.add_argument("--use-dynamic-batch-size", action="store_true", default=False)
    g.add_argument("--max-tokens-per-gpu", type=int, default=None)
    g.add_argument("--log-probs-max-tokens-per-gpu", type=int, default=None)
    g.add_argument("--use-dynamic-global-batch-size", action="store_true", default=False)
    g.add_argument("--data-pad-size-multiplier", type=int, default=128)
    g.add_argument("--start-rollout-id", type=int, default=None)
    g.add_argument("--loss-mask-type", default="qwen")


def add_eval_args(p):
    g = p.add_argument_group("eval")
    g.add_argument("--eval-function-path", default=None)
    g.add_argument("--eval-interval", type=int, default=None)
    g.add_argument("--eval-prompt-data", nargs="+", default=None)
    g.add_argument("--eval-config", default=None)
    g.add_argument("--skip-eval-before-train", action="store_true", default=False)
    g.add_argument("--eval-input-key", default=None)
    g.add_argument("--eval-label-key", default=None)
    g.add_argument("--eval-tool-key", default=None)
    g.add_argument("--n-samples-per-eval-prompt", type=int, default=1)
    g.add_argument("--eval-temperature", type=float, default=None)
    g.add_argument("--eval-top-p", type=float, default=None)
    g.add_argument("--eval-top-k", type=int, default=None)
    g.add_argument("--eval-max-response-len", type=int, default=None)
    g.add_argument("--eval-max-prompt-len", type=int, default=None)
    g.add_argument("--eval-min-new-tokens", type=int, default=None)
    g.add_argument("--eval-max-context-len", type=int, default=None)
    g.add_argument("--eval-reward-key", default=None)


def add_algo_args(p):
    g = p.add_argument_group("algorithm")
    g.add_argument("--ref-load", default=None)
    g.add_argument("--ref-ckpt-step", type=int, default=None)
    g.add_argument("--ref-update-interval", type=int, default=None)
    g.add_argument("--save-hf", default=None)
    g.add_argument("--eps-clip", type=float, default=0.2)
    g.add_argument("--eps-clip-high", type=float, default=None)
    g.add_argument("--eps-clip-c", type=float, default=None)
    g.add_argument("--value-clip", type=float, default=0.2)
    g.add_argument("--kl-coef", type=float, default=0.0)
    g.add_argument("--loss-type", choices=["policy_loss", "sft_loss", "custom_loss"], default="policy_loss")
    g.add_argument("--custom-loss-function-path", default=None)
    g.add_argument("--kl-loss-type", choices=["k1", "k2", "k3", "low_var_kl"], default="k1")
    g.add_argument("--advantage-estimator", default="grpo",
                   choices=["grpo", "gspo", "reinforce_plus_plus", "reinforce_plus_plus_baseline",
                            "ppo", "on_policy_distillation"])
    g.add_argument("--disable-compute-advantages-and-returns", action="store_true", default=False)
    g.add_argument("--use-kl-loss", action="store_true", default=False)
    g.add_argument("--kl-loss-coef", type=float, default=0.0)
    g.add_argument("--use-unbiased-kl", action="store_true", default=False)
    g.add_argument("--entropy-coef", type=float, default=0.0)
    g.add_argument("--gamma", type=float, default=1.0)
    g.add_argument("--lambd", type=float, default=1.0)
    g.add_argument("--normalize-advantages", action="store_true", default=False)
    g.add_argument("--disable-grpo-std-normalization", action="store_true", default=False)
    g.add_argument("--disable-rewards-normalization", action="store_true", default=False)
    g.add_argument("--use-rollout-entropy", action="store_true", default=False)
    g.add_argument("--use-rollout-logprobs", action="store_true", default=False)
    g.add_argument("--use-tis", action="store_true", default=False)
    g.add_argument("--tis-clip", type=float, default=2.0)
    g.add_argument("--tis-clip-low", type=float, default=0.0)
    g.add_argument("--custom-tis-function-path", default=None)
    g.add_argument("--custom-pg-loss-reducer-function-path", default=None)
    g.add_argument("--use-routing-replay", action="store_true", default=False)
    g.add_argument("--use-rollout-routing-replay", action="store_true", default=False)
    g.add_argument("--use-opsm", action="store_true", default=False)
    g.add_argument("--opsm-delta", type=float, default=1e-4)
    g.add_argument("--calculate-per-token-loss", action="store_true", default=False)
    g.add_argument("--get-mismatch-metrics", action="store_true", default=False)


def add_lora_args(p):
    g = p.add_argument_group("lora")
    g.add_argument("--lora-rank", type=int, default=0)
    g.add_argument("--lora-alpha", type=int, default=16)
    g.add_argument("--lora-dropout", type=float, default=0.0)
    g.add_argument("--lora-type", default="lora", choices=["lora", "canonical_lora"])
    g.add_argument("--target-modules", nargs="+", default=None)
    g.add_argument("--exclude-modules", nargs="+", default=None)
    g.add_argument("--lora-adapter-path", default=None)
    g.add_argument("--lora-sync-from-tensor", action="store_true", default=False)


def add_router_args(p):
    g = p.add_argument_group("router")
    g.add_argument("--use-miles-router", action="store_true", default=False)
    g.add_argument("--miles-router-middleware-paths", nargs="+", default=None)
    g.add_argument("--miles-router-timeout", type=float, default=None)
    g.add_argument("--miles-router-max-connections", type=int, default=None)
    g.add_argument("--miles-router-health-check-failure-threshold", type=int, default=3)
    g.add_argument("--http-proxy", default=None)


def add_tracking_args(p):
    g = p.add_argument_group("tracking")
    g.add_argument("--use-wandb", action="store_true", default=False)
    g.add_argument("--wandb-mode", default=None)
    g.add_argument("--wandb-key", default=None)
    g.add_argument("--wandb-host", default=None)
    g.add_argument("--wandb-team", default=None)
    g.add_argument("--wandb-group", default=None)
    g.add_argument("--wandb-project", default=None)
    g.add_argument("--wandb-dir", default=None)
    g.add_argument("--wandb-run-id", default=None)
    g.add_argument("--disable-wandb-random-suffix", action="store_true", default=False)
    g.add_argument("--wandb-always-use-train-step", action="store_true", default=False)
    g.add_argument("--use-tensorboard", action="store_true", default=False)
    g.add_argument("--tb-project-name", default=None)
    g.add_argument("--tb-experiment-name", default=None)
    g.add_argument("--use-prometheus", action="store_true", default=False)
    g.add_argument("--prometheus-port", type=int, default=9090)
    g.add_argument("--prometheus-run-name", default=None)
    g.add_argument("--log-multi-turn", action="store_true", default=False)
    g.add_argument("--log-passrate", action="store_true", default=False)
    g.add_argument("--log-reward-category", default=None)
    g.add_argument("--log-correct-samples", action="store_true", default=False)


def add_debug_args(p):
    g = p.add_argument_group("debug")
    g.add_argument("--save-debug-rollout-data", default=None)
    g.add_argument("--load-debug-rollout-data", default=None)
    g.add_argument("--load-debug-rollout-data-subsample", type=float, default=None)
    g.add_argument("--save-debug-train-data", default=None)
    g.add_argument("--debug-rollout-only", action="store_true", default=False)
    g.add_argument("--debug-train-only", action="store_true", default=False)
    g.add_argument("--dump-details", default=None)
    g.add_argument("--check-weight-update-equal", action="store_true", default=False)
    g.add_argument("--use-pytorch-profiler", action="store_true", default=False)
    g.add_argument("--profile-target", nargs="+", default=["train_overall"],
                   choices=["train_overall", "train_actor", "train_log_probs"])
    g.add_argument("--profile-step-start", type=int, default=10)
    g.add_argument("--profile-step-end", type=int, default=12)
    g.add_argument("--tensorboard-dir", default=None)
    g.add_argument("--record-memory-history", action="store_true", default=False)
    g.add_argument("--memory-recorder", choices=["torch", "memray"], default="torch")
    g.add_argument("--memory-snapshot-dir", default=".")
    g.add_argument("--memory-snapshot-num-steps", type=int, default=None)
    g.add_argument("--dumper-enable", action="store_true", default=False)
    g.add_argument("--dumper-dir", default="/tmp/dumper")
    g.add_argument("--dumper-inference", action="store_true", default=False)
    g.add_argument("--dumper-fwd-only", action="store_true", default=False)
    g.add_argument("--dumper-fwd-bwd", action="store_true", default=False)
    g.add_argument("--dumper-source-patcher-config-train", default=None)
    g.add_argument("--dumper-source-patcher-config-inference", default=None)
    g.add_argument("--env-report", action="store_true", default=False)
    g.add_argument("--disable-weights-backuper", action="store_true", default=False)


def add_reward_args(p):
    g = p.add_argument_group("reward")
    g.add_argument("--rm-type", default=None)
    g.add_argument("--reward-key", default=None)
    g.add_argument("--group-rm", action="store_true", default=False)
    g.add_argument("--rm-url", default=None)
    g.add_argument("--custom-rm-path", default=None)
    g.add_argument("--custom-reward-post-process-path", default=None)
    g.add_argument("--custom-convert-samples-to-train-data-path", default=None)


def add_buffer_filter_args(p):
    g = p.add_argument_group("buffer / filters")
    g.add_argument("--buffer-filter-path", default=None)
    g.add_argument("--rollout-sample-filter-path", default=None)
    g.add_argument("--rollout-all-samples-process-path", default=None)
    g.add_argument("--rollout-data-postprocess-path", default=None)
    g.add_argument("--disable-rollout-trim-samples", action="store_true", default=False)
    g.add_argument("--custom-rollout-log-function-path", default=None)
    g.add_argument("--custom-eval-rollout-log-function-path", default=None)


def add_hook_args(p):
    g = p.add_argument_group("trainer hooks")
    g.add_argument("--custom-megatron-init-path", default=None)
    g.add_argument("--custom-megatron-before-log-prob-hook-path", default=None)
    g.add_argument("--custom-megatron-before-train-step-hook-path", default=None)


def add_misc_args(p):
    g = p.add_argument_group("mtp / pd / ci / session")
    g.add_argument("--enable-mtp-training", action="store_true", default=False)
    g.add_argument("--mtp-num-layers", type=int, default=None)
    g.add_argument("--mtp-loss-scaling-factor", type=float, default=0.2)
    g.add_argument("--prefill-num-servers", type=int, default=None)
    g.add_argument("--ci-test", action="store_true", default=False)
    g.add_argument("--ci-disable-kl-checker", action="store_true", default=False)
    g.add_argument("--ci-disable-logprobs-checker", action="store_true", default=False)
    g.add_argument("--ci-metric-checker-key", default=None)
    g.add_argument("--ci-metric-checker-threshold", type=float, default=None)
    g.add_argument("--ci-save-grad-norm", default=None)
    g.add_argument("--ci-load-grad-norm", default=None)
    g.add_argument("--ci-save-model-hash", default=None)
    g.add_argument("--ci-check-model-hash", default=None)
    g.add_argument("--use-session-server", action="store_true", default=False)
    g.add_argument("--session-server-ip", default="127.0.0.1")
    g.add_argument("--session-server-port", type=int, default=None)
    g.add_argument("--tito-model", default=None)
    g.add_argument("--tito-allowed-append-roles", nargs="+", default=["tool"])
    g.add_argument("--custom-config-path", default=None)
    g.add_argument("--sglang-config", default=None)
    g.add_argument("--sglang-server-concurrency", type=int, default=512)
    g.add_argument("--pin-rollout-manager-to-head", action="store_true", default=False)


ALL_GROUPS = [add_cluster_args, add_train_args, add_rollout_args, add_ft_args, add_data_args,
              add_eval_args, add_algo_args, add_lora_args, add_router_args, add_tracking_args,
              add_debug_args, add_reward_args, add_buffer_filter_args, add_hook_args, add_misc_args]


def build_parser(add_custom_arguments: Callable | None = None) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser("miles_b200", allow_abbrev=False)
    for fn in ALL_GROUPS:
        fn(p)
    if add_custom_arguments is not None:
        add_custom_arguments(p)
    return p


def _apply_yaml(args, path):
    with open(path) as f:
        cfg = yaml.safe_load(f) or {}
    for k, v in cfg.items():
        setattr(args, k.replace("-", "_"), v)


def _add_fn_arguments(parser, argv):
    """Let user rollout / generate functions contribute flags via `fn.add_arguments(parser)`
    (reference arguments.py:1626-1638)."""
    pre, _ = parser.parse_known_args(argv)
    for attr in ("rollout_function_path", "custom_generate_function_path", "eval_function_path"):
        path = getattr(pre, attr, None)
        if not path:
            continue
        try:
            fn = load_function(path)
        except Exception:
            continue
        add = getattr(fn, "add_arguments", None)
        if callable(add):
            add(parser)


def parse_args(argv: list[str] | None = None, add_custom_arguments: Callable | None = None):
    parser = build_parser(add_custom_arguments)
    _add_fn_arguments(parser, argv)
    args, unknown = parser.parse_known_args(argv)
    sglang = {}
    rest = []
    i = 0
    while i < len(unknown):
        tok = unknown[i]
        if tok.startswith("--sglang-"):
            key = tok[len("--sglang-"):].replace("-", "_")
            if "=" in key:
                key, val = key.split("=", 1)
            elif i + 1 < len(unknown) and not unknown[i + 1].startswith("--"):
                val = unknown[i + 1]
                i += 1
            else:
                val = True
            sglang[key] = val
        else:
            rest.append(tok)
        i += 1
    if rest:
        parser.error(f"unrecognized arguments: {' '.join(rest)}")
    args.sglang_args = sglang
    if args.custom_config_path:
        _apply_yaml(args, args.custom_config_path)
    validate_args(args)
    return args


def validate_args(args) -> None:
    """Cross-flag rules of the reference (miles_validate_args, arguments.py:1805-2096)."""
    reject_unsupported(args)
    if getattr(args, "dump_details", None):
        # --dump-details DIR: rollout and train data of every rollout under DIR
        d = args.dump_details
        if not args.save_debug_rollout_data:
            args.save_debug_rollout_data = os.path.join(d, "rollout_data", "{rollout_id}.pkl")
        if not getattr(args, "save_debug_train_data", None):
            args.save_debug_train_data = os.path.join(d, "train_data", "{rollout_id}_{rank}.pkl")
    if args.hf_checkpoint is None and getattr(args, "hf_checkpoint_alias", None):
        args.hf_checkpoint = args.hf_checkpoint_alias
    if args.eps_clip_high is None:
        args.eps_clip_high = args.eps_clip
    if args.kl_coef != 0 and args.use_kl_loss and args.kl_loss_coef != 0:
        raise ValueError("kl_coef and kl_loss_coef are mutually exclusive")
    args.use_critic = args.advantage_estimator == "ppo"
    if args.critic_num_nodes is None:
        args.critic_num_nodes = args.actor_num_nodes
    if args.critic_num_gpus_per_node is None:
        args.critic_num_gpus_per_node = args.actor_num_gpus_per_node
    if args.critic_lr is None:
        args.critic_lr = args.lr
    if args.offload:
        args.offload_train = True if args.offload_train is None else args.offload_train
        args.offload_rollout = True if args.offload_rollout is None else args.offload_rollout
    if args.colocate:
        if args.offload_train is None:
            args.offload_train = True
        if args.offload_rollout is None:
            args.offload_rollout = True
        if args.rollout_num_gpus != args.actor_num_gpus_per_node * args.actor_num_nodes:
            args.rollout_num_gpus = args.actor_num_gpus_per_node * args.actor_num_nodes
        if args.update_weight_transfer_mode == "p2p":
            raise ValueError("--update-weight-transfer-mode p2p cannot be used with --colocate")
    args.offload_train = bool(args.offload_train)
    args.offload_rollout = bool(args.offload_rollout)
    if args.rollout_num_gpus is None:
        args.rollout_num_gpus = args.actor_num_gpus_per_node * args.actor_num_nodes
    if args.over_sampling_batch_size is None:
        args.over_sampling_batch_size = args.rollout_batch_size
    if (args.rollout_batch_size is not None and args.over_sampling_batch_size is not None
            and args.over_sampling_batch_size < args.rollout_batch_size):
        raise ValueError("over_sampling_batch_size must be >= rollout_batch_size")
    if args.use_rollout_routing_replay:
        args.use_routing_replay = True
    if args.num_steps_per_rollout is not None and args.rollout_batch_size is not None:
        args.global_batch_size = (args.rollout_batch_size * args.n_samples_per_prompt
                                  // args.num_steps_per_rollout)
    if args.global_batch_size is None and args.rollout_batch_size is not None:
        args.global_batch_size = args.rollout_batch_size * args.n_samples_per_prompt
    if args.eval_temperature is None:
        args.eval_temperature = args.rollout_temperature
    if args.eval_config:
        args.eval_datasets = load_eval_config(args.eval_config)
    if args.eval_top_p is None:
        args.eval_top_p = args.rollout_top_p
    if args.eval_top_k is None:
        args.eval_top_k = args.rollout_top_k
    if args.eval_max_response_len is None:
        args.eval_max_response_len = args.rollout_max_response_len
    if args.log_probs_max_tokens_per_gpu is None:
        args.log_probs_max_tokens_per_gpu = args.max_tokens_per_gpu
    if args.debug_rollout_only and args.debug_train_only:
        raise ValueError("debug_rollout_only and debug_train_only are exclusive")
    if args.load_debug_rollout_data is not None:
        args.debug_train_only = True
    if args.true_on_policy_mode:
        # rollout and training log-probs are bitwise identical by construction here
        args.use_rollout_logprobs = getattr(args, "use_rollout_logprobs", False)
    if args.num_rollout is None and args.num_epoch is None:
        args.num_rollout = 1
    world = args.actor_num_nodes * args.actor_num_gpus_per_node
    mp = (args.tensor_model_parallel_size * args.pipeline_model_parallel_size
          * args.context_parallel_size)
    if world % mp != 0:
        raise ValueError(f"world size {world} not divisible by TP*PP*CP = {mp}")
    args.data_parallel_size = world // mp
    args.world_size = world
    if args.pipeline_model_parallel_size == 1 and (
            args.decoder_first_pipeline_num_layers is not None
            or args.decoder_last_pipeline_num_layers is not None
            or (args.virtual_pipeline_model_parallel_size or 1) > 1):
        raise ValueError("--decoder-first/last-pipeline-num-layers and "
                         "--virtual-pipeline-model-parallel-size need --pipeline-model-parallel-size > 1")


def load_eval_config(path: str) -> list[dict]:
    """--eval-config YAML: an `eval` mapping (or the root) with optional `defaults` and
    `datasets` (a list of entries with `name`, or a mapping keyed by name). Each dataset entry
    (path, n_samples_per_eval_prompt, temperature, top_p, top_k, max_response_len, input_key,
    label_key, tool_key, rm_type, stop_token_ids, min_new_tokens) falls back to `defaults`,
    then to the eval flags (reference miles/utils/eval_config.py)."""
    with open(path) as f:
        cfg = yaml.safe_load(f) or {}
    if not isinstance(cfg, dict):
        raise ValueError("--eval-config must contain a mapping at the root")
    ev = cfg.get("eval", cfg)
    defaults = dict(ev.get("defaults") or {})
    ds = ev.get("datasets")
    if isinstance(ds, dict):
        ds = [dict(v or {}, name=v.get("name", k) if isinstance(v, dict) else k) for k, v in ds.items()]
    if not ds:
        raise ValueError("--eval-config defines no datasets under `eval.datasets`")
    out = []
    for d in ds:
        if "name" not in d or "path" not in {**defaults, **d}:
            raise ValueError("each eval dataset needs a `name` and a `path`")
        out.append({**defaults, **d})
    return out


# ------------------------------------------------------------------------------------------------
# Flags of the reference that need no action here, and flags whose non-default values are not
# supported. Every other flag is read by the code it configures (tests/test_flag_registry_cpu.py
# checks that each flag is in exactly one of the three groups).
# ------------------------------------------------------------------------------------------------
NO_EFFECT = {
    "num_gpus_per_node": "torchrun starts one process per GPU; the node size comes from it",
    "distributed_backend": "NCCL on GPUs and gloo on CPU are chosen per device",
    "pin_rollout_manager_to_head": "no Ray placement: the rollout manager runs in every rank",
    "miles_router_max_connections": "the router keeps one HTTP session with no connection cap",
    "use_miles_router": "router/router.py is the only router",
    "megatron_to_hf_mode": "one converter (checkpoint/hf.py) serves both modes",
    "qkv_format": "training always packs sequences (thd); bshd is rejected below",
    "seq_length": "packed variable-length batches have no fixed sequence length",
    "padded_vocab_size": "the vocabulary is not padded",
    "data_pad_size_multiplier": "packed (thd) micro-batches carry no padding",
    "allgather_cp": "the DSA indexer inputs are always all-gathered over context parallelism",
    "recompute_loss_function": "LM-head logits are never stored: the backward always recomputes them",
    "p2p_transfer_num_workers": "peer-memory refit runs as device kernels, without a worker pool",
    "p2p_transfer_timeout": "peer-memory refit waits are bounded inside the kernels",
    "use_distributed_post": "requests go to the in-process engine, not over HTTP",
    "lora_sync_from_tensor": "the colocated engine reads the adapters in place",
    "low_memory_resume": "resume loads straight into the flat parameter buffers",
    "loss_mask_type": "multi-turn loss masks come from the chat-template rendering (any family)",
    "pause_generation_mode": "the engine server takes the mode per /pause_generation request",
}

UNSUPPORTED = {  # flag -> default; a different value is rejected at parse time
    "rollout_external": False,
    "rollout_external_engine_addrs": None,
    "rollout_buffer_url": None,
    "fetch_trajectory_retry_times": -1,
    "rollout_task_type": None,
    "min_batch_collection_ratio": 1.0,
    "use_dynamic_global_batch_size": False,
    "use_rollout_entropy": False,
    "lora_type": "lora",
    "dumper_source_patcher_config_train": None,
    "dumper_source_patcher_config_inference": None,
    "memory_recorder": "torch",
}


def reject_unsupported(args) -> None:
    bad = [f"--{k.replace('_', '-')}" for k, d in UNSUPPORTED.items() if getattr(args, k, d) != d]
    if getattr(args, "qkv_format", "thd") != "thd":
        bad.append("--qkv-format bshd")
    if bad:
        raise ValueError(f"not supported by this framework: {', '.join(bad)}")


def reset_arg(parser: argparse.ArgumentParser, name: str, **kwargs) -> None:
    """Change the default / choices of an existing flag (reference arguments.py:22)."""
    for a in parser._actions:
        if name in a.option_strings:
            for k, v in kwargs.items():
                setattr(a, k, v)
            return
    parser.add_argument(name, **kwargs)
