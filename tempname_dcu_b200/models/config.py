"""GPT configuration, validation and parameter accounting (no torch import).

Reference parity: ``python/flux_dcu/model.py:13-59`` (DEFAULT_CONFIG,
validate_config, parameter_counts).  Additions for B200 workloads:

* ``pad_vocab`` -- pad a vocabulary that does not divide the tensor-parallel
  group (GPT-6.7B with vocab 50257) to a multiple of ``vocab_pad_multiple``
  (64: every shard stays a multiple of 8 columns for the GEMM/CE kernels at
  TP <= 8).  Padded logits are masked out of the softmax.
* world_size 1 is allowed (no tensor parallelism).
"""
from __future__ import annotations

import math

DEFAULT_CONFIG = dict(layers=32, hidden=4096, ffn=16384, heads=32, sequence=2048, micro_batch=1,
                      accumulation_steps=4, vocab=33792, chunk_rows=128)
# GPT-6.7B as quoted by the benchmark: vocab 50257 (padded), 8 micro-batches.
BENCH_CONFIG = dict(DEFAULT_CONFIG, vocab=50257, accumulation_steps=8, pad_vocab=True)
SMALL_CONFIG = dict(layers=2, hidden=256, ffn=1024, heads=2, sequence=256, micro_batch=1, accumulation_steps=1,
                    vocab=1024, chunk_rows=128)

HEAD_DIM = 128
_INT_KEYS = tuple(DEFAULT_CONFIG)
_FLOAT_DEFAULTS = (("learning_rate", 1e-4), ("weight_decay", 0.01), ("max_grad_norm", 1.0),
                   ("layer_norm_epsilon", 1e-5))


def padded_vocab(config, world_size=1) -> int:
    vocab = config["vocab"]
    if not config.get("pad_vocab"):
        return vocab
    multiple = int(config.get("vocab_pad_multiple", 64))
    multiple = multiple * world_size // math.gcd(multiple, world_size)
    return -(-vocab // multiple) * multiple


def validate_config(config, world_size=8):
    """Merged, validated configuration; raises ValueError on any partition
    that does not divide the tensor-parallel group."""
    if not isinstance(config, dict):
        raise ValueError("model config must be a dictionary")
    c = dict(DEFAULT_CONFIG)
    c.update(config)
    for key in _INT_KEYS:
        if type(c[key]) is not int or c[key] <= 0:
            raise ValueError(f"{key} must be a positive integer")
    if type(world_size) is not int or world_size < 1:
        raise ValueError("world_size must be a positive integer")
    if type(c.get("pad_vocab", False)) is not bool:
        raise ValueError("pad_vocab must be a bool")
    c["padded_vocab"] = padded_vocab(c, world_size)
    for key in ("hidden", "ffn", "heads"):
        if c[key] % world_size:
            raise ValueError(f"{key} must be divisible by the tensor-parallel size")
    if c["padded_vocab"] % world_size:
        raise ValueError("vocab must be divisible by the tensor-parallel size (or set pad_vocab)")
    if c["hidden"] % c["heads"]:
        raise ValueError("hidden must be divisible by heads")
    rows = c["sequence"] * c["micro_batch"]
    if rows % world_size or (rows // world_size) % c["chunk_rows"]:
        raise ValueError("sequence rows per rank must be divisible by chunk_rows")
    for key, default in _FLOAT_DEFAULTS:
        value = c.get(key, default)
        if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
            raise ValueError(f"{key} must be finite")
        if value < 0 or (key != "weight_decay" and value == 0):
            raise ValueError(f"invalid {key}")
        c[key] = float(value)
    return c


MAX_MICRO_BATCH_TOKENS = 16384  # one-CTA stable token sort of the embedding gradient (tdb_sort_tokens)


def native_shape_ok(c, world_size) -> bool:
    """True when the sm_100a kernels support this configuration (head_dim 128,
    hidden and shard widths multiples of 8, at most 16384 tokens per
    micro-batch)."""
    return (c["hidden"] // c["heads"] == HEAD_DIM and c["hidden"] % 8 == 0 and
            (c["padded_vocab"] // world_size) % 8 == 0 and (c["ffn"] // world_size) % 8 == 0 and
            c["sequence"] * c["micro_batch"] <= MAX_MICRO_BATCH_TOKENS)


def parameter_counts(config, world_size=8):
    """Logical / replicated / sharded parameter counts (tied embedding head;
    QKV and FC1 biases sharded; LayerNorms, row biases and positions
    replicated)."""
    c = validate_config(config, world_size)
    h, f, v, s, layers = c["hidden"], c["ffn"], c["padded_vocab"], c["sequence"], c["layers"]
    logical = v * h + s * h + layers * (4 * h * h + 2 * h * f + 9 * h + f) + 2 * h
    replicated = s * h + layers * 6 * h + 2 * h
    sharded = logical - replicated
    return dict(logical_parameters=logical, replicated_parameters=replicated, sharded_parameters=sharded,
                parameters_per_rank=sharded // world_size + replicated, tied_embedding_head=True)


def train_flops_per_step(config, world_size=1) -> float:
    """Model FLOPs of one optimizer step (forward + backward, all ranks):
    6 * tokens * (matmul parameters) + causal attention (12 * L * s * h per
    token, halved for causality)."""
    c = validate_config(config, world_size)
    h, f, v, s, layers = c["hidden"], c["ffn"], c["padded_vocab"], c["sequence"], c["layers"]
    tokens = s * c["micro_batch"] * c["accumulation_steps"]
    matmul = layers * (4 * h * h + 2 * h * f) + v * h
    attention = layers * 2 * 2 * s * h / 2  # QK^T and PV per token, causal half
    return 6.0 * tokens * matmul + 3.0 * tokens * attention
