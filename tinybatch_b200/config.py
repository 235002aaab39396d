"""Model and engine configuration.

``ModelConfig`` has the fields of the reference's ``ModelConfig``
(``src/tinybatch/model.py:32-62``) and ``EngineConfig`` the knobs of
``src/tinybatch/config.py:7-35``, so code written against the reference keeps
working.  ``NAMED_CONFIGS`` holds the synthetic Qwen2 shapes the benchmarks
and parity tests use.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass
class ModelConfig:
    n_layers: int
    n_heads: int
    n_kv_heads: int
    d_model: int
    head_dim: int
    d_ff: int
    vocab_size: int
    rms_eps: float
    rope_theta: float
    tie_embeddings: bool
    max_position: int

    @staticmethod
    def from_hf(cfg: dict) -> "ModelConfig":
        """Build from a HuggingFace ``config.json`` dict (same keys and
        defaults as ``src/tinybatch/model.py:46-62``)."""
        d_model = cfg["hidden_size"]
        n_heads = cfg["num_attention_heads"]
        return ModelConfig(
            n_layers=cfg["num_hidden_layers"],
            n_heads=n_heads,
            n_kv_heads=cfg["num_key_value_heads"],
            d_model=d_model,
            head_dim=cfg.get("head_dim", d_model // n_heads),
            d_ff=cfg["intermediate_size"],
            vocab_size=cfg["vocab_size"],
            rms_eps=cfg["rms_norm_eps"],
            rope_theta=cfg["rope_theta"],
            tie_embeddings=cfg.get("tie_word_embeddings", False),
            max_position=cfg["max_position_embeddings"],
        )


def _qwen2(n_layers, d, h, kv, hd, ff, vocab, theta, tie, max_pos=32768):
    return ModelConfig(n_layers=n_layers, n_heads=h, n_kv_heads=kv, d_model=d, head_dim=hd,
                       d_ff=ff, vocab_size=vocab, rms_eps=1e-6, rope_theta=theta,
                       tie_embeddings=tie, max_position=max_pos)


# Synthetic shapes (random-init weights; no checkpoint is ever loaded).
NAMED_CONFIGS: dict[str, ModelConfig] = {
    # the reference's own TP test model (tests/test_tensor_parallel.py:14-18)
    "ref-test": _qwen2(4, 64, 4, 2, 16, 128, 97, 1e4, False, 512),
    # tiny synthetic Qwen2: 2 layers, d 64, 4q/2kv, hd 16, ff 128, vocab 256
    "tiny": _qwen2(2, 64, 4, 2, 16, 128, 256, 1e4, False, 4096),
    "qwen2.5-0.5b": _qwen2(24, 896, 14, 2, 64, 4864, 151936, 1e6, True),
    "qwen2.5-14b": _qwen2(48, 5120, 40, 8, 128, 13824, 152064, 1e6, False),
    "qwen2.5-72b": _qwen2(80, 8192, 64, 8, 128, 29568, 152064, 1e6, False),
}


def named_config(name: str, **overrides) -> ModelConfig:
    return replace(NAMED_CONFIGS[name], **overrides)


@dataclass
class EngineConfig:
    """Memory-layout and scheduling knobs (``src/tinybatch/config.py:7-35``).

    ``device``/``dtype`` default to the B200 path: ``cuda`` and ``bfloat16``.
    ``tp`` is the tensor-parallel degree of the model the engine drives."""

    model_id: str = "Qwen/Qwen2.5-0.5B-Instruct"
    device: str = "cuda"
    dtype: str = "bfloat16"

    # paged KV cache
    block_size: int = 16
    num_blocks: int = 512
    enable_prefix_caching: bool = True

    # scheduler
    max_batch_tokens: int = 2048
    max_running: int = 32
    max_model_len: int = 4096

    # sampling defaults
    max_new_tokens: int = 256
    temperature: float = 0.0
    top_p: float = 1.0
    stop_token_ids: tuple = field(default_factory=tuple)

    # engine: in a steady greedy decode batch (prefix caching off), queue step
    # k+1 on the device before reading step k's tokens back
    # (``LLMEngine.step``); tokens and block tables are those of the plain loop
    overlap_steps: bool = False

    def kv_pool_tokens(self) -> int:
        return self.block_size * self.num_blocks
