"""Per-rank checkpoint loading on the CPU: a small Qwen2 checkpoint written
as safetensors files (several shard files, like the hub's) is read slice by
slice; every rank's dict equals the reference split of the whole checkpoint
(``src/tinybatch/tensor_parallel.py:35-61``) cast to bf16."""
from __future__ import annotations

import json

import pytest
import torch

from tinybatch_b200.checkpoint import load_config, load_rank_weights
from tinybatch_b200.config import named_config
from tinybatch_b200.tensor_parallel import shard_weights
from tinybatch_b200.weights import synthetic_weights


def _write_checkpoint(path, cfg, w):
    from safetensors.torch import save_file
    names = sorted(k for k in w if not (cfg.tie_embeddings and k == "lm_head.weight"))
    half = len(names) // 2
    for i, part in enumerate((names[:half], names[half:])):
        save_file({k: w[k].contiguous() for k in part},
                  str(path / f"model-{i + 1:05d}-of-00002.safetensors"))
    hf = {"hidden_size": cfg.d_model, "num_attention_heads": cfg.n_heads,
          "num_key_value_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
          "num_hidden_layers": cfg.n_layers, "intermediate_size": cfg.d_ff,
          "vocab_size": cfg.vocab_size, "rms_norm_eps": cfg.rms_eps,
          "rope_theta": cfg.rope_theta, "tie_word_embeddings": cfg.tie_embeddings,
          "max_position_embeddings": cfg.max_position}
    (path / "config.json").write_text(json.dumps(hf))


@pytest.mark.parametrize("tie", [False, True])
def test_rank_slices_equal_reference_split(tmp_path, tie):
    cfg = named_config("tiny", tie_embeddings=tie, n_heads=4, n_kv_heads=2)
    w = synthetic_weights(cfg, 5)
    _write_checkpoint(tmp_path, cfg, w)
    got_cfg = load_config(str(tmp_path))
    assert got_cfg == cfg
    for world in (1, 2):
        for rank in range(world):
            got = load_rank_weights(str(tmp_path), cfg, rank, world)
            want = shard_weights(w, cfg, rank, world)
            assert set(got) == set(want)
            for k, v in want.items():
                assert got[k].dtype == torch.bfloat16
                assert torch.equal(got[k], v.to(torch.bfloat16)), k
            if tie:
                assert got["lm_head.weight"] is got["model.embed_tokens.weight"]


def test_indivisible_degree_is_refused(tmp_path):
    cfg = named_config("tiny")
    _write_checkpoint(tmp_path, cfg, synthetic_weights(cfg, 5))
    with pytest.raises(AssertionError):
        load_rank_weights(str(tmp_path), cfg, 0, 4)      # 2 kv heads over 4 ranks


@pytest.mark.parametrize("tie", [False, True])
def test_rank_draw_equals_sharded_full_draw(tie):
    """synthetic_rank_weights draws the same values as the full draw, keeping
    only each rank's slices."""
    from tinybatch_b200.weights import synthetic_rank_weights
    cfg = named_config("tiny", tie_embeddings=tie)
    full = synthetic_weights(cfg, 4, dtype=torch.bfloat16)
    for world in (1, 2):
        for rank in range(world):
            got = synthetic_rank_weights(cfg, 4, rank, world)
            want = shard_weights(full, cfg, rank, world)
            assert set(got) == set(want)
            for k in want:
                assert torch.equal(got[k], want[k]), k
