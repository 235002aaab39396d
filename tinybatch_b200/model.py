"""Qwen2 forward over the paged KV cache, on the B200 kernels.

``Qwen2Paged`` keeps the reference's constructor and ``forward`` signature
(``src/tinybatch/model.py:83-158``) and adds ``from_weights`` for
random-init or already-loaded weight dicts (the reference constructor
downloads from the HuggingFace hub).  ``forward`` returns the fp32 logits of
the last token of every sequence, ``[n_seqs, vocab]``, on the model's device.

There is no CPU path: the model lives on a CUDA device and every op runs in
``libtinybatch_b200.so``.
"""
from __future__ import annotations

import torch

from . import _native
from .config import ModelConfig
from .kv_cache import PagedKVCache
from .runtime import DeviceModel, RankWeights, StepMeta


def _to_list(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().tolist()
    return list(x)


class Qwen2Paged:
    """Weights + forward.  Inference only."""

    def __init__(self, model_id: str, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, rank: int = 0, world: int = 1,
                 comm=None, **kw):
        """Load a HF Qwen2 checkpoint (config.json + *.safetensors) from a
        local directory or the hub cache, as the reference does
        (``src/tinybatch/model.py:86-98``).  With ``world`` > 1 this process
        is tensor-parallel rank ``rank``: it reads only its own slices of the
        checkpoint (``checkpoint.load_rank_weights``)."""
        from .checkpoint import load_config, load_rank_weights, resolve
        path = resolve(model_id)
        cfg = load_config(path)
        w = load_rank_weights(path, cfg, rank, world, device, dtype)
        self._setup(cfg, w, device, dtype, rank=rank, world=world, comm=comm, sharded=True, **kw)

    @classmethod
    def from_weights(cls, cfg: ModelConfig, w: dict, device: torch.device | str = "cuda",
                     dtype: torch.dtype = torch.bfloat16, rank: int = 0, world: int = 1,
                     comm=None, sharded: bool = False, **kw) -> "Qwen2Paged":
        self = cls.__new__(cls)
        self._setup(cfg, w, device, dtype, rank, world, comm, sharded=sharded, **kw)
        return self

    def _setup(self, cfg, w, device, dtype, rank, world, comm, sharded=False, **kw):
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("Qwen2Paged runs on the B200 kernels only: device must be cuda")
        if dtype != torch.bfloat16:
            raise ValueError("the kernels compute in bf16 (fp32 accumulation); dtype must be bfloat16")
        _native.load()
        self.cfg, self.device, self.dtype = cfg, device, dtype
        self.rank, self.world = rank, world
        self.weights = RankWeights(cfg, w, rank, world, device, sharded=sharded)
        self.dm = DeviceModel(self.weights, comm=comm, **kw)

    def make_kv_cache(self, num_blocks: int, block_size: int = 16) -> PagedKVCache:
        """A pool sized for this rank's kv heads."""
        return PagedKVCache(self.cfg.n_layers, num_blocks, block_size, self.weights.n_kv,
                            self.cfg.head_dim, self.device, torch.bfloat16)

    def metadata(self, token_ids, positions, seq_slices, block_tables, context_lens,
                 block_size: int) -> StepMeta:
        return StepMeta(_to_list(token_ids), _to_list(positions), list(seq_slices),
                        [list(t) for t in block_tables], _to_list(context_lens), block_size,
                        self.cfg.n_heads // self.cfg.n_kv_heads, self.device)

    @torch.inference_mode()
    def forward(self, token_ids, positions, seq_slices, block_tables, context_lens,
                kv_cache: PagedKVCache) -> torch.Tensor:
        """Logits of the LAST token of each sequence: ``[n_seqs, vocab]`` fp32."""
        md = self.metadata(token_ids, positions, seq_slices, block_tables, context_lens,
                           kv_cache.block_size)
        return self.dm.forward(md, kv_cache.pools).clone()

    @torch.inference_mode()
    def forward_meta(self, md: StepMeta, kv_cache: PagedKVCache, sample: bool = False):
        """Forward over prebuilt metadata; logits stay in the model's buffer
        (valid until the next call)."""
        return self.dm.forward(md, kv_cache.pools, sample=sample)
