"""Seeded synthetic workloads: the BASELINE configs and the reference's official shapes.

What the benchmarks feed the model.  There is no dataset: the reference's
official harness draws its weights from ``torch.manual_seed(seed)`` through
the default ``nn.Linear`` / ``nn.LayerNorm`` init of ``BaselineTransformer``
(official/torch_transformer_benchmark.py:59-172) and its inputs from a seeded
CPU generator (``generate_random_case`` at padding 0, :234-259).  This module
makes the same draws in the same order, so a state dict built here loads into
``UserOptimizedTransformer`` exactly as the reference's baseline state dict
does (``copy_model_weights`` packs q/k/v).  The test suite checks these
tensors bit for bit against the checker's independent generator, which is
itself pinned to checksums of the reference's own state dict.

Construction order per layer (official :70-73, :129-132, :148-160): norm1,
q_proj, k_proj, v_proj, out_proj, norm2, ffn_in, ffn_out; then final_norm.
LayerNorms draw nothing; each Linear draws its weight, then its bias.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import torch
from torch import nn


@dataclass(frozen=True)
class WorkloadConfig:
    """The official ``TransformerConfig`` fields (official :28-37)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool = True

    def as_dict(self) -> dict:
        return asdict(self)

    @property
    def tokens(self) -> int:
        return self.batch_size * self.seq_len


def seeded_state_dict(config: WorkloadConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """The baseline module's fp32 state dict after ``torch.manual_seed(seed)``.

    The global CPU RNG state is restored afterwards.
    """

    d, f = config.d_model, config.ffn_dim
    saved = torch.get_rng_state()
    state: dict[str, torch.Tensor] = {}

    def take(prefix: str, module: nn.Module) -> None:
        state[f"{prefix}.weight"] = module.weight.detach().clone()
        state[f"{prefix}.bias"] = module.bias.detach().clone()

    try:
        torch.manual_seed(seed)
        for layer in range(config.num_layers):
            base = f"layers.{layer}"
            take(f"{base}.norm1", nn.LayerNorm(d))
            for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
                take(f"{base}.attention.{name}", nn.Linear(d, d))
            take(f"{base}.norm2", nn.LayerNorm(d))
            take(f"{base}.ffn_in", nn.Linear(d, f))
            take(f"{base}.ffn_out", nn.Linear(f, d))
        take("final_norm", nn.LayerNorm(d))
    finally:
        torch.set_rng_state(saved)
    return state


def seeded_input(config: WorkloadConfig, seed: int) -> torch.Tensor:
    """``randn(B, S, D)`` fp32 from a CPU generator seeded with ``seed``."""

    generator = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(config.batch_size, config.seq_len, config.d_model, generator=generator)


def seeded_row(config: WorkloadConfig, base_seed: int, row: int) -> torch.Tensor:
    """One ``[1, S, D]`` batch row drawn from its own seed ``base_seed + row``
    (the capacity shape's per-row inputs)."""

    generator = torch.Generator(device="cpu").manual_seed(base_seed + row)
    return torch.randn(1, config.seq_len, config.d_model, generator=generator)


# The reference's official benchmark shapes (official/test_shapes.json:
# case_id -> batch_size, seq_len, qkv_dim, heads, ffn_dim, layers; all causal).
OFFICIAL_SHAPES: dict[str, WorkloadConfig] = {
    "official_01": WorkloadConfig(64, 128, 128, 4, 128, 4),
    "official_02": WorkloadConfig(1, 128, 128, 4, 128, 4),
    "official_03": WorkloadConfig(4, 128, 128, 4, 128, 4),
    "official_04": WorkloadConfig(16, 128, 128, 4, 128, 4),
    "official_05": WorkloadConfig(128, 128, 128, 4, 128, 4),
    "official_06": WorkloadConfig(10000, 128, 128, 4, 128, 4),
    "official_07": WorkloadConfig(64, 128, 32, 4, 32, 4),
    "official_08": WorkloadConfig(64, 128, 1024, 4, 1024, 4),
    "official_09": WorkloadConfig(64, 128, 128, 1, 128, 4),
    "official_10": WorkloadConfig(64, 128, 128, 2, 128, 4),
    "official_11": WorkloadConfig(64, 128, 128, 16, 128, 4),
    "official_12": WorkloadConfig(64, 32, 128, 4, 128, 4),
    "official_13": WorkloadConfig(64, 1024, 128, 4, 128, 4),
    "official_14": WorkloadConfig(32, 100000, 1024, 16, 1024, 2),
}

# The reference's published medians on its own platform (one RTX 4080, fp32
# I/O with fp16 internals; result/20260831T083857.848038Z/final_performance.md:
# 18-30, 36): (its deployed program, the official PyTorch baseline), in ms.
# official_14's baseline was not run (a dense S x S score tensor does not fit).
REFERENCE_PUBLISHED_MS: dict[str, tuple[float, float | None]] = {
    "official_01": (0.218, 1.727),
    "official_02": (0.072, 1.871),
    "official_03": (0.082, 1.866),
    "official_04": (0.097, 1.910),
    "official_05": (0.421, 3.905),
    "official_06": (36.818, 491.954),
    "official_07": (0.074, 1.793),
    "official_08": (6.281, 21.434),
    "official_09": (0.202, 1.513),
    "official_10": (0.198, 1.685),
    "official_11": (0.243, 7.942),
    "official_12": (0.101, 1.756),
    "official_13": (3.337, 120.430),
    "official_14": (17244.0, None),
}


__all__ = [
    "OFFICIAL_SHAPES",
    "REFERENCE_PUBLISHED_MS",
    "WorkloadConfig",
    "seeded_input",
    "seeded_row",
    "seeded_state_dict",
]
