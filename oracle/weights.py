"""Seeded official weights and inputs -- TEST INFRASTRUCTURE ONLY.

The reference's weights are whatever ``BaselineTransformer(cfg)`` draws from
torch's global RNG right after ``torch.manual_seed(seed)``
(official/torch_transformer_benchmark.py:148-160, default nn.Linear /
nn.LayerNorm init).  Reproducing them needs the same draws in the same order:
per layer norm1 (no draw), q_proj, k_proj, v_proj, out_proj (weight then bias
each, :70-73), norm2, ffn_in, ffn_out (:129-132), then final_norm.  This module
constructs plain ``nn.Linear`` layers in exactly that order, so every tensor
is bit-identical to the reference's; tests/golden/ pins that with checksums of
the reference's own state dict.

Inputs follow ``generate_random_case`` at padding 0 (official :234-259): a
CPU ``torch.Generator`` seeded with ``seed`` draws ``randn(B, S, D)``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import nn


@dataclass(frozen=True)
class OfficialConfig:
    """Same fields as official TransformerConfig (official :28-37)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool = True


def official_state_dict(config: OfficialConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """The reference BaselineTransformer's state dict after ``torch.manual_seed(seed)``."""

    d, f = config.d_model, config.ffn_dim
    state: dict[str, torch.Tensor] = {}
    cpu_rng_state = torch.get_rng_state()
    try:
        torch.manual_seed(seed)
        for i in range(config.num_layers):
            p = f"layers.{i}"
            norm1 = nn.LayerNorm(d)
            q, k, v, o = (nn.Linear(d, d) for _ in range(4))
            norm2 = nn.LayerNorm(d)
            ffn_in = nn.Linear(d, f)
            ffn_out = nn.Linear(f, d)
            for name, module in (
                ("norm1", norm1),
                ("attention.q_proj", q),
                ("attention.k_proj", k),
                ("attention.v_proj", v),
                ("attention.out_proj", o),
                ("norm2", norm2),
                ("ffn_in", ffn_in),
                ("ffn_out", ffn_out),
            ):
                state[f"{p}.{name}.weight"] = module.weight.detach().clone()
                state[f"{p}.{name}.bias"] = module.bias.detach().clone()
        final = nn.LayerNorm(d)
        state["final_norm.weight"] = final.weight.detach().clone()
        state["final_norm.bias"] = final.bias.detach().clone()
    finally:
        torch.set_rng_state(cpu_rng_state)
    return state


def official_input(config: OfficialConfig, seed: int, batch_rows: slice | None = None) -> torch.Tensor:
    """``torch.randn(B, S, D)`` from a CPU generator seeded with ``seed`` (fp32)."""

    generator = torch.Generator(device="cpu")
    generator.manual_seed(seed)
    x = torch.randn(
        config.batch_size, config.seq_len, config.d_model, generator=generator, dtype=torch.float32
    )
    return x if batch_rows is None else x[batch_rows].contiguous()


def per_row_input(config: OfficialConfig, base_seed: int, row: int) -> torch.Tensor:
    """One batch row drawn from its own seed ``base_seed + row`` ([1, S, D] fp32).

    The streamed capacity shape generates its input row by row this way.
    """

    generator = torch.Generator(device="cpu")
    generator.manual_seed(base_seed + row)
    return torch.randn(1, config.seq_len, config.d_model, generator=generator, dtype=torch.float32)


def state_to_numpy(state: dict[str, torch.Tensor]) -> dict[str, np.ndarray]:
    return {key: value.detach().cpu().float().numpy() for key, value in state.items()}


def state_checksum(state: dict[str, torch.Tensor]) -> float:
    """Order-independent float64 checksum used to pin the weights to the reference."""

    return float(sum(value.double().sum().item() * (1 + (i % 7)) for i, (_, value) in enumerate(sorted(state.items()))))


__all__ = [
    "OfficialConfig",
    "official_input",
    "official_state_dict",
    "per_row_input",
    "state_checksum",
    "state_to_numpy",
]
