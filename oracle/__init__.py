"""CPU oracle for the Transformer forward -- TEST INFRASTRUCTURE ONLY.

This package restates the reference's forward semantics
(official/torch_transformer_benchmark.py, Wendystar0628/ML-Guided-Program-
Search-for-Shape-Specialized-Transformer-Optimization) in numpy float32, and
reproduces the reference module's seeded default weight initialisation.  It
is the checker for the sm_100a path: only tests/, ``__graft_entry__.smoke()``
and bench.py's CPU-baseline / reference arm may import it.  The product path
(the ``solution`` package and libb200tx) never imports or calls anything here.

Pinning: tests/golden/ holds outputs of the reference itself (its official
``BaselineTransformer`` and its ``solution`` portable program, run on CPU from
the reference sources by tests/golden/make_golden.py); tests/test_oracle.py
checks this restatement against them.
"""

from .reference_forward import (
    attention_core,
    attention_reference,
    attention_rows,
    ffn_reference,
    gelu_erf,
    layer_norm,
    transformer_forward,
    transformer_forward_tail,
)
from .weights import OfficialConfig, official_input, official_state_dict

__all__ = [
    "OfficialConfig",
    "attention_core",
    "attention_reference",
    "attention_rows",
    "ffn_reference",
    "gelu_erf",
    "layer_norm",
    "official_input",
    "official_state_dict",
    "transformer_forward",
    "transformer_forward_tail",
]
