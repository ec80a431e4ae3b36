"""Lazy public solution contract (reference: solution/__init__.py:7-22).

``from solution import UserOptimizedTransformer, copy_model_weights`` loads
the model only when requested, like the reference, so importing the
configuration or planning modules never touches CUDA.
"""

from __future__ import annotations

from typing import Any

__all__ = ["UserOptimizedTransformer", "copy_model_weights"]


def __getattr__(name: str) -> Any:
    if name not in __all__:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    from .transformer import UserOptimizedTransformer, copy_model_weights

    exports = {
        "UserOptimizedTransformer": UserOptimizedTransformer,
        "copy_model_weights": copy_model_weights,
    }
    globals().update(exports)
    return exports[name]
