"""Shared argument checks for the libb200tx wrappers."""

from __future__ import annotations

import torch

from .. import _native


def library_ready() -> bool:
    return _native.library_available()


def is_sm100_cuda(tensor: torch.Tensor) -> bool:
    if tensor.device.type != "cuda" or not torch.cuda.is_available():
        return False
    index = tensor.device.index if tensor.device.index is not None else torch.cuda.current_device()
    return tuple(torch.cuda.get_device_capability(index)) == (10, 0)


def require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


def launch(fn, *args) -> None:  # noqa: ANN001 - thin forwarding helper
    """Run a launch on the tensors' device, translating failures to RuntimeError."""

    try:
        fn(*args)
    except RuntimeError:
        raise
    except Exception as exc:  # ctypes argument errors and the like
        raise RuntimeError(f"libb200tx launch failed: {exc}") from exc
