"""Shared argument checks for the libb200tx wrappers."""

from __future__ import annotations

import torch

from .. import _native


def library_ready() -> bool:
    return _native.library_available()


_SM100_BY_DEVICE: dict[int, bool] = {}


def is_sm100_cuda(tensor: torch.Tensor) -> bool:
    """Whether the tensor lives on a compute capability 10.0 device (cached per
    device index: the capability of a device does not change in a process)."""

    if tensor.device.type != "cuda":
        return False
    index = tensor.device.index if tensor.device.index is not None else torch.cuda.current_device()
    known = _SM100_BY_DEVICE.get(index)
    if known is None:
        known = torch.cuda.is_available() and tuple(torch.cuda.get_device_capability(index)) == (10, 0)
        _SM100_BY_DEVICE[index] = known
    return known


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
