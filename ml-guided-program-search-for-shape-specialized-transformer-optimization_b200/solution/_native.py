"""ctypes binding of libb200tx (include/b200tx.h).

This module is the only place that touches the C ABI.  It loads the in-tree
``solution/_lib/libb200tx.so`` and exposes one checked Python call per entry
point.  There is no fallback: when the library is missing or the device is not
an sm_100 part, every call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libb200tx.so"
ABI_VERSION = 2

F32 = 0
BF16 = 1
EPI_BIAS = 0
EPI_BIAS_GELU = 1
GEMM_1SM = 0
GEMM_PAIR = 1
GEMM_WARP = 2
ATTN_PAIRED = 0
ATTN_SINGLE = 1
ATTN_QUAD = 2
ATTN_PERSISTENT = 3
ATTN_DUO = 4
ATTN_PINGPONG = 5
MASK_DROP_UPDATE = 1
MASK_ZERO_RESIDUAL = 2
MASK_ZERO_NORMED = 4

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_load_error: str | None = None

_c_int64 = ctypes.c_int64
_c_void_p = ctypes.c_void_p


def _declare(lib: ctypes.CDLL) -> None:
    lib.b200tx_abi_version.restype = ctypes.c_int
    lib.b200tx_abi_version.argtypes = []
    lib.b200tx_last_error.restype = ctypes.c_char_p
    lib.b200tx_last_error.argtypes = []
    lib.b200tx_device_error.restype = ctypes.c_int
    lib.b200tx_device_error.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
    lib.b200tx_device_error_async.restype = ctypes.c_int
    lib.b200tx_device_error_async.argtypes = [_c_void_p, _c_void_p]
    lib.b200tx_device_check.restype = ctypes.c_int
    lib.b200tx_device_check.argtypes = [
        ctypes.POINTER(ctypes.c_int),
        ctypes.POINTER(ctypes.c_int),
        ctypes.POINTER(ctypes.c_int),
    ]
    lib.b200tx_residual_layer_norm.restype = ctypes.c_int
    lib.b200tx_residual_layer_norm.argtypes = [
        _c_void_p,  # residual_in
        ctypes.c_int,  # in_dtype
        _c_void_p,  # update
        ctypes.c_int,  # update_dtype
        _c_void_p,  # residual_out
        _c_void_p,  # normed
        ctypes.c_int,  # out_dtype
        _c_void_p,  # gamma
        _c_void_p,  # beta
        _c_int64,  # rows
        _c_int64,  # cols
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_residual_layer_norm_masked.restype = ctypes.c_int
    lib.b200tx_residual_layer_norm_masked.argtypes = [
        _c_void_p,  # residual_in
        ctypes.c_int,  # in_dtype
        _c_void_p,  # update
        ctypes.c_int,  # update_dtype
        _c_void_p,  # residual_out
        _c_void_p,  # normed
        ctypes.c_int,  # out_dtype
        _c_void_p,  # gamma
        _c_void_p,  # beta
        _c_void_p,  # row_valid
        ctypes.c_int,  # mask_mode
        _c_int64,  # rows
        _c_int64,  # cols
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    _tail = [
        _c_void_p,  # residual_in
        ctypes.c_int,  # in_dtype
        _c_void_p,  # residual_out
        _c_void_p,  # normed
        ctypes.c_int,  # out_dtype
        _c_void_p,  # gamma
        _c_void_p,  # beta
        _c_void_p,  # row_valid
        ctypes.c_int,  # mask_mode
        ctypes.c_int,  # update_dtype
        _c_int64,  # rows
        _c_int64,  # cols
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_linear_residual_layer_norm.restype = ctypes.c_int
    lib.b200tx_linear_residual_layer_norm.argtypes = [
        _c_void_p,  # x
        _c_void_p,  # w
        _c_void_p,  # bias
        _c_int64,  # inner
        *_tail,
    ]
    lib.b200tx_mlp_residual_layer_norm.restype = ctypes.c_int
    lib.b200tx_mlp_residual_layer_norm.argtypes = [
        _c_void_p,  # x
        _c_void_p,  # w1
        _c_void_p,  # b1
        _c_void_p,  # w2
        _c_void_p,  # b2
        _c_int64,  # ffn_dim
        *_tail,
    ]
    lib.b200tx_linear.restype = ctypes.c_int
    lib.b200tx_linear.argtypes = [
        _c_void_p,  # a
        _c_void_p,  # w
        _c_void_p,  # bias
        _c_void_p,  # out
        ctypes.c_int,  # out_dtype
        _c_int64,  # M
        _c_int64,  # N
        _c_int64,  # K
        ctypes.c_int,  # epilogue
        _c_void_p,  # stream
    ]
    lib.b200tx_linear_ex.restype = ctypes.c_int
    lib.b200tx_linear_ex.argtypes = [
        _c_void_p,  # a
        _c_void_p,  # w
        _c_void_p,  # bias
        _c_void_p,  # out
        ctypes.c_int,  # out_dtype
        _c_int64,  # M
        _c_int64,  # N
        _c_int64,  # K
        ctypes.c_int,  # epilogue
        ctypes.c_int,  # variant
        _c_void_p,  # stream
    ]
    lib.b200tx_attention.restype = ctypes.c_int
    lib.b200tx_attention.argtypes = [
        _c_void_p,  # qkv
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # heads
        _c_int64,  # head_dim
        ctypes.c_float,  # scale
        ctypes.c_int,  # causal
        _c_void_p,  # stream
    ]
    lib.b200tx_attention_ex.restype = ctypes.c_int
    lib.b200tx_attention_ex.argtypes = [
        _c_void_p,  # qkv
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # heads
        _c_int64,  # head_dim
        ctypes.c_float,  # scale
        ctypes.c_int,  # causal
        ctypes.c_int,  # variant
        _c_void_p,  # stream
    ]
    lib.b200tx_peer_alloc.restype = ctypes.c_int
    lib.b200tx_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
    lib.b200tx_peer_open.restype = ctypes.c_int
    lib.b200tx_peer_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.b200tx_peer_close.restype = ctypes.c_int
    lib.b200tx_peer_close.argtypes = [_c_void_p]
    lib.b200tx_peer_free.restype = ctypes.c_int
    lib.b200tx_peer_free.argtypes = [_c_void_p]
    lib.b200tx_peer_signal.restype = ctypes.c_int
    lib.b200tx_peer_signal.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_uint32, _c_void_p]
    lib.b200tx_residual_layer_norm_peer.restype = ctypes.c_int
    lib.b200tx_residual_layer_norm_peer.argtypes = [
        _c_void_p,  # residual_in (fp32)
        ctypes.POINTER(ctypes.c_void_p),  # partials
        ctypes.c_int,  # count
        ctypes.c_int,  # self
        _c_void_p,  # flags
        ctypes.c_uint32,  # epoch
        _c_void_p,  # residual_out
        _c_void_p,  # normed
        ctypes.c_int,  # out_dtype
        _c_void_p,  # gamma
        _c_void_p,  # beta
        _c_void_p,  # row_valid
        ctypes.c_int,  # mask_mode
        _c_int64,  # rows
        _c_int64,  # cols
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_residual_layer_norm_peer_rs.restype = ctypes.c_int
    lib.b200tx_residual_layer_norm_peer_rs.argtypes = [
        _c_void_p,  # residual_in (fp32)
        ctypes.POINTER(ctypes.c_void_p),  # partials
        ctypes.c_int,  # count
        ctypes.c_int,  # self
        _c_void_p,  # flags
        ctypes.c_uint32,  # epoch
        _c_int64,  # row_begin
        _c_int64,  # row_count
        _c_void_p,  # residual_out
        ctypes.POINTER(ctypes.c_void_p),  # outs
        ctypes.c_int,  # out_dtype
        _c_void_p,  # gamma
        _c_void_p,  # beta
        ctypes.POINTER(ctypes.c_void_p),  # done_slots
        _c_void_p,  # counter
        ctypes.c_uint32,  # counter_base
        ctypes.POINTER(ctypes.c_uint32),  # counter_after
        _c_int64,  # rows
        _c_int64,  # cols
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_seq_weight_image.restype = ctypes.c_int
    lib.b200tx_seq_weight_image.argtypes = [_c_void_p, _c_void_p, _c_void_p]
    lib.b200tx_sequence_forward.restype = ctypes.c_int
    lib.b200tx_sequence_forward.argtypes = [
        _c_void_p,  # x
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # d_model
        _c_int64,  # heads
        _c_int64,  # ffn_dim
        ctypes.c_int,  # num_layers
        ctypes.POINTER(SeqLayer),  # layers
        _c_void_p,  # ln0 gamma
        _c_void_p,  # ln0 beta
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_sequence_forward_noalloc.restype = ctypes.c_int
    lib.b200tx_sequence_forward_noalloc.argtypes = [
        _c_void_p,  # x
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # d_model
        _c_int64,  # heads
        _c_int64,  # ffn_dim
        ctypes.c_int,  # num_layers
        ctypes.POINTER(SeqLayerWeights),  # layers
        _c_void_p,  # ln0 gamma
        _c_void_p,  # ln0 beta
        ctypes.c_float,  # eps
        _c_void_p,  # stream
    ]
    lib.b200tx_peer_wait.restype = ctypes.c_int
    lib.b200tx_peer_wait.argtypes = [_c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint32, _c_void_p]
    lib.b200tx_attention_generic.restype = ctypes.c_int
    lib.b200tx_attention_generic.argtypes = [
        _c_void_p,  # qkv
        _c_void_p,  # key_valid (nullable)
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # heads
        _c_int64,  # head_dim
        ctypes.c_float,  # scale
        ctypes.c_int,  # causal
        _c_void_p,  # stream
    ]
    lib.b200tx_attention_mma.restype = ctypes.c_int
    lib.b200tx_attention_mma.argtypes = list(lib.b200tx_attention_generic.argtypes)
    lib.b200tx_attention_masked.restype = ctypes.c_int
    lib.b200tx_attention_masked.argtypes = [
        _c_void_p,  # qkv
        _c_void_p,  # key_valid
        _c_void_p,  # out
        _c_int64,  # batch
        _c_int64,  # seq
        _c_int64,  # heads
        _c_int64,  # head_dim
        ctypes.c_float,  # scale
        ctypes.c_int,  # causal
        ctypes.c_int,  # variant
        _c_void_p,  # stream
    ]


def library_path() -> Path:
    return LIB_PATH


def library_available() -> bool:
    """Whether the shared library can be loaded (does not require a GPU)."""

    try:
        load()
    except RuntimeError:
        return False
    return True


def load() -> ctypes.CDLL:
    """Load libb200tx once; raise RuntimeError with the reason on failure."""

    global _lib, _load_error
    with _lock:
        if _lib is not None:
            return _lib
        if _load_error is not None:
            raise RuntimeError(_load_error)
        if not LIB_PATH.exists():
            _load_error = (
                f"libb200tx.so not built at {LIB_PATH}; run build_native.py "
                "(there is no CPU or Triton fallback)"
            )
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            _load_error = f"cannot load {LIB_PATH}: {exc}"
            raise RuntimeError(_load_error) from exc
        _declare(lib)
        version = lib.b200tx_abi_version()
        if version != ABI_VERSION:
            _load_error = f"libb200tx ABI {version} != expected {ABI_VERSION}; rebuild it"
            raise RuntimeError(_load_error)
        _lib = lib
        return lib


def _check(status: int, what: str) -> None:
    if status != 0:
        message = load().b200tx_last_error().decode("utf-8", "replace")
        raise RuntimeError(f"{what} failed (status {status}): {message}")


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The cudaStream_t of the device's current stream (a graph capture's
    stream while capturing).  Read through torch's raw-stream accessor where
    it exists: building a ``torch.cuda.Stream`` object per launch is a
    measurable share of the host time of a small eager forward."""

    current = torch.cuda.current_device()
    index = device.index if device.index is not None else current
    if index != current:
        # libb200tx resolves its per-device state (SM count, kernel
        # attributes, error word) from the current device, so a launch onto
        # another device's stream would run with the wrong state.
        raise RuntimeError(
            f"libb200tx launches on the current device: the operands are on cuda:{index} "
            f"while cuda:{current} is current (use torch.cuda.device(...))"
        )
    if _RAW_STREAM is not None:
        return int(_RAW_STREAM(index))
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return F32
    if dtype == torch.bfloat16:
        return BF16
    raise ValueError(f"unsupported dtype {dtype}; libb200tx takes float32 or bfloat16")


def device_check() -> tuple[int, int, int]:
    """Return (sm_count, cc_major, cc_minor) of the current device; raise if not sm_100."""

    lib = load()
    sm = ctypes.c_int(0)
    major = ctypes.c_int(0)
    minor = ctypes.c_int(0)
    _check(
        lib.b200tx_device_check(ctypes.byref(sm), ctypes.byref(major), ctypes.byref(minor)),
        "b200tx_device_check",
    )
    return sm.value, major.value, minor.value


def device_error(clear: bool = True) -> int:
    """Read the device error word (synchronises the device)."""

    lib = load()
    code = ctypes.c_uint(0)
    _check(lib.b200tx_device_error(int(clear), ctypes.byref(code)), "b200tx_device_error")
    return int(code.value)


def device_error_async(word: torch.Tensor) -> None:
    """Queue a copy of the device error word into ``word`` (one int32 element,
    pinned host or device memory) on the current stream of the current device.
    Nothing is synchronised; read ``word`` after the stream got there."""

    if word.numel() != 1 or word.element_size() != 4:
        raise ValueError("the error word destination is one 32-bit element")
    device = word.device if word.is_cuda else torch.device("cuda", torch.cuda.current_device())
    _check(load().b200tx_device_error_async(word.data_ptr(), _stream(device)), "b200tx_device_error_async")


def residual_layer_norm(
    residual_in: torch.Tensor,
    update: torch.Tensor | None,
    residual_out: torch.Tensor | None,
    normed: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
) -> None:
    """Launch b200tx_residual_layer_norm (or its _masked form when ``row_valid``
    is given: uint8 [rows] flags, 0 = padding row, handled per ``mask_mode``)
    on the current stream (no checks beyond the C side)."""

    cols = residual_in.shape[-1]
    rows = residual_in.numel() // cols
    lib = load()
    common = (
        residual_in.data_ptr(),
        dtype_code(residual_in.dtype),
        None if update is None else update.data_ptr(),
        F32 if update is None else dtype_code(update.dtype),
        None if residual_out is None else residual_out.data_ptr(),
        normed.data_ptr(),
        dtype_code(normed.dtype),
        gamma.data_ptr(),
        beta.data_ptr(),
    )
    stream = _stream(residual_in.device)
    if row_valid is None:
        _check(
            lib.b200tx_residual_layer_norm(*common, rows, cols, float(eps), stream),
            "b200tx_residual_layer_norm",
        )
        return
    _check(
        lib.b200tx_residual_layer_norm_masked(
            *common, row_valid.data_ptr(), int(mask_mode), rows, cols, float(eps), stream
        ),
        "b200tx_residual_layer_norm_masked",
    )


def _boundary_tail(
    residual_in: torch.Tensor,
    residual_out: torch.Tensor | None,
    normed: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    row_valid: torch.Tensor | None,
    mask_mode: int,
    update_dtype: torch.dtype,
) -> tuple:
    cols = residual_in.shape[-1]
    return (
        residual_in.data_ptr(),
        dtype_code(residual_in.dtype),
        None if residual_out is None else residual_out.data_ptr(),
        normed.data_ptr(),
        dtype_code(normed.dtype),
        gamma.data_ptr(),
        beta.data_ptr(),
        None if row_valid is None else row_valid.data_ptr(),
        int(mask_mode),
        dtype_code(update_dtype),
        residual_in.numel() // cols,
        cols,
        float(eps),
        _stream(residual_in.device),
    )


def linear_residual_layer_norm(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor,
    residual_in: torch.Tensor,
    residual_out: torch.Tensor | None,
    normed: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
    update_dtype: torch.dtype = torch.bfloat16,
) -> None:
    """Launch b200tx_linear_residual_layer_norm: LN(residual_in + round(x . w^T + bias))."""

    _check(
        load().b200tx_linear_residual_layer_norm(
            x.data_ptr(),
            w.data_ptr(),
            bias.data_ptr(),
            x.shape[-1],
            *_boundary_tail(residual_in, residual_out, normed, gamma, beta, eps, row_valid, mask_mode, update_dtype),
        ),
        "b200tx_linear_residual_layer_norm",
    )


def mlp_residual_layer_norm(
    x: torch.Tensor,
    w1: torch.Tensor,
    b1: torch.Tensor,
    w2: torch.Tensor,
    b2: torch.Tensor,
    residual_in: torch.Tensor,
    residual_out: torch.Tensor | None,
    normed: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
    update_dtype: torch.dtype = torch.bfloat16,
) -> None:
    """Launch b200tx_mlp_residual_layer_norm: LN(residual_in + round(GELU(x . w1^T + b1) . w2^T + b2))."""

    _check(
        load().b200tx_mlp_residual_layer_norm(
            x.data_ptr(),
            w1.data_ptr(),
            b1.data_ptr(),
            w2.data_ptr(),
            b2.data_ptr(),
            w1.shape[0],
            *_boundary_tail(residual_in, residual_out, normed, gamma, beta, eps, row_valid, mask_mode, update_dtype),
        ),
        "b200tx_mlp_residual_layer_norm",
    )


def linear(
    a: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor | None,
    out: torch.Tensor,
    epilogue: int,
    variant: int = GEMM_PAIR,
) -> None:
    """Launch b200tx_linear_ex: out = epilogue(a . w^T + bias) with the given
    kernel variant (GEMM_1SM, GEMM_PAIR or GEMM_WARP)."""

    k = a.shape[-1]
    m = a.numel() // k
    n = w.shape[0]
    lib = load()
    _check(
        lib.b200tx_linear_ex(
            a.data_ptr(),
            w.data_ptr(),
            None if bias is None else bias.data_ptr(),
            out.data_ptr(),
            dtype_code(out.dtype),
            m,
            n,
            k,
            int(epilogue),
            int(variant),
            _stream(a.device),
        ),
        "b200tx_linear_ex",
    )


def attention(
    qkv: torch.Tensor,
    out: torch.Tensor,
    batch: int,
    seq: int,
    heads: int,
    head_dim: int,
    scale: float,
    causal: bool,
    variant: int = ATTN_QUAD,
    key_valid: torch.Tensor | None = None,
) -> None:
    """Launch b200tx_attention_ex over a packed [B, S, 3D] projection, or
    b200tx_attention_masked when ``key_valid`` (uint8 [B, S], 0 = padding key)
    is given."""

    lib = load()
    shape = (int(batch), int(seq), int(heads), int(head_dim), float(scale), int(bool(causal)), int(variant))
    if key_valid is None:
        _check(
            lib.b200tx_attention_ex(qkv.data_ptr(), out.data_ptr(), *shape, _stream(qkv.device)),
            "b200tx_attention_ex",
        )
        return
    _check(
        lib.b200tx_attention_masked(
            qkv.data_ptr(), key_valid.data_ptr(), out.data_ptr(), *shape, _stream(qkv.device)
        ),
        "b200tx_attention_masked",
    )


def attention_mma(
    qkv: torch.Tensor,
    out: torch.Tensor,
    batch: int,
    seq: int,
    heads: int,
    head_dim: int,
    scale: float,
    causal: bool,
    key_valid: torch.Tensor | None = None,
) -> None:
    """Launch b200tx_attention_mma (warp-level tensor-core attention, head_dim 8..128)."""

    lib = load()
    _check(
        lib.b200tx_attention_mma(
            qkv.data_ptr(),
            None if key_valid is None else key_valid.data_ptr(),
            out.data_ptr(),
            int(batch),
            int(seq),
            int(heads),
            int(head_dim),
            float(scale),
            int(bool(causal)),
            _stream(qkv.device),
        ),
        "b200tx_attention_mma",
    )


def attention_generic(
    qkv: torch.Tensor,
    out: torch.Tensor,
    batch: int,
    seq: int,
    heads: int,
    head_dim: int,
    scale: float,
    causal: bool,
    key_valid: torch.Tensor | None = None,
) -> None:
    """Launch b200tx_attention_generic (CUDA-core attention, head_dim 8..256)."""

    lib = load()
    _check(
        lib.b200tx_attention_generic(
            qkv.data_ptr(),
            None if key_valid is None else key_valid.data_ptr(),
            out.data_ptr(),
            int(batch),
            int(seq),
            int(heads),
            int(head_dim),
            float(scale),
            int(bool(causal)),
            _stream(qkv.device),
        ),
        "b200tx_attention_generic",
    )


IPC_HANDLE_BYTES = 64


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """A zero-filled device buffer of this library's own and its IPC handle."""

    lib = load()
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib.b200tx_peer_alloc(int(nbytes), ctypes.byref(ptr), handle), "b200tx_peer_alloc")
    return int(ptr.value), bytes(handle.raw)


def peer_open(handle: bytes) -> int:
    lib = load()
    ptr = ctypes.c_void_p()
    _check(lib.b200tx_peer_open(handle, ctypes.byref(ptr)), "b200tx_peer_open")
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    _check(load().b200tx_peer_close(ptr), "b200tx_peer_close")


def peer_free(ptr: int) -> None:
    _check(load().b200tx_peer_free(ptr), "b200tx_peer_free")


def peer_signal(slots: list[int], epoch: int, device: torch.device) -> None:
    arr = (ctypes.c_void_p * len(slots))(*slots)
    _check(load().b200tx_peer_signal(arr, len(slots), epoch & 0xFFFFFFFF, _stream(device)), "b200tx_peer_signal")


def residual_layer_norm_peer(
    residual_in: torch.Tensor,
    partials: list[int],
    self_index: int,
    flags: int,
    epoch: int,
    residual_out: torch.Tensor | None,
    normed: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    row_valid: torch.Tensor | None = None,
    mask_mode: int = 0,
) -> None:
    """Launch b200tx_residual_layer_norm_peer: residual + sum of the group's
    bf16 partials (device pointers, partials[self_index] local), normalised."""

    cols = residual_in.shape[-1]
    rows = residual_in.numel() // cols
    arr = (ctypes.c_void_p * len(partials))(*partials)
    _check(
        load().b200tx_residual_layer_norm_peer(
            residual_in.data_ptr(),
            arr,
            len(partials),
            int(self_index),
            flags,
            epoch & 0xFFFFFFFF,
            None if residual_out is None else residual_out.data_ptr(),
            normed.data_ptr(),
            dtype_code(normed.dtype),
            gamma.data_ptr(),
            beta.data_ptr(),
            None if row_valid is None else row_valid.data_ptr(),
            int(mask_mode),
            rows,
            cols,
            float(eps),
            _stream(residual_in.device),
        ),
        "b200tx_residual_layer_norm_peer",
    )


def residual_layer_norm_peer_rs(
    residual_in: torch.Tensor,
    partials: list[int],
    self_index: int,
    flags: int,
    epoch: int,
    row_begin: int,
    row_count: int,
    residual_out: torch.Tensor | None,
    outs: list[int],
    out_dtype: torch.dtype,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    done_slots: list[int],
    counter: int,
    counter_base: int,
) -> int:
    """Launch b200tx_residual_layer_norm_peer_rs: this rank's rows of
    residual + the group's partials, normalised into every rank's output
    buffer (device pointers, index = group rank); returns the CTA counter's
    value once the launch is done."""

    cols = residual_in.shape[-1]
    rows = residual_in.numel() // cols
    count = len(partials)
    parts = (ctypes.c_void_p * count)(*partials)
    out_arr = (ctypes.c_void_p * count)(*outs)
    slots = (ctypes.c_void_p * count)(*[s or None for s in done_slots])
    after = ctypes.c_uint32(0)
    _check(
        load().b200tx_residual_layer_norm_peer_rs(
            residual_in.data_ptr(),
            parts,
            count,
            int(self_index),
            flags,
            epoch & 0xFFFFFFFF,
            int(row_begin),
            int(row_count),
            None if residual_out is None else residual_out.data_ptr(),
            out_arr,
            dtype_code(out_dtype),
            gamma.data_ptr(),
            beta.data_ptr(),
            slots,
            counter,
            counter_base & 0xFFFFFFFF,
            ctypes.byref(after),
            rows,
            cols,
            float(eps),
            _stream(residual_in.device),
        ),
        "b200tx_residual_layer_norm_peer_rs",
    )
    return int(after.value)


class SeqLayer(ctypes.Structure):
    """b200tx_seq_layer: device pointers of one layer of the whole-forward kernel."""

    _fields_ = [
        ("weight_images", ctypes.c_void_p),
        ("b_qkv", ctypes.c_void_p),
        ("b_o", ctypes.c_void_p),
        ("b_1", ctypes.c_void_p),
        ("b_2", ctypes.c_void_p),
        ("ln2_gamma", ctypes.c_void_p),
        ("ln2_beta", ctypes.c_void_p),
        ("next_gamma", ctypes.c_void_p),
        ("next_beta", ctypes.c_void_p),
    ]


class SeqLayerWeights(ctypes.Structure):
    """b200tx_seq_layer_weights: device pointers of one layer for
    b200tx_sequence_forward_noalloc (plain bf16 weights, no images)."""

    _fields_ = [
        ("w_qkv", ctypes.c_void_p),
        ("w_o", ctypes.c_void_p),
        ("w_1", ctypes.c_void_p),
        ("w_2", ctypes.c_void_p),
        ("b_qkv", ctypes.c_void_p),
        ("b_o", ctypes.c_void_p),
        ("b_1", ctypes.c_void_p),
        ("b_2", ctypes.c_void_p),
        ("ln2_gamma", ctypes.c_void_p),
        ("ln2_beta", ctypes.c_void_p),
        ("next_gamma", ctypes.c_void_p),
        ("next_beta", ctypes.c_void_p),
    ]


SEQ_IMAGE_BYTES = 128 * 128 * 2
SEQ_NOALLOC_MAX_LAYERS = 4  # B200TX_SEQ_NOALLOC_MAX_LAYERS


def seq_weight_image(weight: torch.Tensor, image: torch.Tensor) -> None:
    """Launch b200tx_seq_weight_image: a [128, 128] bf16 weight into its 32 KB operand image."""

    _check(load().b200tx_seq_weight_image(weight.data_ptr(), image.data_ptr(), _stream(weight.device)),
           "b200tx_seq_weight_image")


def sequence_forward(
    x: torch.Tensor,
    out: torch.Tensor,
    heads: int,
    layers: ctypes.Array,
    ln0_gamma: torch.Tensor,
    ln0_beta: torch.Tensor,
    eps: float,
) -> None:
    """Launch b200tx_sequence_forward: the whole forward of x [B, S, 128] into
    out; `layers` a ctypes array of SeqLayer (built once by the caller)."""

    batch, seq, d_model = x.shape
    _check(
        load().b200tx_sequence_forward(
            x.data_ptr(), out.data_ptr(), batch, seq, d_model, int(heads), d_model, len(layers), layers,
            ln0_gamma.data_ptr(), ln0_beta.data_ptr(), float(eps), _stream(x.device),
        ),
        "b200tx_sequence_forward",
    )


def peer_wait(flags: int, count: int, self_index: int, epoch: int, device: torch.device) -> None:
    """Launch b200tx_peer_wait: hold the stream until every peer's flag reaches `epoch`."""

    _check(load().b200tx_peer_wait(flags, int(count), int(self_index), epoch & 0xFFFFFFFF, _stream(device)),
           "b200tx_peer_wait")


__all__ = [
    "IPC_HANDLE_BYTES",
    "peer_alloc",
    "peer_close",
    "peer_free",
    "peer_open",
    "peer_signal",
    "peer_wait",
    "residual_layer_norm_peer",
    "SEQ_IMAGE_BYTES",
    "SeqLayer",
    "SeqLayerWeights",
    "seq_weight_image",
    "sequence_forward",
    "residual_layer_norm_peer_rs",
    "ABI_VERSION",
    "ATTN_DUO",
    "ATTN_PINGPONG",
    "ATTN_PAIRED",
    "ATTN_PERSISTENT",
    "ATTN_QUAD",
    "ATTN_SINGLE",
    "BF16",
    "EPI_BIAS",
    "EPI_BIAS_GELU",
    "F32",
    "GEMM_1SM",
    "GEMM_PAIR",
    "MASK_DROP_UPDATE",
    "MASK_ZERO_NORMED",
    "MASK_ZERO_RESIDUAL",
    "attention",
    "attention_generic",
    "device_check",
    "device_error",
    "device_error_async",
    "dtype_code",
    "library_available",
    "library_path",
    "linear",
    "load",
    "residual_layer_norm",
]
