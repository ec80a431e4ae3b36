"""Multi-GPU execution of the sm100 forward, one process per GPU.

Two partitionings, both built on batch-row / head independence of the block
(the reference relies on the same independence in
solution/runtimes/batch_tiled_graph.py:13-15 and
solution/shape14/executor.py:12-49; the reference itself is single-GPU):

* Batch sharding (`batch_shard_bounds`): rank r owns a contiguous slice of
  batch rows and runs the unmodified single-GPU program on it.  No
  collective is needed on the data path.

* Head-sharded tensor parallelism (`TensorParallelTransformer`), for batches
  smaller than the GPU count (B=4 on 8 GPUs), over the
  whole world or over the tensor-parallel groups of `tensor_parallel_groups`
  (data-parallel replicas of tp ranks, each taking its own batch rows).  Rank r owns
  heads [r H/W, (r+1) H/W) and FFN columns [r F/W, (r+1) F/W):
      qkv   = n . Wqkv_r^T + bqkv_r           local heads only (column parallel)
      ctx_r = attention(qkv)                  local heads
      u     = allreduce_sum(ctx_r . Wo_r^T) + bo       (row parallel)
      r, n  = r + u, LN(r)                    replicated on every rank
      h_r   = GELU(n . W1_r^T + b1_r)         (column parallel)
      u     = allreduce_sum(h_r . W2_r^T) + b2         (row parallel)
  The biases of the row-parallel projections are added once, by rank 0's
  partial.  Every rank ends with the full output.  Two reductions are built:
  * ``reduction="nccl"``: the partial is all-reduced by NCCL (NVLink/NVSwitch)
    and the residual LayerNorm reads the sum;
  * ``reduction="peer"`` (`PeerReduction`): the GEMM writes its partial into a
    buffer the other ranks of the group mapped through CUDA IPC, a one-warp
    kernel publishes an epoch into each peer's flag array, and the residual
    LayerNorm kernel itself waits for the peers' epochs and sums all partials
    over NVLink loads while it normalises -- the reduction is fused into the
    kernel that consumes it, and no all-reduce moves the data twice.  Groups
    of three or more (``peer_scatter``) reduce and normalise only their own
    slice of the rows and write it into every rank's gather buffer, so a
    rank moves (P - 1)/P of the rows each way instead of P - 1 whole
    partials; the residual stream then stays sharded by rows.

Failures inside a step.  On the NCCL path a departed peer ends the step's
collective with an error after the process group's timeout.  On the peer
path no collective runs inside the step: the LayerNorm's wait for a peer's
epoch is bounded (2 s) and, when it runs out, records its code in the device
error word and writes nothing; ``forward`` then reads the word after the
step and raises ``PeerWaitTimeout`` (``check_peer_errors``).  Failures
between steps are caught on the host by ``StepLiveness``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..kernels import (
    sm100_flash_attention,
    sm100_initial_layer_norm,
    sm100_linear,
    sm100_residual_layer_norm,
)
from .liveness import StepLiveness

HEAD_DIM = 64


class PeerWaitTimeout(RuntimeError):
    """A device-side wait of the tensor-parallel step ran out: a peer of the
    group did not publish its partial in time, so the step's output was not
    written."""

    def __init__(self, code: int) -> None:
        self.code = code
        super().__init__(
            f"a device wait ran out during the tensor-parallel step (device error 0x{code:x}); the output "
            "was not written.  The error word stays set (later kernels on this device stop early) until "
            "solution._native.device_error(clear=True)."
        )


def raise_on_error_word(word: int) -> None:
    """Raise PeerWaitTimeout when the device error word read after a step is set."""

    code = int(word) & 0xFFFFFFFF
    if code != 0:
        raise PeerWaitTimeout(code)


class _DeviceBuffer:
    """A raw device allocation of this library, addressed by the launch
    wrappers like a contiguous tensor (they read data_ptr() and dtype)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], dtype: torch.dtype) -> None:
        self.ptr = ptr
        self.shape = shape
        self.dtype = dtype

    def data_ptr(self) -> int:
        return self.ptr


class _CudaArray:
    """A device allocation of this library presented to torch through the
    CUDA array interface (no ownership: the owner frees it)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None,
        }


def _tensor_view(ptr: int, shape: tuple[int, int], dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch tensor over `ptr` (bf16 through its 16-bit bit pattern)."""

    typestr = {torch.float32: "<f4", torch.bfloat16: "<u2"}[dtype]
    with torch.cuda.device(device):
        t = torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class PeerReduction:
    """Partial-sum exchange of one tensor-parallel group over NVLink peer memory.

    Every rank owns two bf16 partial buffers (used alternately by the two
    reductions of a block) and a flag array with one uint32 slot per group
    rank, all allocated by libb200tx and shared with the group through CUDA
    IPC handles (exchanged once with ``all_gather_object``).  ``signal()``
    publishes the next epoch into this rank's slot of every peer's flags
    after the partial is written; the peer LayerNorm waits for all epochs.

    Reuse needs no extra acknowledgement: a rank rewrites buffer k only two
    reductions later, after its own LayerNorm waited for the peers' epoch of
    the reduction in between, which each peer publishes only after its
    LayerNorm finished reading buffer k.

    ``scatter`` (the default for groups of three or more) reduces each rank's
    slice of the rows only and gathers the normalised rows: every rank also
    owns a bf16 and an fp32 [rows, cols] gather buffer that all ranks write
    their slices into, a second flag array ("slice landed", published by the
    last CTA of the slice's LayerNorm) and a CTA counter.  A rank's gather
    buffer is written by a peer only after that peer waited for this rank's
    partial epoch of the same reduction, published after every earlier read
    of the buffer here; so it too needs no acknowledgement.  The residual
    stream then stays sharded by rows: each rank keeps its slice only.
    """

    def __init__(
        self, group: object, rows: int, cols: int, device: torch.device, *, scatter: bool | None = None
    ) -> None:
        import torch.distributed as dist

        from .. import _native

        self._native = _native
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer reduction is built for groups of up to 8 ranks")
        self.rows, self.cols, self.device = rows, cols, device
        self.scatter = self.world >= 3 if scatter is None else bool(scatter)
        if self.scatter and self.world < 2:
            raise ValueError("the scattered reduction needs a group of two or more ranks")
        # Flag block: [0, 32) partial epochs by peer, [32, 64) "slice landed"
        # epochs by peer, [64, 68) this rank's CTA counter.
        sizes = [rows * cols * 2, rows * cols * 2, 128]
        if self.scatter:
            sizes += [rows * cols * 2, rows * cols * 4]  # gather buffers: bf16 normed, fp32 final
        with torch.cuda.device(device):
            own = [_native.peer_alloc(n) for n in sizes]
        self._own = [ptr for ptr, _ in own]
        gathered: list[object] = [None] * self.world
        dist.all_gather_object(gathered, [h for _, h in own], group=group)
        self._opened: list[int] = []
        mapped: list[list[int]] = []
        with torch.cuda.device(device):
            for r, hs in enumerate(gathered):
                if r == self.rank:
                    ptrs = self._own
                else:
                    ptrs = [_native.peer_open(h) for h in hs]
                    self._opened += ptrs
                mapped.append(ptrs)
        self.partials = [[m[0] for m in mapped], [m[1] for m in mapped]]
        peer_flags = [m[2] for m in mapped]
        self.flags = self._own[2]
        self.done_flags = self.flags + 32
        self.counter = self.flags + 64
        self.counter_value = 0
        # This rank's slot in each peer's flag arrays (its own slot unused).
        self.slots = [peer_flags[r] + 4 * self.rank for r in range(self.world) if r != self.rank]
        self.done_slots = [0 if r == self.rank else peer_flags[r] + 32 + 4 * self.rank for r in range(self.world)]
        self.gather_bf16 = [m[3] for m in mapped] if self.scatter else []
        self.gather_f32 = [m[4] for m in mapped] if self.scatter else []
        self.epoch = 0
        self._buffer = 0

    def partial(self, rows: int) -> _DeviceBuffer:
        """This rank's buffer for the next reduction."""

        if rows > self.rows:
            raise ValueError(f"{rows} rows exceed the {self.rows} the peer buffers were sized for")
        return _DeviceBuffer(self._own[self._buffer], (rows, self.cols), torch.bfloat16)

    def signal(self) -> None:
        self.epoch += 1
        self._native.peer_signal(self.slots, self.epoch, self.device)

    def reduce_layer_norm(self, residual_in: torch.Tensor, **kwargs: object) -> None:
        """residual_in + the group's partials of this reduction, normalised."""

        self._native.residual_layer_norm_peer(
            residual_in, self.partials[self._buffer], self.rank, self.flags, self.epoch, **kwargs
        )
        self._buffer ^= 1

    def slice_bounds(self, rows: int) -> tuple[int, int]:
        """This rank's rows [start, stop) of a scattered reduction."""

        return batch_shard_bounds(rows, self.rank, self.world)

    def gather_tensor(self, rows: int, dtype: torch.dtype) -> torch.Tensor:
        """This rank's gather buffer as a [rows, cols] tensor (bf16: the
        normalised input of the next projections; fp32: the final output)."""

        if not self.scatter:
            raise RuntimeError("gather buffers exist in the scattered mode only")
        if rows > self.rows:
            raise ValueError(f"{rows} rows exceed the {self.rows} the peer buffers were sized for")
        ptr = self._own[3] if dtype == torch.bfloat16 else self._own[4]
        return _tensor_view(ptr, (rows, self.cols), dtype, self.device)

    def reduce_layer_norm_scattered(
        self, residual_in: torch.Tensor, residual_out: torch.Tensor | None, out_dtype: torch.dtype,
        gamma: torch.Tensor, beta: torch.Tensor, eps: float,
    ) -> None:
        """This rank's slice of residual_in + the partials, normalised into
        every rank's gather buffer of `out_dtype`; then the stream waits until
        every peer's slice has landed in this rank's buffer."""

        rows = residual_in.numel() // residual_in.shape[-1]
        start, stop = self.slice_bounds(rows)
        outs = self.gather_bf16 if out_dtype == torch.bfloat16 else self.gather_f32
        if stop > start:
            self.counter_value = self._native.residual_layer_norm_peer_rs(
                residual_in, self.partials[self._buffer], self.rank, self.flags, self.epoch, start, stop - start,
                residual_out, outs, out_dtype, gamma, beta, eps, self.done_slots, self.counter, self.counter_value,
            )
        else:
            # An empty slice still publishes its epoch, so the peers' waits end.
            self._native.peer_signal([s for s in self.done_slots if s], self.epoch, self.device)
        self._native.peer_wait(self.done_flags, self.world, self.rank, self.epoch, self.device)
        self._buffer ^= 1

    def close(self) -> None:
        """Unmap the peers' buffers, then (once every rank has) free our own.

        Collective over the group: every rank must call it.
        """

        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self._native.peer_close(ptr)
        self._opened = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._own:
                self._native.peer_free(ptr)
        self._own = []


def batch_shard_bounds(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous rows [start, stop) of a batch owned by `rank` (sizes differ by <= 1)."""

    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def tensor_parallel_groups(tp: int) -> tuple[object, int, int]:
    """Split the world into data-parallel replicas of `tp` consecutive ranks.

    Every rank must call this with the same `tp` (collective group creation).
    Returns (this rank's tensor-parallel process group, its replica index,
    the number of replicas).  With tp == world there is one replica over all
    ranks; with tp == 1 every rank is its own replica.
    """

    import torch.distributed as dist

    world = dist.get_world_size()
    rank = dist.get_rank()
    if isinstance(tp, bool) or not isinstance(tp, int) or tp <= 0 or world % tp:
        raise ValueError(f"tensor-parallel size {tp} must divide the world size {world}")
    mine = None
    for first in range(0, world, tp):
        group = dist.new_group(list(range(first, first + tp)))
        if first <= rank < first + tp:
            mine = group
    return mine, rank // tp, world // tp


@dataclass
class LayerShard:
    """One rank's slice of a block's projection weights (any dtype)."""

    w_qkv: torch.Tensor  # [3 D/W, D]: this rank's q rows; k rows; v rows
    b_qkv: torch.Tensor  # [3 D/W]
    w_o: torch.Tensor  # [D, D/W]: out-proj columns of this rank's heads
    b_o: torch.Tensor  # [D] on rank 0, zeros elsewhere
    w_1: torch.Tensor  # [F/W, D]
    b_1: torch.Tensor  # [F/W]
    w_2: torch.Tensor  # [D, F/W]
    b_2: torch.Tensor  # [D] on rank 0, zeros elsewhere


def shard_layer(
    w_qkv: torch.Tensor,
    b_qkv: torch.Tensor,
    w_o: torch.Tensor,
    b_o: torch.Tensor,
    w_1: torch.Tensor,
    b_1: torch.Tensor,
    w_2: torch.Tensor,
    b_2: torch.Tensor,
    *,
    num_heads: int,
    rank: int,
    world: int,
) -> LayerShard:
    """Cut one block's full weights into rank `rank`'s tensor-parallel shard.

    ``w_qkv`` is the packed [3D, D] projection with rows q;k;v (the layout
    ``copy_model_weights`` produces); ``w_o`` is [D, D]; ``w_1`` [F, D];
    ``w_2`` [D, F].  Raises ValueError when heads or FFN columns do not split
    evenly over `world` ranks.
    """

    d_model = w_qkv.shape[1]
    ffn = w_1.shape[0]
    if num_heads % world or ffn % world:
        raise ValueError(f"{num_heads} heads / FFN {ffn} do not split over {world} ranks")
    d_local = d_model // world
    f_local = ffn // world
    heads = slice(rank * d_local, (rank + 1) * d_local)
    cols = slice(rank * f_local, (rank + 1) * f_local)

    def block(t: torch.Tensor, which: int) -> torch.Tensor:
        return t[which * d_model + heads.start : which * d_model + heads.stop]

    owner = rank == 0
    return LayerShard(
        w_qkv=torch.cat([block(w_qkv, i) for i in range(3)], dim=0).contiguous(),
        b_qkv=torch.cat([block(b_qkv, i) for i in range(3)], dim=0).contiguous(),
        w_o=w_o[:, heads].contiguous(),
        b_o=b_o.clone() if owner else torch.zeros_like(b_o),
        w_1=w_1[cols].contiguous(),
        b_1=b_1[cols].contiguous(),
        w_2=w_2[:, cols].contiguous(),
        b_2=b_2.clone() if owner else torch.zeros_like(b_2),
    )


class TensorParallelTransformer:
    """Head-sharded forward of a `UserOptimizedTransformer` over a process group.

    Built once per rank from the full fp32 model (the same weights on every
    rank); holds this rank's bf16 weight shards on its GPU.  `forward(x)` takes
    the full [B, S, D] input on every rank and returns the full output on
    every rank.  Only inference; the plan-level checks of the single-GPU model
    (sm100 device, head_dim 64, contiguous fp32/bf16 input) apply unchanged.
    """

    def __init__(
        self,
        model: torch.nn.Module,
        *,
        group: object | None = None,
        partial_dtype: torch.dtype = torch.float32,
        reduction: str = "nccl",
        liveness: StepLiveness | None = None,
        check_peer_errors: bool = True,
        peer_scatter: bool | None = None,
    ) -> None:
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("TensorParallelTransformer needs an initialised process group")
        if partial_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("partial_dtype must be float32 or bfloat16")
        if reduction not in ("nccl", "peer"):
            raise ValueError("reduction must be 'nccl' or 'peer'")
        self.reduction = reduction
        self.peer_scatter = peer_scatter
        self.liveness = liveness
        self.check_peer_errors = check_peer_errors
        self._error_word: torch.Tensor | None = None
        self._peer: PeerReduction | None = None
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.config = model.config
        if self.config.num_heads % self.world:
            raise ValueError("num_heads must divide evenly over the ranks")
        self.heads_local = self.config.num_heads // self.world
        self.partial_dtype = partial_dtype
        device = next(model.parameters()).device
        if device.type != "cuda":
            raise RuntimeError("TensorParallelTransformer runs on CUDA devices only")
        self.device = device
        self.causal = bool(self.config.causal)
        self.layers: list[LayerShard] = []
        self.norms: list[tuple[torch.nn.LayerNorm, torch.nn.LayerNorm]] = []
        with torch.no_grad():
            for layer in model.layers:
                shard = shard_layer(
                    layer.attention.qkv_proj.weight.detach(),
                    layer.attention.qkv_proj.bias.detach(),
                    layer.attention.out_proj.weight.detach(),
                    layer.attention.out_proj.bias.detach(),
                    layer.ffn_in.weight.detach(),
                    layer.ffn_in.bias.detach(),
                    layer.ffn_out.weight.detach(),
                    layer.ffn_out.bias.detach(),
                    num_heads=self.config.num_heads,
                    rank=self.rank,
                    world=self.world,
                )
                self.layers.append(
                    LayerShard(
                        w_qkv=shard.w_qkv.to(torch.bfloat16).contiguous(),
                        b_qkv=shard.b_qkv.float().contiguous(),
                        w_o=shard.w_o.to(torch.bfloat16).contiguous(),
                        b_o=shard.b_o.float().contiguous(),
                        w_1=shard.w_1.to(torch.bfloat16).contiguous(),
                        b_1=shard.b_1.float().contiguous(),
                        w_2=shard.w_2.to(torch.bfloat16).contiguous(),
                        b_2=shard.b_2.float().contiguous(),
                    )
                )
                self.norms.append((layer.norm1.kernel_norm(), layer.norm2.kernel_norm()))
        self.final_norm = model.final_norm.kernel_norm()

    def _all_reduce(self, partial: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)

    def _peer_reduction(self, rows: int, d_model: int) -> PeerReduction:
        if self._peer is None or self._peer.rows < rows:
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerReduction(self.group, rows, d_model, self.device, scatter=self.peer_scatter)
        return self._peer

    def close(self) -> None:
        """Release the peer buffers (the group must still be alive)."""

        if self._peer is not None:
            self._peer.close()
            self._peer = None

    @torch.inference_mode()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .. import _native
        from ..kernels.projection import can_use_sm100_linear

        if x.device != self.device or not x.is_contiguous() or x.dim() != 3:
            raise ValueError("x must be a contiguous [B, S, D] tensor on this rank's GPU")
        if self.liveness is not None:
            # Every rank of the group is alive at this step boundary, or
            # RankFailure is raised before anything of this step is launched.
            self.liveness.enter()
        batch, seq, d_model = x.shape
        rows = batch * seq
        d_local = d_model // self.world
        f_local = self.layers[0].w_1.shape[0] if self.layers else 0
        flat = x.reshape(rows, d_model)
        out = torch.empty_like(x)
        if not self.layers:
            sm100_initial_layer_norm(flat, self.final_norm, out_dtype=x.dtype, normalized_out=out.view(rows, d_model))
            return out
        peer = None
        if self.reduction == "peer":
            if x.dtype != torch.float32:
                raise ValueError("the peer reduction reads the fp32 input as the first residual")
            peer = self._peer_reduction(rows, d_model)
        residual = torch.empty((rows, d_model), dtype=torch.float32, device=x.device)
        scattered = peer is not None and peer.scatter
        # Scattered: the normalised rows are gathered into this rank's peer
        # buffer, which the next projections read in place.
        normed = (
            peer.gather_tensor(rows, torch.bfloat16)
            if scattered
            else torch.empty((rows, d_model), dtype=torch.bfloat16, device=x.device)
        )
        qkv = torch.empty((batch, seq, 3 * d_local), dtype=torch.bfloat16, device=x.device)
        context = torch.empty((batch, seq, d_local), dtype=torch.bfloat16, device=x.device)
        hidden = torch.empty((rows, f_local), dtype=torch.bfloat16, device=x.device)
        partial = (
            None if peer is not None else torch.empty((rows, d_model), dtype=self.partial_dtype, device=x.device)
        )

        def reduce_norm(
            a: torch.Tensor,
            w: torch.Tensor,
            b: torch.Tensor,
            residual_in: torch.Tensor,
            norm: torch.nn.LayerNorm,
            *,
            last: bool,
            normalized_out: torch.Tensor,
        ) -> None:
            """Row-parallel projection, group reduction, residual add + LN."""

            out_dtype = x.dtype if last else torch.bfloat16
            if peer is None:
                sm100_linear(a, w, b, out_dtype=self.partial_dtype, out=partial)
                self._all_reduce(partial)
                sm100_residual_layer_norm(
                    residual_in, partial, norm, final_boundary=last, out_dtype=out_dtype,
                    residual_out=None if last else residual, keep_residual=not last,
                    normalized_out=normalized_out,
                )
                return
            if not can_use_sm100_linear(a, w, b):
                raise RuntimeError("sm100 linear is ineligible for the requested operands")
            _native.linear(a, w, b, peer.partial(rows), _native.EPI_BIAS, _native.GEMM_PAIR)
            peer.signal()
            if scattered:
                # This rank's slice of the rows; residual stays sharded by rows.
                peer.reduce_layer_norm_scattered(
                    residual_in, None if last else residual, out_dtype, norm.weight, norm.bias, norm.eps
                )
                if last:
                    normalized_out.copy_(peer.gather_tensor(rows, out_dtype))
                return
            peer.reduce_layer_norm(
                residual_in, residual_out=residual, normed=normalized_out,
                gamma=norm.weight, beta=norm.bias, eps=norm.eps,
            )

        sm100_initial_layer_norm(flat, self.norms[0][0], normalized_out=normed)
        source = flat
        for index, shard in enumerate(self.layers):
            sm100_linear(normed, shard.w_qkv, shard.b_qkv, out=qkv.view(rows, 3 * d_local))
            sm100_flash_attention(qkv, self.heads_local, causal=self.causal, out=context)
            reduce_norm(
                context.view(rows, d_local), shard.w_o, shard.b_o, source, self.norms[index][1],
                last=False, normalized_out=normed,
            )
            source = residual
            sm100_linear(normed, shard.w_1, shard.b_1, gelu=True, out=hidden)
            last = index == len(self.layers) - 1
            next_norm = self.final_norm if last else self.norms[index + 1][0]
            reduce_norm(
                hidden, shard.w_2, shard.b_2, residual, next_norm,
                last=last, normalized_out=out.view(rows, d_model) if last else normed,
            )
        if peer is not None and self.check_peer_errors:
            self._raise_on_device_error()
        return out

    def _raise_on_device_error(self) -> None:
        """Wait for this step and read the device error word.

        The peer LayerNorm waits (bounded, 2 s) for every peer's epoch; a wait
        that runs out writes nothing and records kErrPeerWait (0x301) in the
        device error word instead.  No collective runs inside a peer-path
        step, so this check is what turns a departed or stalled peer into an
        exception rather than an output that was never written.  It costs one
        host synchronisation per forward; ``check_peer_errors=False`` leaves
        the check to the caller (``_native.device_error()``).
        """

        from .. import _native

        if self._error_word is None:
            self._error_word = torch.zeros(1, dtype=torch.int32).pin_memory()
        _native.device_error_async(self._error_word)
        torch.cuda.current_stream(self.device).synchronize()
        raise_on_error_word(int(self._error_word.item()))

    __call__ = forward


__all__ = [
    "LayerShard",
    "PeerReduction",
    "PeerWaitTimeout",
    "TensorParallelTransformer",
    "batch_shard_bounds",
    "raise_on_error_word",
    "shard_layer",
    "tensor_parallel_groups",
]
