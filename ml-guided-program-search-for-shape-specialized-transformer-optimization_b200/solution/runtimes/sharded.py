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
  The partial sums travel through NCCL (NVLink/NVSwitch) into local buffers;
  the biases of the row-parallel projections are added once, after the
  reduction, by rank 0's partial.  Every rank ends with the full output.
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

HEAD_DIM = 64


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
    ) -> None:
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("TensorParallelTransformer needs an initialised process group")
        if partial_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("partial_dtype must be float32 or bfloat16")
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

    @torch.inference_mode()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.device != self.device or not x.is_contiguous() or x.dim() != 3:
            raise ValueError("x must be a contiguous [B, S, D] tensor on this rank's GPU")
        batch, seq, d_model = x.shape
        rows = batch * seq
        d_local = d_model // self.world
        f_local = self.layers[0].w_1.shape[0] if self.layers else 0
        flat = x.reshape(rows, d_model)
        out = torch.empty_like(x)
        if not self.layers:
            sm100_initial_layer_norm(flat, self.final_norm, out_dtype=x.dtype, normalized_out=out.view(rows, d_model))
            return out
        residual = torch.empty((rows, d_model), dtype=torch.float32, device=x.device)
        normed = torch.empty((rows, d_model), dtype=torch.bfloat16, device=x.device)
        qkv = torch.empty((batch, seq, 3 * d_local), dtype=torch.bfloat16, device=x.device)
        context = torch.empty((batch, seq, d_local), dtype=torch.bfloat16, device=x.device)
        hidden = torch.empty((rows, f_local), dtype=torch.bfloat16, device=x.device)
        partial = torch.empty((rows, d_model), dtype=self.partial_dtype, device=x.device)

        sm100_initial_layer_norm(flat, self.norms[0][0], normalized_out=normed)
        source = flat
        for index, shard in enumerate(self.layers):
            sm100_linear(normed, shard.w_qkv, shard.b_qkv, out=qkv.view(rows, 3 * d_local))
            sm100_flash_attention(qkv, self.heads_local, causal=self.causal, out=context)
            sm100_linear(
                context.view(rows, d_local), shard.w_o, shard.b_o, out_dtype=self.partial_dtype, out=partial
            )
            self._all_reduce(partial)
            sm100_residual_layer_norm(
                source, partial, self.norms[index][1], final_boundary=False,
                residual_out=residual, normalized_out=normed,
            )
            source = residual
            sm100_linear(normed, shard.w_1, shard.b_1, gelu=True, out=hidden)
            sm100_linear(hidden, shard.w_2, shard.b_2, out_dtype=self.partial_dtype, out=partial)
            self._all_reduce(partial)
            last = index == len(self.layers) - 1
            next_norm = self.final_norm if last else self.norms[index + 1][0]
            sm100_residual_layer_norm(
                residual, partial, next_norm, final_boundary=last,
                out_dtype=x.dtype if last else torch.bfloat16,
                residual_out=residual,
                normalized_out=out.view(rows, d_model) if last else normed,
            )
        return out

    __call__ = forward


__all__ = [
    "LayerShard",
    "TensorParallelTransformer",
    "batch_shard_bounds",
    "shard_layer",
    "tensor_parallel_groups",
]
