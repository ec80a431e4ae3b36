"""Multi-process sharding: batch partition, head-sharded tensor-parallel math
and its collective plumbing.

CPU tests run the tensor-parallel composition with gloo ranks (world size 2)
and numpy/torch CPU arithmetic on the very shards ``shard_layer`` produces,
against the single-process oracle.  The GPU test (two or more GPUs) runs
``TensorParallelTransformer`` over NCCL against the single-GPU model.
"""

from __future__ import annotations

import os
import socket
import tempfile
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import OfficialConfig, official_input, official_state_dict, transformer_forward
from oracle.reference_forward import gelu_erf, layer_norm
from oracle.weights import state_to_numpy
from solution.runtimes.sharded import batch_shard_bounds, shard_layer

CFG = OfficialConfig(2, 24, 256, 4, 512, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_batch_shard_bounds_partition() -> None:
    for batch in (1, 4, 7, 8, 32):
        for world in (1, 2, 3, 8):
            spans = [batch_shard_bounds(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        batch_shard_bounds(4, 2, 2)


def _packed_layer(state: dict[str, torch.Tensor], i: int) -> tuple[torch.Tensor, ...]:
    p = f"layers.{i}"
    w_qkv = torch.cat([state[f"{p}.attention.{n}_proj.weight"] for n in "qkv"], dim=0)
    b_qkv = torch.cat([state[f"{p}.attention.{n}_proj.bias"] for n in "qkv"], dim=0)
    return (
        w_qkv,
        b_qkv,
        state[f"{p}.attention.out_proj.weight"],
        state[f"{p}.attention.out_proj.bias"],
        state[f"{p}.ffn_in.weight"],
        state[f"{p}.ffn_in.bias"],
        state[f"{p}.ffn_out.weight"],
        state[f"{p}.ffn_out.bias"],
    )


def test_shards_reassemble_the_full_projections() -> None:
    state = official_state_dict(CFG, seed=0)
    full = _packed_layer(state, 0)
    world = 4
    shards = [shard_layer(*full, num_heads=CFG.num_heads, rank=r, world=world) for r in range(world)]
    x = torch.randn(5, CFG.d_model, dtype=torch.float64)
    ctx = torch.randn(5, CFG.d_model, dtype=torch.float64)
    h = torch.randn(5, CFG.ffn_dim, dtype=torch.float64)
    d_local = CFG.d_model // world
    f_local = CFG.ffn_dim // world
    # Column-parallel QKV: each rank's outputs are its heads' q, k, v columns.
    qkv_full = x @ full[0].double().T + full[1].double()
    for r, sh in enumerate(shards):
        local = x @ sh.w_qkv.double().T + sh.b_qkv.double()
        for which in range(3):
            cols = slice(which * CFG.d_model + r * d_local, which * CFG.d_model + (r + 1) * d_local)
            np.testing.assert_allclose(local[:, which * d_local : (which + 1) * d_local], qkv_full[:, cols])
    # Row-parallel out-proj and FFN-down: partial sums add up to the full map.
    o_sum = sum(ctx[:, r * d_local : (r + 1) * d_local] @ sh.w_o.double().T + sh.b_o.double() for r, sh in enumerate(shards))
    np.testing.assert_allclose(o_sum, ctx @ full[2].double().T + full[3].double(), atol=1e-10)
    f_sum = sum(h[:, r * f_local : (r + 1) * f_local] @ sh.w_2.double().T + sh.b_2.double() for r, sh in enumerate(shards))
    np.testing.assert_allclose(f_sum, h @ full[6].double().T + full[7].double(), atol=1e-10)
    with pytest.raises(ValueError):
        shard_layer(*full, num_heads=CFG.num_heads, rank=0, world=3)


def _tp_forward_cpu(x: np.ndarray, state: dict[str, torch.Tensor], rank: int, world: int) -> np.ndarray:
    """The tensor-parallel composition on CPU: local shards + gloo all-reduce."""

    ns = state_to_numpy(state)
    batch, seq, d = x.shape
    heads_local = CFG.num_heads // world
    d_local = d // world
    out = x.astype(np.float32).copy()
    for i in range(CFG.num_layers):
        sh = shard_layer(*_packed_layer(state, i), num_heads=CFG.num_heads, rank=rank, world=world)
        p = f"layers.{i}"
        n = layer_norm(out, ns[f"{p}.norm1.weight"], ns[f"{p}.norm1.bias"])
        qkv = n @ sh.w_qkv.numpy().T + sh.b_qkv.numpy()
        q, k, v = (qkv[..., j * d_local : (j + 1) * d_local].reshape(batch, seq, heads_local, 64).transpose(0, 2, 1, 3) for j in range(3))
        scores = q @ k.transpose(0, 1, 3, 2) / 8.0
        scores = np.where(np.triu(np.ones((seq, seq), bool), 1)[None, None], -np.inf, scores)
        probs = np.exp(scores - scores.max(-1, keepdims=True))
        probs /= probs.sum(-1, keepdims=True)
        ctx = (probs @ v).transpose(0, 2, 1, 3).reshape(batch, seq, d_local)
        partial = torch.from_numpy((ctx @ sh.w_o.numpy().T + sh.b_o.numpy()).astype(np.float32))
        dist.all_reduce(partial)
        out = out + partial.numpy()
        n = layer_norm(out, ns[f"{p}.norm2.weight"], ns[f"{p}.norm2.bias"])
        h = gelu_erf(n @ sh.w_1.numpy().T + sh.b_1.numpy())
        partial = torch.from_numpy((h @ sh.w_2.numpy().T + sh.b_2.numpy()).astype(np.float32))
        dist.all_reduce(partial)
        out = out + partial.numpy()
    return layer_norm(out, ns["final_norm.weight"], ns["final_norm.bias"])


def _gloo_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state = official_state_dict(CFG, seed=0)
        x = official_input(CFG, 3).numpy()
        y = _tp_forward_cpu(x, state, rank, world)
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), y)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_composition_over_gloo() -> None:
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_gloo_worker, args=(world, _free_port(), tmp), nprocs=world, start_method="spawn")
        outs = [np.load(os.path.join(tmp, f"rank{r}.npy")) for r in range(world)]
    state = state_to_numpy(official_state_dict(CFG, seed=0))
    ref = transformer_forward(official_input(CFG, 3).numpy(), state, num_heads=CFG.num_heads, num_layers=CFG.num_layers)
    for y in outs:
        np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-4)
    np.testing.assert_array_equal(outs[0], outs[1])


def _nccl_worker(
    rank: int, world: int, port: int, result_dir: str, partials: str = "fp32", reduction: str = "nccl"
) -> None:
    import datetime

    from solution.runtimes.sharded import TensorParallelTransformer
    from solution.transformer import UserOptimizedTransformer, copy_model_weights

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        cfg = OfficialConfig(2, 640, 512, 8, 1024, 2)
        model = UserOptimizedTransformer(SimpleNamespace(**cfg.__dict__))
        copy_model_weights(official_state_dict(cfg, seed=0), model)
        model = model.to(f"cuda:{rank}").eval()
        from solution.runtimes.liveness import StepLiveness

        # Every forward passes the host-side liveness check of the group first.
        live = StepLiveness(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=60.0)
        tp = TensorParallelTransformer(
            model,
            partial_dtype=torch.bfloat16 if partials == "bf16" else torch.float32,
            reduction="peer" if reduction.startswith("peer") else reduction,
            liveness=live,
            peer_scatter=True if reduction == "peer_scatter" else None,
        )
        x = official_input(cfg, 5).to(f"cuda:{rank}")
        y_tp = tp(x)
        # Repeated forwards reuse the partial buffers and flags: same bits.
        for _ in range(4):
            assert torch.equal(tp(x), y_tp)
        from solution import _native

        assert _native.device_error(clear=True) == 0
        tp.close()
        with torch.inference_mode():
            y_single = model(x)
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"tp{rank}.npy"), y_tp.cpu().numpy())
        np.save(os.path.join(result_dir, f"single{rank}.npy"), y_single.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize(
    ("partials", "reduction", "world"),
    [
        ("fp32", "nccl", 2),
        ("bf16", "nccl", 2),
        ("bf16", "peer", 2),
        # the reduce-scatter + gather form: forced on two ranks, the default on four
        ("bf16", "peer_scatter", 2),
        ("bf16", "peer", 4),
        ("bf16", "nccl", 4),
    ],
)
def test_tensor_parallel_matches_single_gpu(partials: str, reduction: str, world: int) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(
            _nccl_worker, args=(world, _free_port(), tmp, partials, reduction), nprocs=world, start_method="spawn"
        )
        tp = [np.load(os.path.join(tmp, f"tp{r}.npy")) for r in range(world)]
        single = np.load(os.path.join(tmp, "single0.npy"))
    for r in range(1, world):
        np.testing.assert_array_equal(tp[0], tp[r])
    diff = tp[0].astype(np.float64) - single
    assert np.abs(diff).max() < 2e-2
    assert np.linalg.norm(diff) / np.linalg.norm(single) < 5e-3


def _groups_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    from solution.runtimes.sharded import tensor_parallel_groups

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        group, replica, replicas = tensor_parallel_groups(2)
        value = torch.tensor([float(rank)])
        dist.all_reduce(value, group=group)
        bad = False
        try:
            tensor_parallel_groups(3)
        except ValueError:
            bad = True
        np.save(os.path.join(result_dir, f"g{rank}.npy"), np.array([value.item(), replica, replicas, bad]))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_groups_split_the_world_into_replicas() -> None:
    world = 4
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_groups_worker, args=(world, _free_port(), tmp), nprocs=world, start_method="spawn")
        got = [np.load(os.path.join(tmp, f"g{r}.npy")) for r in range(world)]
    # ranks {0,1} and {2,3}: group sums 1 and 5; replicas 0,0,1,1 of 2
    assert [g[0] for g in got] == [1.0, 1.0, 5.0, 5.0]
    assert [g[1] for g in got] == [0, 0, 1, 1]
    assert all(g[2] == 2 and g[3] == 1 for g in got)


def test_error_word_turns_into_peer_wait_timeout() -> None:
    """The post-step check of the peer path: a clear word passes, a set one
    raises with the device's code."""

    from solution.runtimes.sharded import PeerWaitTimeout, raise_on_error_word

    raise_on_error_word(0)
    with pytest.raises(PeerWaitTimeout) as info:
        raise_on_error_word(0x301)
    assert info.value.code == 0x301
    assert isinstance(info.value, RuntimeError)


@pytest.mark.gpu
def test_peer_layer_norm_wait_runs_out_and_is_reported() -> None:
    """A peer that never publishes its epoch: the flag array is zero and no
    kernel ever writes it.  The fused LayerNorm's bounded wait (2 s) runs out,
    the kernel records kErrPeerWait and writes nothing, and the stream-ordered
    read of the error word that TensorParallelTransformer.forward makes after
    a peer-path step sees the code.  One GPU; no peer memory is involved (both
    'partials' are local buffers), and the context stays usable."""

    import time

    from solution import _native
    from solution.runtimes.sharded import PeerWaitTimeout, raise_on_error_word

    dev = torch.device("cuda", 0)
    _native.device_error(clear=True)
    rows, cols = 64, 256
    g = torch.Generator().manual_seed(0)
    resid = torch.randn(rows, cols, generator=g).to(dev)
    normed = torch.full((rows, cols), 7.0, dtype=torch.bfloat16, device=dev)
    gamma = torch.ones(cols, device=dev)
    beta = torch.zeros(cols, device=dev)
    partials = [torch.zeros(rows, cols, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    word = torch.zeros(1, dtype=torch.int32).pin_memory()
    start = time.monotonic()
    _native.residual_layer_norm_peer(
        resid, [p.data_ptr() for p in partials], 0, flags.data_ptr(), 1, None, normed, gamma, beta, 1e-5
    )
    _native.device_error_async(word)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - start
    assert int(word.item()) == 0x301
    assert 1.0 < elapsed < 30.0
    assert torch.all(normed == 7.0), "a timed-out wait must not write"
    with pytest.raises(PeerWaitTimeout):
        raise_on_error_word(int(word.item()))
    # Sticky until cleared; afterwards kernels run normally again.
    assert _native.device_error(clear=True) == 0x301
    assert _native.device_error(clear=True) == 0
    flags.fill_(1)
    _native.residual_layer_norm_peer(
        resid, [p.data_ptr() for p in partials], 0, flags.data_ptr(), 1, None, normed, gamma, beta, 1e-5
    )
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    ref = torch.nn.functional.layer_norm(resid, (cols,), eps=1e-5)
    assert torch.allclose(normed.float(), ref, atol=3e-2)
