"""Host-side logic that needs no GPU: weight mapping, the no-fallback rule,
the streamed executor, the deployment registry and the C ABI surface."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
from conftest import PACKAGE_DIR, REPO

from deployment.environment import EnvironmentFingerprint, ImplementationScope, stable_digest
from deployment.registry import (
    ShapeFingerprint,
    iter_deployed_configs,
    publish_deployed_config,
    resolve_deployed_config,
)
from oracle import OfficialConfig, official_state_dict
from solution import _native
from solution.config import RuntimeBackend, default_program, default_schedule, ConfigSpec, portable_config
from solution.plan_builder import ConfigRejectedError
from solution.shape14.defaults import default_streamed_config, is_streamed_shape
from solution.shape14.executor import execute_streamed
from solution.transformer import UserOptimizedTransformer, copy_model_weights

CFG = SimpleNamespace(batch_size=2, seq_len=16, d_model=128, num_heads=2, ffn_dim=256, num_layers=2, causal=True)


def _official_state() -> dict[str, torch.Tensor]:
    return official_state_dict(
        OfficialConfig(CFG.batch_size, CFG.seq_len, CFG.d_model, CFG.num_heads, CFG.ffn_dim, CFG.num_layers), 0
    )


def test_copy_model_weights_packs_qkv_rows() -> None:
    state = _official_state()
    model = UserOptimizedTransformer(CFG)
    copy_model_weights(state, model)
    packed = model.layers[1].attention.qkv_proj.weight.detach()
    d = CFG.d_model
    assert torch.equal(packed[:d], state["layers.1.attention.q_proj.weight"])
    assert torch.equal(packed[d : 2 * d], state["layers.1.attention.k_proj.weight"])
    assert torch.equal(packed[2 * d :], state["layers.1.attention.v_proj.weight"])
    bias = model.layers[0].attention.qkv_proj.bias.detach()
    assert torch.equal(bias[d : 2 * d], state["layers.0.attention.k_proj.bias"])
    assert torch.equal(model.final_norm.weight.detach(), state["final_norm.weight"])


def test_copy_model_weights_strict_failures() -> None:
    state = _official_state()
    del state["layers.0.ffn_in.bias"]
    model = UserOptimizedTransformer(CFG)
    with pytest.raises(RuntimeError, match="strict weight mapping failed"):
        copy_model_weights(state, model)
    with pytest.warns(RuntimeWarning):
        copy_model_weights(state, model, strict=False)


def test_weight_load_clears_shadows() -> None:
    model = UserOptimizedTransformer(CFG)
    model._materialize_shadow_weights()
    assert model.layers[0].ffn_in._bf16_shadow_weight is not None
    copy_model_weights(_official_state(), model)
    assert model.layers[0].ffn_in._bf16_shadow_weight is None
    model._materialize_shadow_weights()
    model.load_state_dict(model.state_dict())
    assert model.layers[0].ffn_in._bf16_shadow_weight is None


def test_no_cpu_fallback() -> None:
    model = UserOptimizedTransformer(CFG).eval()
    x = torch.randn(2, 16, 128)
    with torch.inference_mode(), pytest.raises(ConfigRejectedError) as info:
        model(x)
    codes = {v.code for v in info.value.rejection.violations}
    assert "requires_cuda" in codes


def test_configure_execution_is_strict() -> None:
    model = UserOptimizedTransformer(CFG).eval()
    with pytest.raises(ConfigRejectedError):
        model.configure_execution(config=portable_config())
    with pytest.raises(TypeError):
        model.configure_execution(config={"runtime": "eager"})  # type: ignore[arg-type]


def test_streamed_executor_order_and_slices() -> None:
    calls: list[tuple[int, int, bool]] = []

    outputs: list[int] = []

    def forward(chunk: torch.Tensor, mask: torch.Tensor | None, *, out: torch.Tensor) -> torch.Tensor:
        # Each microbatch writes its own rows of the one output, in place.
        calls.append((int(chunk[0, 0, 0].item()), chunk.shape[0], mask is not None))
        outputs.append(out.data_ptr())
        torch.mul(chunk, 2, out=out)
        return out

    x = torch.arange(6, dtype=torch.float32).view(6, 1, 1).expand(6, 2, 3).contiguous()
    mask = torch.ones(6, 2, dtype=torch.bool)
    out = execute_streamed(x, mask, microbatch_size=2, forward_chunk=forward)
    assert calls == [(0, 2, True), (2, 2, True), (4, 2, True)]
    assert torch.equal(out, x * 2)
    row = out[0].numel() * out.element_size()
    assert outputs == [out.data_ptr(), out.data_ptr() + 2 * row, out.data_ptr() + 4 * row]
    given = torch.empty_like(x)
    assert execute_streamed(x, None, microbatch_size=3, forward_chunk=forward) is not given
    assert execute_streamed(x, None, microbatch_size=3, forward_chunk=forward, output=given) is given
    with pytest.raises(ValueError):
        execute_streamed(x, None, microbatch_size=4, forward_chunk=forward)
    with pytest.raises(ValueError):
        execute_streamed(x, None, microbatch_size=0, forward_chunk=forward)
    with pytest.raises(ValueError):
        execute_streamed(x, mask[:3], microbatch_size=2, forward_chunk=forward)


def test_streamed_defaults() -> None:
    assert is_streamed_shape(100000, 1024)
    assert not is_streamed_shape(16384, 2048)
    assert default_streamed_config(32).schedule.microbatch_size == 4
    assert default_streamed_config(6).schedule.microbatch_size == 3
    assert default_streamed_config(1).schedule.microbatch_size == 1


def _hardware(driver: str = "580.159") -> EnvironmentFingerprint:
    return EnvironmentFingerprint(
        device_name="NVIDIA B200",
        compute_capability="10.0",
        driver_version=driver,
        torch_version="2.11.0+cu128",
        cuda_runtime_version="12.8",
        kernel_library_version="abi-1",
        solution_implementation_digest="abc",
        scope=ImplementationScope.RESIDENT,
    )


def test_registry_round_trip(tmp_path: Path) -> None:
    path = tmp_path / "deployed.json"
    shape = ShapeFingerprint(8, 1024, 16, 2048, 2, True, 4096, "float32", 0.0, 1.0)
    cfg = ConfigSpec(program=default_program(), schedule=default_schedule(RuntimeBackend.CUDA_GRAPH))
    assert resolve_deployed_config(hardware=_hardware(), shape=shape, path=path) is None
    publish_deployed_config(hardware=_hardware(), shape=shape, config=cfg, path=path)
    assert resolve_deployed_config(hardware=_hardware(), shape=shape, path=path) == cfg
    # The source digest is not part of the measurement identity.
    other_digest = EnvironmentFingerprint.from_dict({**_hardware().to_dict(), "solution_implementation_digest": "zzz"})
    assert resolve_deployed_config(hardware=other_digest, shape=shape, path=path) == cfg
    assert resolve_deployed_config(hardware=_hardware("999.0"), shape=shape, path=path) is None
    pairs = iter_deployed_configs(hardware=_hardware(), path=path)
    assert pairs == ((shape, cfg),)
    publish_deployed_config(hardware=_hardware(), shape=shape, config=portable_config(), path=path)
    assert resolve_deployed_config(hardware=_hardware(), shape=shape, path=path) == portable_config()
    assert len(iter_deployed_configs(hardware=_hardware(), path=path)) == 1


def test_registry_keeps_entry_order_and_sees_rewritten_files(tmp_path: Path) -> None:
    """A replaced entry keeps its place, new shapes go last, a table of another
    schema is started afresh, and the cached index follows the file when it
    is rewritten behind the registry's back."""

    import json

    path = tmp_path / "deployed.json"
    shapes = [ShapeFingerprint(b, 1024, 16, 2048, 2, True, 4096, "float32", 0.0, 1.0) for b in (1, 2, 4)]
    graph = ConfigSpec(program=default_program(), schedule=default_schedule(RuntimeBackend.CUDA_GRAPH))
    for shape in shapes:
        publish_deployed_config(hardware=_hardware(), shape=shape, config=portable_config(), path=path)
    publish_deployed_config(hardware=_hardware(), shape=shapes[1], config=graph, path=path)
    pairs = iter_deployed_configs(hardware=_hardware(), path=path)
    assert [shape for shape, _ in pairs] == shapes
    assert [cfg for _, cfg in pairs] == [portable_config(), graph, portable_config()]
    assert not list(tmp_path.glob("*.tmp"))  # the atomic write left no temporary behind

    document = json.loads(path.read_text())
    document["bundles"][0]["entries"] = document["bundles"][0]["entries"][:1]
    path.write_text(json.dumps(document, indent=1))
    assert resolve_deployed_config(hardware=_hardware(), shape=shapes[1], path=path) is None
    assert resolve_deployed_config(hardware=_hardware(), shape=shapes[0], path=path) == portable_config()

    path.write_text(json.dumps({"schema_version": 3, "bundles": document["bundles"]}))
    assert iter_deployed_configs(hardware=_hardware(), path=path) == ()
    publish_deployed_config(hardware=_hardware(), shape=shapes[2], config=graph, path=path)
    assert json.loads(path.read_text())["schema_version"] == 4
    assert iter_deployed_configs(hardware=_hardware(), path=path) == ((shapes[2], graph),)


def test_fingerprint_round_trip() -> None:
    hw = _hardware()
    assert EnvironmentFingerprint.from_dict(hw.to_dict()) == hw
    assert hw.identity == stable_digest(hw.to_dict())
    with pytest.raises(ValueError):
        EnvironmentFingerprint.from_dict({**hw.to_dict(), "device_name": ""})


def test_shipped_registry_parses() -> None:
    import json

    document = json.loads((PACKAGE_DIR / "deployment" / "deployed_configs.json").read_text())
    assert document["schema_version"] == 4
    for bundle in document["bundles"]:
        EnvironmentFingerprint.from_dict(bundle["hardware"])
        for entry in bundle["entries"]:
            ShapeFingerprint.from_dict(entry["shape"])
            ConfigSpec.from_dict(entry["config"])


def test_every_deployed_entry_compiles_for_its_shape() -> None:
    """A deployed config the plan builder rejects would silently fall back to
    the default program on the device it was measured on."""
    import json

    from solution.plan import ExecutionContext
    from solution.plan_builder import HardwareCapabilities, PlanBuilder

    document = json.loads((PACKAGE_DIR / "deployment" / "deployed_configs.json").read_text())
    for bundle in document["bundles"]:
        for entry in bundle["entries"]:
            shape = ShapeFingerprint.from_dict(entry["shape"])
            config = ConfigSpec.from_dict(entry["config"])
            context = ExecutionContext(
                batch_size=shape.batch_size, seq_len=shape.seq_len, d_model=shape.qkv_dim,
                num_heads=shape.heads, causal=shape.causal, device=torch.device("cuda", 0),
                dtype=getattr(torch, shape.dtype), training=False, grad_enabled=False,
                input_contiguous=True, has_valid_token_mask=False, mask_compatible=True,
                ffn_dim=shape.ffn_dim, num_layers=shape.layers,
            )
            result = PlanBuilder().evaluate(config, context, HardwareCapabilities.sm100())
            assert result.accepted, (shape, [v.message for v in result.violations])


# ------------------------------------------------------------------ C ABI

def _header_functions() -> list[str]:
    text = (REPO / "include" / "b200tx.h").read_text()
    return sorted(set(re.findall(r"\b(b200tx_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol() -> None:
    lib = _native.load()
    names = _header_functions()
    assert {"b200tx_linear", "b200tx_attention", "b200tx_residual_layer_norm"} <= set(names)
    raw = ctypes.CDLL(str(_native.library_path()))
    for name in names:
        assert hasattr(raw, name), name
    assert lib.b200tx_abi_version() == _native.ABI_VERSION


def test_ctypes_declarations_match_the_header_arity() -> None:
    """Every declared entry point is bound with as many arguments as the header
    gives it (a missing or extra ctypes argument would shift every later one)."""

    text = (REPO / "include" / "b200tx.h").read_text()
    lib = _native.load()
    declared = re.findall(r"\bint\s+(b200tx_[a-z0-9_]+)\s*\(([^;]*?)\);", text, flags=re.S)
    assert len(declared) >= 15
    for name, params in declared:
        params = params.strip()
        arity = 0 if params in ("", "void") else params.count(",") + 1
        argtypes = getattr(lib, name).argtypes
        assert argtypes is not None, name
        assert len(argtypes) == arity, (name, len(argtypes), arity)


def test_argument_errors_are_reported_before_any_launch() -> None:
    lib = _native.load()
    rc = lib.b200tx_linear(None, None, None, None, 1, 128, 256, 64, 0, None)
    assert rc == -1
    assert b"null" in lib.b200tx_last_error()
    rc = lib.b200tx_attention(None, None, 1, 128, 1, 64, ctypes.c_float(0.125), 1, None)
    assert rc == -1
    buf = ctypes.create_string_buffer(64)
    rc = lib.b200tx_attention(buf, buf, 1, 128, 1, 128, ctypes.c_float(0.125), 1, None)
    assert rc == -2 and b"head_dim" in lib.b200tx_last_error()
    rc = lib.b200tx_attention_ex(buf, buf, 1, 128, 1, 64, ctypes.c_float(0.125), 1, 7, None)
    assert rc == -1 and b"variant" in lib.b200tx_last_error()
    rc = lib.b200tx_linear(buf, buf, None, buf, 1, 16, 20, 64, 0, None)
    assert rc == -2 and b"multiples of 8" in lib.b200tx_last_error()
    rc = lib.b200tx_residual_layer_norm(buf, 5, None, 0, None, buf, 1, buf, buf, 4, 8, ctypes.c_float(1e-5), None)
    assert rc == -1 and b"in_dtype" in lib.b200tx_last_error()
    rc = lib.b200tx_linear_ex(buf, buf, None, buf, 1, 16, 16, 64, 0, 9, None)
    assert rc == -1 and b"variant" in lib.b200tx_last_error()
    rc = lib.b200tx_attention_generic(buf, None, buf, 1, 16, 1, 48, ctypes.c_float(0.125), 1, None)
    assert rc == -2 and b"head_dim" in lib.b200tx_last_error()
    rc = lib.b200tx_attention_mma(buf, None, buf, 1, 16, 1, 256, ctypes.c_float(0.125), 1, None)
    assert rc == -2 and b"head_dim" in lib.b200tx_last_error()
    rc = lib.b200tx_attention_mma(None, None, buf, 1, 16, 1, 32, ctypes.c_float(0.125), 1, None)
    assert rc == -1 and b"null" in lib.b200tx_last_error()
    rc = lib.b200tx_attention_masked(buf, None, buf, 1, 16, 1, 64, ctypes.c_float(0.125), 1, 2, None)
    assert rc == -1 and b"key_valid" in lib.b200tx_last_error()
    slots = (ctypes.c_void_p * 1)(None)
    rc = lib.b200tx_peer_signal(slots, 0, 1, None)
    assert rc == -1 and b"count" in lib.b200tx_last_error()
    parts = (ctypes.c_void_p * 2)(ctypes.addressof(buf), ctypes.addressof(buf))
    rc = lib.b200tx_residual_layer_norm_peer(
        buf, parts, 2, 2, buf, 1, None, buf, 1, buf, buf, None, 0, 4, 128, ctypes.c_float(1e-5), None
    )
    assert rc == -1 and b"self" in lib.b200tx_last_error()
    rc = lib.b200tx_residual_layer_norm_peer(
        buf, parts, 2, 0, buf, 1, None, buf, 1, buf, buf, None, 0, 4, 100, ctypes.c_float(1e-5), None
    )
    assert rc == -2 and b"cols" in lib.b200tx_last_error()


def test_kernel_wrappers_refuse_cpu_tensors() -> None:
    from solution.kernels import (
        can_use_sm100_flash_attention,
        can_use_sm100_linear,
        can_use_sm100_residual_layer_norm,
        sm100_linear,
    )

    a = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, dtype=torch.bfloat16)
    assert not can_use_sm100_linear(a, w, None)
    assert not can_use_sm100_flash_attention(torch.zeros(1, 4, 192, dtype=torch.bfloat16), 1)
    assert not can_use_sm100_residual_layer_norm(torch.zeros(4, 64), None, torch.nn.LayerNorm(64))
    with pytest.raises(RuntimeError, match="ineligible"):
        sm100_linear(a, w, None)


# ------------------------------------------------------- reference install

def test_build_restores_the_reference_install_only_when_it_can(tmp_path: Path, monkeypatch) -> None:  # noqa: ANN001
    """__graft_entry__._install_reference: nothing to do when baseline/_ref is
    there, or when BASELINE.json names no reference checkout that exists;
    otherwise it runs baseline/install_reference.py with that checkout.  It
    never raises."""

    import subprocess
    import sys

    sys.path.insert(0, str(REPO))
    import __graft_entry__ as entry

    calls: list[list[str]] = []

    def fake_run(cmd, **kwargs):  # noqa: ANN001, ANN003
        calls.append(cmd)
        return SimpleNamespace(returncode=0, stdout="", stderr="")

    monkeypatch.setattr(subprocess, "run", fake_run)
    monkeypatch.setattr(entry, "REPO", tmp_path)

    (tmp_path / "BASELINE.json").write_text('{"metric": "m"}')  # no reference_path
    entry._install_reference()
    checkout = tmp_path / "ref"
    (tmp_path / "BASELINE.json").write_text('{"reference_path": "%s"}' % checkout)
    entry._install_reference()  # the checkout is absent
    assert calls == []

    (checkout / "official").mkdir(parents=True)
    entry._install_reference()
    assert len(calls) == 1 and calls[0][-1] == str(checkout) and calls[0][-2].endswith("install_reference.py")

    installed = tmp_path / "baseline" / "_ref" / "official"
    installed.mkdir(parents=True)
    (installed / "torch_transformer_benchmark.py").write_text("")
    entry._install_reference()
    assert len(calls) == 1
