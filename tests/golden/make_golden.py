"""Generate tests/golden/*.npz from the reference implementation itself.

Run in the development container, where the reference sources are readable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's official harness (``official.torch_transformer_benchmark``:
``TransformerConfig``, ``BaselineTransformer``, ``generate_random_case``) and the
reference's own ``solution`` package (``UserOptimizedTransformer`` with its
portable program + ``copy_model_weights``), runs them on CPU in fp32, and
stores inputs, masks, outputs and weight checksums.  The fixtures travel with
the repository; nothing at test time reads the reference.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

CASES = [
    # name, (B, S, D, H, F, L, causal), input seed, padding ratio, store input
    ("c1_official", (2, 128, 256, 4, 1024, 2, True), 0, 0.0, False),
    ("tiny", (1, 16, 64, 1, 256, 1, True), 5, 0.0, True),
    ("ragged_s300", (1, 300, 128, 2, 256, 1, True), 6, 0.0, False),
    ("noncausal", (2, 64, 128, 2, 256, 2, False), 7, 0.0, False),
    ("masked", (2, 96, 128, 2, 256, 2, True), 8, 0.3, True),
    ("s1", (3, 1, 128, 2, 512, 2, True), 9, 0.0, False),
]


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    sys.path.insert(1, str(REPO))
    from official import torch_transformer_benchmark as official  # noqa: PLC0415
    from solution import UserOptimizedTransformer, copy_model_weights  # noqa: PLC0415

    from oracle.weights import state_checksum  # noqa: PLC0415

    torch.set_num_threads(8)
    for name, (b, s, d, h, f, layers, causal), seed, padding, store_input in CASES:
        cfg = official.TransformerConfig(
            batch_size=b, seq_len=s, d_model=d, num_heads=h, ffn_dim=f, num_layers=layers, causal=causal
        )
        torch.manual_seed(0)
        baseline = official.BaselineTransformer(cfg).eval()
        x, mask = official.generate_random_case(
            cfg, torch.device("cpu"), torch.float32, seed, padding, 1.0
        )
        run_mask = mask if padding > 0 else None
        with torch.inference_mode():
            y_official = baseline(x, run_mask)
            y_all_true = baseline(x, mask)  # the harness always passes its mask
        optimized = UserOptimizedTransformer(cfg).eval()
        copy_model_weights(baseline, optimized)
        with torch.inference_mode():
            y_solution = optimized(x, mask)
        payload = {
            "config": np.array([b, s, d, h, f, layers, int(causal)], dtype=np.int64),
            "input_seed": np.array(seed, dtype=np.int64),
            "padding_ratio": np.array(padding, dtype=np.float64),
            "weight_checksum": np.array(state_checksum(baseline.state_dict()), dtype=np.float64),
            "input_checksum": np.array(float(x.double().sum()), dtype=np.float64),
            "input_abs_checksum": np.array(float(x.double().abs().sum()), dtype=np.float64),
            "output": y_official.numpy().astype(np.float32),
            "solution_max_abs_diff": np.array(
                float((y_solution - y_official).abs().max()), dtype=np.float64
            ),
            "all_true_mask_max_abs_diff": np.array(
                float((y_all_true - y_official).abs().max()), dtype=np.float64
            ),
            "mask": mask.numpy(),
        }
        if store_input:
            payload["input"] = x.numpy().astype(np.float32)
        np.savez_compressed(HERE / f"{name}.npz", **payload)
        print(
            f"{name}: out {tuple(y_official.shape)} solution-vs-official "
            f"{payload['solution_max_abs_diff']:.3e}"
        )


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py REFERENCE_ROOT")
    main(sys.argv[1])
