"""The CPU oracle is pinned to the reference before anything is compared with it.

The golden vectors were produced by the muSPACE reference's own
``multi_scale_deformable_attn_pytorch`` (``tests/golden/gen_golden.py``). Both
oracle restatements must reproduce them: the C oracle (fp32 geometry, double
sums) within float rounding, the torch restatement bit for bit.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_names, load_golden
from oracle import oracle_backward, oracle_forward
from oracle.msda_torch import msda_grid_sample_fwd_bwd

NAMES = golden_names()
OUTPUTS = ("output", "grad_value", "grad_sampling_locations", "grad_attention_weights")


def _oracle_all(g):
    args = (g["value"], g["spatial_shapes"], g["level_start_index"], g["sampling_locations"], g["attention_weights"])
    out = oracle_forward(*args)
    gv, gl, gw = oracle_backward(*args, g["grad_output"])
    return dict(output=out, grad_value=gv, grad_sampling_locations=gl, grad_attention_weights=gw)


def test_golden_manifest_matches_files():
    manifest = json.loads((GOLDEN / "MANIFEST.json").read_text())
    assert sorted(manifest["cases"]) == NAMES
    for name, meta in manifest["cases"].items():
        digest = hashlib.sha256((GOLDEN / f"{name}.npz").read_bytes()).hexdigest()
        assert digest == meta["sha256"], name


@pytest.mark.parametrize("name", NAMES)
def test_c_oracle_matches_reference_golden(name):
    g = load_golden(name)
    got = _oracle_all(g)
    for key in OUTPUTS:
        ref = g[key]
        scale = 1.0 + float(np.abs(ref).max(initial=0.0))
        err = float(np.abs(got[key] - ref).max(initial=0.0))
        # the oracle sums in double, the reference in fp32: a few fp32 ulps of the peak
        assert err <= 2e-6 * scale, f"{name}:{key} max-abs {err:.3g} (scale {scale:.3g})"


@pytest.mark.parametrize("name", NAMES)
def test_torch_restatement_matches_reference_golden_exactly(name):
    g = load_golden(name)
    t = {k: torch.from_numpy(v) for k, v in g.items()}
    out, gv, gl, gw = msda_grid_sample_fwd_bwd(
        t["value"], t["spatial_shapes"], t["sampling_locations"], t["attention_weights"], t["grad_output"]
    )
    for got, key in ((out, "output"), (gv, "grad_value"), (gl, "grad_sampling_locations"), (gw, "grad_attention_weights")):
        np.testing.assert_array_equal(got.numpy(), g[key], err_msg=f"{name}:{key}")


def test_known_answer_2048():
    """Reference test_native_bf16_keeps_sampling_geometry_in_fp32: x = 499.5 between 0 and 4096."""
    g = load_golden("known_2048")
    assert g["output"].item() == 2048.0
    assert _oracle_all(g)["output"].item() == 2048.0


def test_out_of_range_samples_are_zero_with_zero_gradients():
    g = load_golden("all_oob")
    got = _oracle_all(g)
    for key in OUTPUTS:
        assert not np.any(got[key]), key
        assert not np.any(g[key]), key


def test_bf16_quantised_cases_hold_bf16_values():
    for name in ("c0_small_bf16q", "c2_small_bf16q"):
        g = load_golden(name)
        for key in ("value", "sampling_locations", "attention_weights", "grad_output"):
            t = torch.from_numpy(g[key])
            assert torch.equal(t, t.to(torch.bfloat16).float()), f"{name}:{key}"


def test_oracle_grad_value_accumulates_like_the_reference_contract():
    """grad_value is a sum over samples: splitting the queries in two and adding
    the halves gives the whole (the property the query-sharded backward uses)."""
    g = load_golden("c2_small")
    args = (g["value"], g["spatial_shapes"], g["level_start_index"])
    half = g["sampling_locations"].shape[1] // 2
    parts = []
    for sl in (slice(0, half), slice(half, None)):
        gv, _, _ = oracle_backward(
            *args, g["sampling_locations"][:, sl], g["attention_weights"][:, sl], g["grad_output"][:, sl]
        )
        parts.append(gv)
    np.testing.assert_allclose(parts[0] + parts[1], g["grad_value"], rtol=1e-5, atol=1e-5)
