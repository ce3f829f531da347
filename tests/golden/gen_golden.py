"""Generate the MSDA golden vectors from the muSPACE reference itself.

Run once, in a container that has the reference tree (it is read, never copied):

    python tests/golden/gen_golden.py <muSPACE checkout>

For every case below it draws fp32 inputs from a fixed seed, evaluates the
reference's own ``mu_space.ops.multi_scale_deformable_attn.multi_scale_deformable_attn_pytorch``
(``mu_space/ops/multi_scale_deformable_attn.py:26-58``: grid_sample, bilinear,
zero padding, align_corners=False) forward and, through autograd, its backward
for a seeded ``grad_output``, and stores inputs and outputs in ``<case>.npz``.
The ``*_bf16q`` cases hold inputs already rounded to bfloat16 (stored as the
exactly representable fp32 values) with the fp32 answer, the way the
reference's bf16 parity test evaluates its oracle
(``tests/ops/test_multi_scale_deformable_attn.py:378-424``).
``known_2048`` is the reference's known-answer case (same file, 430-468).
"""

from __future__ import annotations

import hashlib
import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _reference_fn(reference_root: str):
    sys.path.insert(0, reference_root)
    module = importlib.import_module("mu_space.ops.multi_scale_deformable_attn")
    origin = Path(module.__file__).resolve()
    if not str(origin).startswith(str(Path(reference_root).resolve())):
        raise SystemExit(f"imported {origin}, not the reference under {reference_root}")
    return module.multi_scale_deformable_attn_pytorch, str(origin)


def _start(shapes):
    sizes = [h * w for h, w in shapes]
    return np.cumsum([0] + sizes[:-1]).astype(np.int64)


def _softmax_weights(gen, shape):
    logits = torch.randn(shape[:3] + (shape[3] * shape[4],), generator=gen)
    return torch.softmax(logits, dim=-1).view(shape)


def _case(name, *, batch, queries, heads, channels, shapes, points, loc="uniform", seed=20260714,
          oob_fraction=0.0, bf16q=False, weights="softmax", value_scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    lin = sum(h * w for h, w in shapes)
    levels = len(shapes)
    value = torch.randn((batch, lin, heads, channels), generator=gen) * value_scale
    lshape = (batch, queries, heads, levels, points, 2)
    if loc == "uniform":
        locations = torch.rand(lshape, generator=gen) * 1.1 - 0.05
    elif loc == "unit":
        locations = torch.rand(lshape, generator=gen)
    elif loc == "clustered":
        centre = torch.rand((batch, queries, heads, 1, 1, 2), generator=gen)
        locations = (centre + torch.randn(lshape, generator=gen) * 0.02).clamp(-0.05, 1.05)
    elif loc == "grid":
        (h, w), = shapes
        rows = torch.arange(h, dtype=torch.float32).repeat_interleave(w)
        cols = torch.arange(w, dtype=torch.float32).repeat(h)
        own = torch.stack(((cols + 0.5) / w, (rows + 0.5) / h), dim=-1).view(1, queries, 1, 1, 1, 2)
        locations = own + torch.randn(lshape, generator=gen) * 0.03
    elif loc == "all_oob":
        locations = torch.full(lshape, -1.0)
    elif loc == "edges":
        # exact level borders and the skip-test boundary: x*W - 0.5 in {-1, -0.5, 0, W-1, W-0.5, W}
        picks = []
        for h, w in shapes:
            xs = torch.tensor([-0.5 / w, 0.0, 0.5 / w, 1.0 - 0.5 / w, 1.0, 1.0 + 0.5 / w, 0.25, 0.75])
            ys = torch.tensor([-0.5 / h, 0.0, 0.5 / h, 1.0 - 0.5 / h, 1.0, 1.0 + 0.5 / h, 0.25, 0.75])
            picks.append((xs, ys))
        locations = torch.empty(lshape)
        for lv, (xs, ys) in enumerate(picks):
            ix = torch.randint(0, 8, lshape[:3] + (points,), generator=gen)
            iy = torch.randint(0, 8, lshape[:3] + (points,), generator=gen)
            locations[:, :, :, lv, :, 0] = xs[ix]
            locations[:, :, :, lv, :, 1] = ys[iy]
    else:
        raise ValueError(loc)
    if oob_fraction:
        far = torch.rand(lshape, generator=gen) * 1.4 - 0.2
        pick = torch.rand(lshape[:-1] + (1,), generator=gen) < oob_fraction
        locations = torch.where(pick, far, locations)
    wshape = (batch, queries, heads, levels, points)
    if weights == "softmax":
        attention = _softmax_weights(gen, wshape)
    elif weights == "rand_softmax_last":
        attention = torch.softmax(torch.rand(wshape, generator=gen), dim=-1)
    else:
        attention = torch.full(wshape, float(weights))
    grad = torch.randn((batch, queries, heads * channels), generator=gen)
    if bf16q:
        value, locations, attention, grad = (
            t.to(torch.bfloat16).float() for t in (value, locations, attention, grad)
        )
    return name, dict(
        value=value,
        spatial_shapes=torch.tensor(shapes, dtype=torch.int64),
        level_start_index=torch.from_numpy(_start(shapes)),
        sampling_locations=locations,
        attention_weights=attention,
        grad_output=grad,
    )


def cases():
    yield _case("ref_fixture_a", batch=1, queries=5, heads=2, channels=3, shapes=((2, 2),), points=4,
                loc="unit", weights="rand_softmax_last")
    yield _case("ref_fixture_b", batch=2, queries=3, heads=4, channels=2, shapes=((1, 3), (2, 1)), points=2,
                loc="unit", weights="rand_softmax_last")
    yield _case("ref_fixture_c", batch=1, queries=7, heads=1, channels=8, shapes=((1, 1), (1, 2), (2, 2)),
                points=3, loc="unit", weights="rand_softmax_last")
    yield _case("all_oob", batch=1, queries=2, heads=1, channels=2, shapes=((2, 2),), points=2, loc="all_oob")
    yield _case("c0_small", batch=1, queries=64, heads=8, channels=32,
                shapes=((16, 16), (8, 8), (4, 4), (2, 2)), points=4, seed=2333)
    yield _case("c1_small", batch=2, queries=40, heads=4, channels=32,
                shapes=((10, 17), (5, 9), (3, 5), (2, 3)), points=4, seed=2335)
    yield _case("c2_small", batch=2, queries=24, heads=8, channels=32,
                shapes=((15, 26), (8, 13), (4, 7), (2, 4)), points=8, loc="clustered", seed=2337)
    yield _case("c3_small", batch=2, queries=256, heads=4, channels=32, shapes=((16, 16),), points=4,
                loc="grid", seed=2339)
    yield _case("c4_small_oob", batch=2, queries=24, heads=2, channels=32,
                shapes=((15, 26), (8, 13), (4, 7), (2, 4)), points=8, loc="clustered", oob_fraction=0.1,
                seed=2341)
    yield _case("c0_small_bf16q", batch=1, queries=64, heads=8, channels=32,
                shapes=((16, 16), (8, 8), (4, 4), (2, 2)), points=4, seed=2343, bf16q=True)
    yield _case("c2_small_bf16q", batch=1, queries=24, heads=8, channels=32,
                shapes=((15, 26), (8, 13), (4, 7), (2, 4)), points=8, loc="clustered", seed=2345, bf16q=True)
    yield _case("edges", batch=2, queries=16, heads=4, channels=32, shapes=((5, 7), (3, 4), (1, 1)), points=4,
                loc="edges", seed=2347)
    yield _case("ragged_d16", batch=2, queries=9, heads=3, channels=16, shapes=((3, 5), (2, 2)), points=3,
                seed=2349)
    yield _case("wide_d64", batch=1, queries=12, heads=2, channels=64, shapes=((6, 7),), points=2, seed=2351)
    yield _case("odd_d5", batch=2, queries=6, heads=3, channels=5, shapes=((4, 3), (2, 2)), points=3, seed=2353)
    # the reference known answer: value pixels 500.. hold 4096, the query samples x = 499.5
    width = 1000
    value = torch.zeros(1, width, 1, 1)
    value[:, width // 2 :] = 4096.0
    yield "known_2048", dict(
        value=value,
        spatial_shapes=torch.tensor([[1, width]], dtype=torch.int64),
        level_start_index=torch.zeros(1, dtype=torch.int64),
        sampling_locations=torch.full((1, 1, 1, 1, 1, 2), 0.5),
        attention_weights=torch.ones(1, 1, 1, 1, 1),
        grad_output=torch.ones(1, 1, 1),
    )


def main(reference_root: str) -> None:
    fn, origin = _reference_fn(reference_root)
    manifest = {"generator": "tests/golden/gen_golden.py", "reference_function": origin.split("/mu_space/", 1)[-1],
                "torch": torch.__version__, "cases": {}}
    for name, t in cases():
        value = t["value"].clone().requires_grad_(True)
        loc = t["sampling_locations"].clone().requires_grad_(True)
        weight = t["attention_weights"].clone().requires_grad_(True)
        out = fn(value, t["spatial_shapes"], loc, weight)
        out.backward(t["grad_output"])
        arrays = {k: v.numpy() for k, v in t.items()}
        arrays.update(
            output=out.detach().numpy(),
            grad_value=value.grad.numpy(),
            grad_sampling_locations=loc.grad.numpy(),
            grad_attention_weights=weight.grad.numpy(),
        )
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        manifest["cases"][name] = {
            "sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
            "value_shape": list(arrays["value"].shape),
            "loc_shape": list(arrays["sampling_locations"].shape),
        }
        print(f"{name}: out {tuple(out.shape)} |out|max {out.abs().max().item():.4g}")
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: gen_golden.py <muSPACE checkout>")
    main(sys.argv[1])
