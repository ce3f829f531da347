"""Seeded synthetic MSDA workloads: the benchmark cases and the parity-test shapes.

No dataset is used anywhere: every tensor is drawn from a fixed seed with the
shapes and value distributions of the workload it stands in for.

``CONFIGS`` holds the five BEVFormer / Deformable-DETR configurations the B200
build is measured on (c0..c4) and ``bevformer-1l``, the reference's own
published benchmark case (``benchmarks/msda/msda_single_level_case.py:41-82`` in
the muSPACE tree: seed 2333 forward / 2334 backward, value scaled by 1.38 /
1.25, locations ``U * 1.035 - 0.0175``, weights 0.25, ``grad_output`` scaled by
6.3e-6 with stride ``(1, 512, 2)``).

Layouts follow the operator: value ``(B, Lin, Hh, D)``, sampling_locations
``(B, Lq, Hh, L, P, 2)`` with the last dim ``(x, y)``, attention_weights
``(B, Lq, Hh, L, P)``, output / grad_output ``(B, Lq, Hh*D)``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import torch

DEFAULT_SEED = 2333


@dataclass(frozen=True)
class MSDAConfig:
    name: str
    batch: int
    shapes: tuple[tuple[int, int], ...]
    queries: int
    points: int
    heads: int = 8
    channels: int = 32
    locations: str = "uniform"  # uniform | clustered | clustered_oob | grid | bevformer
    description: str = ""
    dtypes: tuple[str, ...] = ("float32",)
    scope: str = "fwd+bwd"
    extra: dict = field(default_factory=dict)

    @property
    def levels(self) -> int:
        return len(self.shapes)

    @property
    def spatial_size(self) -> int:
        return sum(h * w for h, w in self.shapes)

    def with_(self, **kwargs) -> "MSDAConfig":
        return replace(self, **kwargs)


DETR_SHAPES = ((100, 167), (50, 84), (25, 42), (13, 21))
BEVFORMER_SCA_SHAPES = ((116, 200), (58, 100), (29, 50), (15, 25))

CONFIGS: dict[str, MSDAConfig] = {
    "c0": MSDAConfig(
        "c0",
        batch=1,
        shapes=((32, 32), (16, 16), (8, 8), (4, 4)),
        queries=1360,
        points=4,
        description="CPU-runnable encoder self-attention, Len_in=Lq=1360",
    ),
    "c1": MSDAConfig(
        "c1",
        batch=2,
        shapes=DETR_SHAPES,
        queries=22223,
        points=4,
        dtypes=("float32", "bfloat16"),
        description="Deformable-DETR encoder, Len_in=Lq=22223",
    ),
    "c2": MSDAConfig(
        "c2",
        batch=6,
        shapes=BEVFORMER_SCA_SHAPES,
        queries=10000,
        points=8,
        locations="clustered",
        dtypes=("bfloat16",),
        description="BEVFormer-base spatial cross-attention, 6 cameras folded into batch",
    ),
    "c3": MSDAConfig(
        "c3",
        batch=2,
        shapes=((200, 200),),
        queries=40000,
        points=4,
        locations="grid",
        dtypes=("bfloat16",),
        description="BEVFormer temporal self-attention, current+previous BEV in batch",
    ),
    "c4": MSDAConfig(
        "c4",
        batch=48,
        shapes=BEVFORMER_SCA_SHAPES,
        queries=10000,
        points=8,
        locations="clustered_oob",
        dtypes=("bfloat16",),
        description="BEVFormer-base SCA at batch 8 x 6 cameras (bs_eff=48), 10% OOB locations",
    ),
    "bevformer-1l": MSDAConfig(
        "bevformer-1l",
        batch=2,
        shapes=((200, 200),),
        queries=40000,
        points=4,
        locations="bevformer",
        dtypes=("float32", "bfloat16"),
        description="reference benchmark case: BEVFormer single-level MSDA",
    ),
}


def level_start_index(shapes) -> torch.Tensor:
    sizes = torch.tensor([h * w for h, w in shapes], dtype=torch.int64)
    return torch.cat([sizes.new_zeros(1), sizes.cumsum(0)[:-1]])


def _locations(cfg: MSDAConfig, gen: torch.Generator, device) -> torch.Tensor:
    b, q, hh, lv, p = cfg.batch, cfg.queries, cfg.heads, cfg.levels, cfg.points
    shape = (b, q, hh, lv, p, 2)
    kind = cfg.locations
    if kind == "uniform":
        return torch.rand(shape, generator=gen, device=device) * 1.1 - 0.05
    if kind in ("clustered", "clustered_oob"):
        centre = torch.rand((b, q, hh, 1, 1, 2), generator=gen, device=device)
        jitter = torch.randn(shape, generator=gen, device=device) * 0.02
        loc = (centre + jitter).clamp_(-0.05, 1.05)
        if kind == "clustered_oob":
            far = torch.rand(shape, generator=gen, device=device) * 1.4 - 0.2
            pick = torch.rand((b, q, hh, lv, p, 1), generator=gen, device=device) < 0.1
            loc = torch.where(pick, far, loc)
        return loc
    if kind == "grid":
        (h, w), = cfg.shapes
        if q != h * w:
            raise ValueError("grid locations need Lq == H*W")
        rows = torch.arange(h, device=device, dtype=torch.float32).repeat_interleave(w)
        cols = torch.arange(w, device=device, dtype=torch.float32).repeat(h)
        own = torch.stack(((cols + 0.5) / w, (rows + 0.5) / h), dim=-1)  # (Lq, 2) as (x, y)
        own = own.view(1, q, 1, 1, 1, 2)
        return own + torch.randn(shape, generator=gen, device=device) * 0.03
    if kind == "bevformer":
        return torch.rand(shape, generator=gen, device=device).mul_(1.035).add_(-0.0175)
    raise ValueError(f"unknown location distribution {kind!r}")


def _weights(cfg: MSDAConfig, gen: torch.Generator, device) -> torch.Tensor:
    b, q, hh, lv, p = cfg.batch, cfg.queries, cfg.heads, cfg.levels, cfg.points
    if cfg.locations == "bevformer":
        return torch.full((b, q, hh, lv, p), 0.25, device=device)
    logits = torch.randn((b, q, hh, lv * p), generator=gen, device=device)
    return torch.softmax(logits, dim=-1).view(b, q, hh, lv, p)


def make_inputs(
    cfg: MSDAConfig,
    *,
    dtype: torch.dtype = torch.float32,
    seed: int = DEFAULT_SEED,
    device: str | torch.device = "cpu",
    with_grad: bool = True,
) -> dict[str, torch.Tensor]:
    """Draw one case in fp32 on ``device`` from ``seed``, then narrow to ``dtype``.

    The forward tensors come from ``seed`` and ``grad_output`` from ``seed + 1``
    (the reference harness convention). Drawing in fp32 first means a GPU run
    and the CPU oracle see identical quantised inputs when both draw on CPU.
    """
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    scale = 1.38 if cfg.locations == "bevformer" else 1.0
    value = torch.randn(
        (cfg.batch, cfg.spatial_size, cfg.heads, cfg.channels), generator=gen, device=device
    ) * scale
    loc = _locations(cfg, gen, device)
    weight = _weights(cfg, gen, device)
    out = {
        "value": value.to(dtype),
        "spatial_shapes": torch.tensor(cfg.shapes, dtype=torch.int64, device=device),
        "level_start_index": level_start_index(cfg.shapes).to(device),
        "sampling_locations": loc.to(dtype),
        "attention_weights": weight.to(dtype),
    }
    if with_grad:
        ggen = torch.Generator(device=device).manual_seed(seed + 1)
        if cfg.locations == "bevformer":
            # (Lq, Hh*D, B) permuted to (B, Lq, Hh*D): stride (1, 512, 2) for B=2
            raw = torch.randn(
                (cfg.queries, cfg.heads * cfg.channels, cfg.batch), generator=ggen, device=device
            )
            grad = raw.permute(2, 0, 1).mul(6.3e-6)
        else:
            grad = torch.randn(
                (cfg.batch, cfg.queries, cfg.heads * cfg.channels), generator=ggen, device=device
            )
        out["grad_output"] = grad.to(dtype)
    return out


def compulsory_bytes(cfg: MSDAConfig, dtype: torch.dtype, scope: str = "fwd+bwd") -> dict[str, int]:
    """Algorithmic HBM bytes of one call (the roofline numerator).

    fwd = value + locations + weights + output in the storage dtype.
    bwd = value + locations + weights + grad_output reads in the storage dtype,
          plus fp32 writes of grad_value, grad_locations and grad_weights.
    Memsets, ``.contiguous()`` copies and L2 re-gathers are not counted.
    """
    es = torch.empty((), dtype=dtype).element_size()
    b, q, hh, d = cfg.batch, cfg.queries, cfg.heads, cfg.channels
    n_value = b * cfg.spatial_size * hh * d
    n_w = b * q * hh * cfg.levels * cfg.points
    n_loc = 2 * n_w
    n_out = b * q * hh * d
    fwd = (n_value + n_loc + n_w + n_out) * es
    bwd = (n_value + n_loc + n_w + n_out) * es + (n_value + n_loc + n_w) * 4
    if scope == "fwd":
        return {"fwd": fwd, "bwd": 0, "total": fwd}
    return {"fwd": fwd, "bwd": bwd, "total": fwd + bwd}


# ---------------------------------------------------------------------------
# workloads of the ops next to MSDA (deformable aggregation, FlashSCA, the
# fused SCA scatter): seeded synthetic tensors with the reference's shapes
# ---------------------------------------------------------------------------
SPARSEDRIVE_SHAPES = ((64, 176), (32, 88), (16, 44), (8, 22))


def deformable_aggregation_inputs(device, *, batch=8, anchors=900, pts=13, cams=6, channels=256, groups=8,
                                  active=0.40, seed=0):
    """The reference test's SparseDrive production shapes
    (``tests/ops/test_deformable_aggregation.py:29-79`` in the muSPACE tree):
    mc_ms_feat [B, 6 * 14960, 256], 6 cameras x 4 scales
    [(64,176),(32,88),(16,44),(8,22)], 900 anchors x 13 points, 8 groups; a
    fraction ``active`` of the (pt, cam) pairs lies inside the image, the rest
    at N(0, 10) (outside); weights U(0, 0.004). Returns the five inputs and a
    N(0, 1) grad_output."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    sizes = [h * w for h, w in SPARSEDRIVE_SHAPES]
    spatial = torch.tensor([list(map(list, SPARSEDRIVE_SHAPES))] * cams, dtype=torch.int32)
    start = torch.tensor([[sum(sizes) * c + sum(sizes[:s]) for s in range(len(sizes))] for c in range(cams)],
                         dtype=torch.int32)
    mc = torch.randn(batch, sum(sizes) * cams, channels, generator=g)
    pshape = (batch, anchors, pts, cams)
    inside_mask = torch.rand(*pshape, generator=g) < active
    outside = torch.randn(*pshape, 2, generator=g) * 10.0
    inside = torch.rand(*pshape, 2, generator=g) * 0.98 + 0.01
    loc = torch.where(inside_mask.unsqueeze(-1), inside, outside)
    weights = torch.rand(*pshape, len(sizes), groups, generator=g) * 0.004
    grad = torch.randn(batch, anchors, channels, generator=g)
    return [x.to(device) for x in (mc, spatial, start, loc, weights)], grad.to(device)


def pinhole_cameras(batch, cams, image_hw, gen, height=1.5):
    """Cameras at (0, 0, height) looking outwards at evenly spread yaws (with a
    little seeded jitter): 3x4 projection matrices [B, cams, 3, 4]."""
    img_h, img_w = image_hw
    mats = torch.zeros(batch, cams, 3, 4)
    for b in range(batch):
        for c in range(cams):
            yaw = 2 * math.pi * c / cams + float(torch.randn((), generator=gen)) * 0.05
            rot = torch.tensor([[math.sin(yaw), -math.cos(yaw), 0.0], [0.0, 0.0, -1.0],
                                [math.cos(yaw), math.sin(yaw), 0.0]])
            k = torch.tensor([[img_w * 0.5, 0.0, img_w * 0.5], [0.0, img_h * 0.5, img_h * 0.5], [0.0, 0.0, 1.0]])
            mats[b, c, :, :3] = k @ rot
            mats[b, c, :, 3] = k @ (-(rot @ torch.tensor([0.0, 0.0, height])))
    return mats


def flash_sca_inputs(device, *, batch=1, cams=6, grid=(200, 200, 4), channels=256, heads=8, points=2, seed=5):
    """BEVFormer-base spatial cross-attention without rebatching: 6 cameras
    around the ego car, 4 levels of a 480x800 image, 8 heads x 32 channels,
    a 200x200 BEV grid over [-51.2, 51.2]^2 with 4 heights in [-5, 3], 2
    points per height. Returns the seven tensors and the grid keywords."""
    g = torch.Generator().manual_seed(seed)
    image_hw = (480, 800)
    shapes = [(60, 100), (30, 50), (15, 25), (8, 13)]
    sizes = [h * w for h, w in shapes]
    value = torch.randn(batch, cams, sum(sizes), channels, generator=g)
    proj = pinhole_cameras(batch, cams, image_hw, g)
    gx, gy, gz = grid
    offsets = torch.randn(batch, gy, gx, heads, len(shapes), points, gz, 2, generator=g) * 2.0
    weights = torch.rand(batch, gy, gx, heads, len(shapes), points, gz, generator=g) / (len(shapes) * points * gz)
    tensors = [value, proj, torch.tensor(shapes, dtype=torch.int32),
               torch.tensor([sum(sizes[:i]) for i in range(len(shapes))], dtype=torch.int32),
               torch.tensor(image_hw, dtype=torch.int32), offsets, weights]
    kw = dict(grid_size=grid, voxel_size=(102.4 / gx, 102.4 / gy, 8.0 / gz), voxel_min=(-51.2, -51.2, -5.0))
    return [x.to(device) for x in tensors], kw


def sca_scatter_inputs(device, *, dtype=torch.bfloat16, batch=1, cams=6, max_len=10000, num_query=40000,
                       lens=(10000, 9000, 8000, 10000, 7000, 6000), seed=0):
    """BEVFormer-base rebatched SCA: the c2 MSDA shapes for the B * 6 camera
    images (max_len rebatched queries each), each camera seeing ``lens[cam]``
    distinct BEV queries of 40000, count = cameras per BEV query (min 1)."""
    cfg = CONFIGS["c2"].with_(batch=batch * cams, queries=max_len)
    inp = make_inputs(cfg, dtype=dtype, seed=2333 + seed, device=device, with_grad=False)
    g = torch.Generator(device="cpu").manual_seed(seed)
    indexes = [torch.randperm(num_query, generator=g)[:n].sort().values.to(device) for n in lens[:cams]]
    count = torch.zeros(batch, num_query, device=device)
    for idx in indexes:
        count[:, idx] += 1
    count = count.clamp_(min=1).to(dtype)
    slots = torch.zeros(batch, num_query, cfg.heads * cfg.channels, dtype=dtype, device=device)
    return inp, indexes, count, slots
