"""Host logic of the multi-GPU decompositions, on CPU ranks over gloo.

Two processes (world size 2) stand in for two GPUs. The C oracle stands in for
the kernel on each rank's shard (tests may run the oracle; the product never
does), so what is checked is exactly the sharding and the collective:
batch shards need no exchange, query shards reduce-scatter grad_value into
the single-process answer.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden
from muspace_b200.sharding import (all_gather_grad_value, image_shard_numel, padded_numel, reduce_scatter_grad_value,
                                   reduce_scatter_image, shard_range)


def test_shard_range_covers_every_unit_once():
    for n in (0, 1, 5, 48, 10000, 10001):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for rank in range(world):
                a, b = shard_range(n, world, rank)
                assert 0 <= a <= b <= n
                seen.extend(range(a, b))
            assert seen == list(range(n))
            sizes = [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_padded_numel():
    assert padded_numel(10, 4) == 12
    assert padded_numel(12, 4) == 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    from oracle import oracle_backward, oracle_forward

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        g = load_golden("c2_small")
        args = [g[k] for k in ("value", "spatial_shapes", "level_start_index")]
        # query sharding: value replicated, queries split, grad_value reduce-scattered
        q0, q1 = shard_range(g["sampling_locations"].shape[1], world, rank)
        loc = g["sampling_locations"][:, q0:q1]
        w = g["attention_weights"][:, q0:q1]
        grad = g["grad_output"][:, q0:q1]
        out = oracle_forward(*args, loc, w)
        gv, gl, gw = oracle_backward(*args, loc, w, grad)
        shard, offset = reduce_scatter_grad_value(torch.from_numpy(gv))
        full = all_gather_grad_value(shard, gv.shape)
        # per camera image, as the overlapped GPU step exchanges it
        image_shards = torch.empty(gv.shape[0], image_shard_numel(gv[0].size, world))
        for i in range(gv.shape[0]):
            reduce_scatter_image(torch.from_numpy(gv[i]), image_shards[i])
        # batch sharding: each rank owns whole batch entries, no exchange at all
        b0, b1 = shard_range(g["value"].shape[0], world, rank)
        bout = oracle_forward(g["value"][b0:b1], g["spatial_shapes"], g["level_start_index"],
                              g["sampling_locations"][b0:b1], g["attention_weights"][b0:b1])
        np.savez(
            os.path.join(result_dir, f"rank{rank}.npz"),
            out=out, gl=gl, gw=gw, shard=shard.numpy(), offset=offset, full=full.numpy(), bout=bout, q=(q0, q1), b=(b0, b1),
            image_shards=image_shards.numpy(),
        )
    finally:
        dist.destroy_process_group()


def test_two_rank_query_and_batch_sharding_reproduce_the_single_process_answer(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    g = load_golden("c2_small")
    gv_ref = g["grad_value"].reshape(-1)
    for rank in range(world):
        r = np.load(tmp_path / f"rank{rank}.npz")
        q0, q1 = r["q"]
        b0, b1 = r["b"]
        np.testing.assert_allclose(r["out"], g["output"][:, q0:q1], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(r["gl"], g["grad_sampling_locations"][:, q0:q1], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(r["gw"], g["grad_attention_weights"][:, q0:q1], rtol=1e-4, atol=1e-4)
        off = int(r["offset"])
        shard = r["shard"]
        valid = max(0, min(shard.size, gv_ref.size - off))
        np.testing.assert_allclose(shard[:valid], gv_ref[off : off + valid], rtol=1e-5, atol=1e-5)
        assert not np.any(shard[valid:]), "padding must stay zero"
        np.testing.assert_allclose(r["full"], g["grad_value"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(r["bout"], g["output"][b0:b1], rtol=1e-5, atol=1e-5)
        per_image = r["image_shards"]
        for i in range(g["grad_value"].shape[0]):
            flat = g["grad_value"][i].reshape(-1)
            n = per_image.shape[1]
            lo = rank * n
            valid = max(0, min(n, flat.size - lo))
            np.testing.assert_allclose(per_image[i, :valid], flat[lo : lo + valid], rtol=1e-5, atol=1e-5)
            assert not np.any(per_image[i, valid:]), "padding must stay zero"
