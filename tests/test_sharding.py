"""Multi-rank logic on CPU (gloo, world sizes 2 and 3): asset shards, Morton
ranges, and the halo plan/exchange.  Each rank's conv over its halo-extended
buffer must equal the global conv's rows exactly (the reference's own chunk
test shows that a chunk without a halo does not:
burn_trellis/src/runtime_model/sparse_decoder_tests.rs:238-292)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bevy_synth_b200 import sharding, synth


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_asset_shard_partitions_all_assets():
    for world in (1, 2, 3, 8):
        got = sum((sharding.asset_shard(64, r, world) for r in range(world)), [])
        assert got == list(range(64))
    assert sharding.asset_shard(64, 7, 8) == list(range(56, 64))


def test_morton_ranges_cover_rows():
    r = sharding.morton_ranges(10, 3)
    assert r == [(0, 4), (4, 7), (7, 10)]


def _grid():
    coords = synth.morton_sort(synth.unique_cells(0, synth.ellipsoid_shell(40, (20.3, 19.7, 20.1),
                                                                             (13.0, 9.0, 15.0), 1.0)))
    return coords


def _oracle_map(all_c: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    cfg = oracle.OracleConfig(1, 1)
    m = oracle.build_neighbor_rows(cfg, all_c.numpy().astype(np.uint32), oracle.DUP_LOWEST,
                                   q.numpy().astype(np.uint32))
    return torch.from_numpy(m)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        coords = torch.from_numpy(_grid())
        n = coords.shape[0]
        ranges = sharding.morton_ranges(n, world)
        plan = sharding.HaloPlan.build(coords, ranges, rank, _oracle_map)
        rng = np.random.default_rng(1)
        c = 8
        x = rng.standard_normal((n, c)).astype(np.float32)
        w = (rng.standard_normal((c, 3, 3, 3, c)) * 0.1).astype(np.float32)
        b = rng.standard_normal(c).astype(np.float32)
        lo, hi = ranges[rank]
        buf = plan.buffer(c, torch.float32, "cpu")
        buf[:plan.n_local] = torch.from_numpy(x[lo:hi])
        plan.exchange(buf)
        np.testing.assert_array_equal(buf[plan.n_local:].numpy(), x[plan.halo_global.numpy()])
        cfg = oracle.OracleConfig(c, c)
        local = oracle.subm_conv_flex(cfg, w, b, buf.numpy(), plan.nbr_local.numpy(), threads=1)
        full_map = oracle.build_neighbor_rows(cfg, coords.numpy().astype(np.uint32))
        glob = oracle.subm_conv_flex(cfg, w, b, x, full_map, threads=1)[lo:hi]
        q.put((rank, bool(np.array_equal(local, glob)), plan.n_halo, int(plan.send_idx.numel())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_reproduces_global_conv(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(ok for _, ok, _, _ in res)
    # halo rows received in total == rows sent in total, and a cut grid needs some
    assert sum(r[2] for r in res) == sum(r[3] for r in res) > 0
