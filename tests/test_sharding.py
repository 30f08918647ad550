"""Multi-rank logic on CPU (gloo, world sizes 2, 3 and 4): asset shards, Morton
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


def _oracle_query(table: torch.Tensor, q: torch.Tensor, cfg) -> torch.Tensor:
    """The map on the CPU oracle (lib.rs:69-109, lowest row on duplicates)."""
    oc = oracle.OracleConfig(1, 1, cfg.kernel_d, cfg.kernel_h, cfg.kernel_w, axis_order=cfg.axis_order,
                             axis_sign=cfg.axis_sign)
    m = oracle.build_neighbor_rows(oc, table.numpy().astype(np.uint32), oracle.DUP_LOWEST,
                                   q.numpy().astype(np.uint32))
    return torch.from_numpy(m)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bevy_synth_b200 import flex_gmm as F
        coords = torch.from_numpy(_grid())
        n = coords.shape[0]
        ranges = sharding.morton_ranges(n, world)
        lo, hi = ranges[rank]
        fcfg = F.SparseSubmConvConfig.subm3(8, 8)
        plan = sharding.HaloPlan.build_local(coords[lo:hi].contiguous(), fcfg, query_fn=_oracle_query)
        assert plan.lo == lo and plan.n_local == hi - lo
        rng = np.random.default_rng(1)
        c = 8
        x = rng.standard_normal((n, c)).astype(np.float32)
        w = (rng.standard_normal((c, 3, 3, 3, c)) * 0.1).astype(np.float32)
        b = rng.standard_normal(c).astype(np.float32)
        order = plan.order.numpy().astype(np.int64)
        buf = plan.buffer(c, torch.float32, "cpu")
        buf[:plan.n_local] = torch.from_numpy(x[lo:hi][order])
        plan.exchange(buf)
        np.testing.assert_array_equal(buf[plan.n_local:].numpy(), x[plan.halo_global.numpy()])
        cfg = oracle.OracleConfig(c, c)
        full_map = oracle.build_neighbor_rows(cfg, coords.numpy().astype(np.uint32))
        # the local map, with plan rows and halo rows put back to global ids, is the global map's rows
        glob_of = np.concatenate([lo + order, plan.halo_global.numpy()])
        nl = plan.nbr_local.numpy()
        remapped = np.where(nl >= 0, glob_of[np.maximum(nl, 0)], -1)
        maps_equal = bool(np.array_equal(remapped, full_map[lo + order]))
        # interior rows read no halo row; boundary rows hold every sent row
        ni = plan.n_interior
        interior_ok = bool((nl[:ni] < plan.n_local).all()) and bool((plan.send_idx.numpy() >= ni).all())
        local = oracle.subm_conv_flex(cfg, w, b, buf.numpy(), nl, threads=1)
        glob = oracle.subm_conv_flex(cfg, w, b, x, full_map, threads=1)[lo:hi][order]
        q.put((rank, bool(np.array_equal(local, glob)) and maps_equal and interior_ok, plan.n_halo,
               int(plan.send_idx.numel())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
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
