"""CPU, two gloo ranks: the N-sharding host logic (column ranges and the
all-gather + re-layout of Y shards) reproduces the unsharded result.  Each
rank computes its shard with the double-precision oracle (no GPU)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, n: int, out_path: str) -> None:
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import datetime

    import torch
    import torch.distributed as dist
    from conftest import load_package
    load_package()
    from oracle.oracle import Oracle
    from spaceslug_b200 import sharding, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    k, m = 128, 6
    w_kn, packed, scales = synth.make_weights(k, n, 0.003, 0.01, seed=1)
    x = synth.make_x(m, k, seed=2)
    c0, c1 = sharding.shard_columns(n, world, rank)
    width = sharding.shard_width(n, world)
    y_shard = np.zeros((m, width), np.float32)
    y_shard[:, : c1 - c0] = Oracle().gemm(x, w_kn[:, c0:c1], scales[c0:c1]).astype(np.float32)
    y = sharding.allgather_columns(torch.from_numpy(y_shard), n, dist)
    if rank == 0:
        np.save(out_path, y.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("n", [64, 200])
def test_sharded_columns_gather_to_full_result(tmp_path, oracle, n):
    from spaceslug_b200 import synth
    out = str(tmp_path / "y.npy")
    mp.start_processes(_worker, args=(2, _free_port(), n, out), nprocs=2, join=True, start_method="spawn")
    w_kn, packed, scales = synth.make_weights(128, n, 0.003, 0.01, seed=1)
    x = synth.make_x(6, 128, seed=2)
    ref = oracle.gemm(x, w_kn, scales).astype(np.float32)
    assert np.array_equal(np.load(out), ref)


def test_shard_columns_cover_every_column_once():
    from spaceslug_b200 import sharding
    for n, world in [(28672, 8), (28672, 2), (11008, 4), (4096, 3), (200, 2)]:
        cols = []
        for r in range(world):
            c0, c1 = sharding.shard_columns(n, world, r)
            assert (c1 - c0) % 8 == 0 or c1 == n
            cols.extend(range(c0, c1))
        assert cols == list(range(n))


def test_plan_bands_cover_rows_in_tile_multiples():
    from spaceslug_b200 import sharding
    assert sharding.plan_bands(4096, 2) == [(0, 2048), (2048, 4096)]
    assert sharding.plan_bands(4096, 4) == [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    assert sharding.plan_bands(300, 4) == [(0, 300)]            # a 44-row tail joins the band before it
    assert sharding.plan_bands(520, 2) == [(0, 256), (256, 520)]
    assert sharding.plan_bands(600, 4) == [(0, 256), (256, 600)]
    assert sharding.plan_bands(5, 3) == [(0, 5)]
    for m in (1, 255, 256, 257, 4095, 4096, 5000):
        for b in (1, 2, 3, 4, 8):
            bands = sharding.plan_bands(m, b)
            assert bands[0][0] == 0 and bands[-1][1] == m and len(bands) <= b
            assert all(r0 < r1 for r0, r1 in bands)
            assert all(a[1] == c[0] for a, c in zip(bands, bands[1:]))
            assert all(r0 % 256 == 0 for r0, _ in bands)
            assert len(bands) == 1 or all(r1 - r0 >= 256 for r0, r1 in bands)


def test_exchange_table_and_pick_fastest(pkg):
    from spaceslug_b200 import sharding
    assert sharding.choose_exchange(1)["engine"] == "none"
    assert sharding.choose_exchange(2)["engine"] == "epilogue"
    assert sharding.choose_exchange(3) == sharding.choose_exchange(2)  # nearest listed size below
    assert sharding.choose_exchange(16) == sharding.choose_exchange(8)
    cands = sharding.CANDIDATES
    best = sharding.pick_fastest(cands, [0.9, 0.7, 0.7, 0.8])
    assert {k: best[k] for k in ("engine", "bands", "push_sms")} == cands[1]  # tie -> earlier candidate
    assert len(best["tuning_ms"]) == len(cands)
