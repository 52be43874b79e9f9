"""Host-side multi-GPU logic of bench.py with world_size-2 gloo ranks on CPU.

Heads are independent, so the data path has no collective: each rank gets a shard
(weak: the whole config on its own inputs; strong: contiguous (batch, kv-head) groups)
and the only collective is the max-over-ranks of the timed region.
"""
from __future__ import annotations

import json
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        shards = {name: bench.shard_config(cfg, rank, world, "strong")[0] for name, cfg in bench.CONFIGS.items()
                  if (cfg["B"] * cfg["Hkv"]) % world == 0}
        weak_cfg, weak_seed = bench.shard_config(bench.CONFIGS["c5"], rank, world, "weak")
        timing = bench.reduce_max([10.0 + rank, 5.0 - rank], dist)
        dist.barrier()
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"shards": shards, "weak": weak_cfg, "seed": weak_seed, "timing": timing}, f)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    # max over ranks, identical on every rank
    assert res[0]["timing"] == res[1]["timing"] == [11.0, 5.0]
    # weak scaling: whole config per rank, distinct input seeds
    assert res[0]["weak"] == res[1]["weak"] == bench.CONFIGS["c5"]
    assert res[0]["seed"] != res[1]["seed"]
    # strong scaling: the ranks' FLOP add up to the whole config's
    for name, cfg in bench.CONFIGS.items():
        if name not in res[0]["shards"]:
            continue
        total = bench.flop_per_unit_pairs(cfg) * cfg["B"] * cfg["Hq"]
        parts = sum(bench.flop_per_unit_pairs(r["shards"][name]) * r["shards"][name]["B"] * r["shards"][name]["Hq"]
                    for r in res)
        assert parts == total, name


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_shards_keep_whole_gqa_groups(world):
    cfg = bench.CONFIGS["c5"]
    shard, _ = bench.shard_config(cfg, 0, world, "strong")
    assert shard["Hq"] // shard["Hkv"] == cfg["Hq"] // cfg["Hkv"]
    assert shard["Hkv"] * world == cfg["Hkv"]


def test_strong_sharding_rejects_uneven_split():
    with pytest.raises(ValueError):
        bench.shard_config(bench.CONFIGS["c1"], 0, 3, "strong")


def test_clock_summary_keeps_samples_inside_the_timed_region():
    """The bench line's `clocks` field: nvidia-smi samples (timestamped, every 20 ms) are kept only
    when they fall inside the timed region; with none inside, the two nearest are reported and
    labelled as such.  No GPU and no nvidia-smi needed: the sampler's output is given as text."""
    import datetime

    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.proc = None
    t = datetime.datetime(2026, 12, 2, 6, 0, 0)

    def line(dt_ms, mhz, power_cap):
        ts = (t + datetime.timedelta(milliseconds=dt_ms)).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        cap = "Active" if power_cap else "Not Active"
        return f"{ts}, 0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, {cap}"

    s.lines = [line(0, 1965, False), line(100, 1700, True), line(120, 1680, True), line(140, 1690, True),
               line(400, 1965, False)]
    s.t0 = (t + datetime.timedelta(milliseconds=95)).timestamp()
    s.t1 = (t + datetime.timedelta(milliseconds=150)).timestamp()
    out = s.summary()
    assert out["samples"] == 3 and out["sm_mhz"] == 1690.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and "note" not in out
    # a region between two samples: the nearest ones, labelled
    s.t0 = (t + datetime.timedelta(milliseconds=200)).timestamp()
    s.t1 = (t + datetime.timedelta(milliseconds=230)).timestamp()
    out = s.summary()
    assert out["samples"] == 2 and "note" in out
