#!/usr/bin/env python3
"""Benchmark: attention forward TFLOP/s (mask-adjusted) on 1..8 B200s.

Workload: BASELINE config 5 -- causal GQA forward, B=1, Hq=64, Hkv=8, N=32768,
d=128, bf16 Q/K/V i.i.d. N(0,1) generated on the device from a seed, bf16 O +
fp32 LSE.  By default (strong scaling) its 8 (batch, kv-head) groups are split
evenly over the ranks: 8/4/2/1 groups per GPU at 1/2/4/8 GPUs, each group with
its 8 query heads, so no K/V crosses ranks; `--scaling weak` runs the whole
config on every rank instead.  One step = one forward over the rank's inputs
(at N=1: Q 512 MiB + K/V 128 MiB + O 512 MiB, all larger than L2, so no flush
is needed between steps).  FLOP are mask-adjusted:
4 * d * (#unmasked (q, k) pairs) per head = 4*128*64*N(N+1)/2 = 1.7593e13.

Ranks share nothing on the data path (heads are independent): the only
collectives are the barrier and the max-over-ranks of the timed region.

Usage:
  python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--config c1..c5|mha8k_causal|mha8k_dense|bias8k|bias8k_full|decode8k|decode32k_gqa]
  torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dnn-flash_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "attention fwd TFLOP/s (mask-adjusted)"

# BASELINE.json configs (name -> shape and score_mod)
CONFIGS = {
    "c1": dict(B=1, Hq=4, Hkv=4, N=512, D=64, causal=False, alibi=False, softcap=0.0, in_scale=1.0,
               out="f32", mask=None),
    "c2": dict(B=4, Hq=16, Hkv=16, N=2048, D=64, causal=True, alibi=False, softcap=0.0, in_scale=1.0,
               out="f32", mask=None),
    "c3": dict(B=2, Hq=32, Hkv=32, N=8192, D=128, causal=True, alibi=True, softcap=50.0, in_scale=0.5,
               out="bf16", mask=None),
    "c4": dict(B=8, Hq=16, Hkv=16, N=4096, D=128, causal=True, alibi=False, softcap=0.0, in_scale=1.0,
               out="bf16", mask="window4_prefix4"),
    "c5": dict(B=1, Hq=64, Hkv=8, N=32768, D=128, causal=True, alibi=False, softcap=0.0, in_scale=1.0,
               out="bf16", mask=None),
    # Not BASELINE configs: the north-star shape (causal N=8192, d=128) as multi-head attention,
    # causal and dense, used to profile the kernel's K/V reuse in L2 (no GQA sharing of K/V).
    "mha8k_causal": dict(B=2, Hq=32, Hkv=32, N=8192, D=128, causal=True, alibi=False, softcap=0.0,
                         in_scale=1.0, out="bf16", mask=None),
    "mha8k_dense": dict(B=2, Hq=32, Hkv=32, N=8192, D=128, causal=False, alibi=False, softcap=0.0,
                        in_scale=1.0, out="bf16", mask=None),
    # The same-shape additive bias (BiasKind::SameShapeTile) on the north-star shape: one fp32 [N, N]
    # matrix shared by every (batch, head) (tensor-bound), and a full fp32 [B, H, N, N] tensor, whose
    # reads dominate the bytes (HBM-bound).
    "bias8k": dict(B=2, Hq=32, Hkv=32, N=8192, D=128, causal=True, alibi=False, softcap=0.0, in_scale=1.0,
                   out="bf16", mask=None, bias="broadcast"),
    "bias8k_full": dict(B=1, Hq=16, Hkv=16, N=8192, D=128, causal=True, alibi=False, softcap=0.0, in_scale=1.0,
                        out="bf16", mask=None, bias="full"),
    # Not BASELINE configs: few query rows (M) over a long key range (N), whose query-tile items
    # would leave most SMs idle; the launch splits the key range (decode / chunked prefill).
    "decode8k": dict(B=1, Hq=8, Hkv=8, M=128, N=8192, D=128, causal=False, alibi=False, softcap=0.0, in_scale=1.0,
                     out="bf16", mask=None),
    "decode32k_gqa": dict(B=1, Hq=8, Hkv=1, M=64, N=32768, D=128, causal=False, alibi=False, softcap=0.0,
                          in_scale=1.0, out="bf16", mask=None),
}
WORKLOAD_NAMES = {
    "c1": "c1_mha_noncausal_b1h4_n512_d64",
    "c2": "c2_mha_causal_b4h16_n2048_d64",
    "c3": "c3_causal_alibi_softcap50_b2h32_n8192_d128",
    "c4": "c4_block_sparse_window512_prefix4_b8h16_n4096_d128",
    "c5": "c5_gqa_causal_hq64_hkv8_n32768_d128",
    "mha8k_causal": "mha_causal_b2h32_n8192_d128",
    "mha8k_dense": "mha_dense_b2h32_n8192_d128",
    "bias8k": "bias_broadcast_nxn_causal_b2h32_n8192_d128",
    "bias8k_full": "bias_full_bhnn_causal_b1h16_n8192_d128",
    "decode8k": "decode_b1h8_m128_n8192_d128",
    "decode32k_gqa": "decode_gqa_b1_hq8_hkv1_m64_n32768_d128",
}


def block_mask_for(cfg):
    """The c4 workload's 128x128 block mask: allowed(qb, kb) = kb <= qb and (qb - kb < 4 or kb < 4)
    (a 512-token sliding window plus 4 global prefix blocks), u8 row-major, nonzero = allowed."""
    if cfg["mask"] is None:
        return None
    import numpy as np

    qb = np.arange(cfg["N"] // 128)[:, None]
    kb = np.arange(cfg["N"] // 128)[None, :]
    return ((kb <= qb) & ((qb - kb < 4) | (kb < 4))).astype(np.uint8)


def kv_split_room(q, k, v, o, lse, cfg):
    """Workspace bytes the launch asks for beyond its 256-byte counter without a block mask: room for
    the partial results of KV splits (or, for causal ALiBi at d = 128, the far-tile bound)."""
    import ctypes as C

    import odf_b200

    p, _keep = odf_b200.fill_params(q, k, v, o, lse, causal=cfg["causal"], scale=1.0 / math.sqrt(cfg["D"]),
                                    block_mask=None, mask_block=(128, 128), alibi=cfg["alibi"],
                                    alibi_slopes_host=None, softcap=cfg["softcap"], workspace=None, visits=None)
    return odf_b200.load_library().odf_fwd_workspace_size(C.byref(p)) - 256


def unmasked_pairs(cfg):
    """#unmasked (query, key) pairs of one (batch, q-head)."""
    return flop_per_unit_pairs(cfg) // (4 * cfg["D"])


def bias_planes(cfg):
    """fp32 bias planes the config reads: 0 (no bias), 1 (one [N, N] matrix for all), B * Hq (full)."""
    kind = cfg.get("bias")
    return 0 if kind is None else (1 if kind == "broadcast" else cfg["B"] * cfg["Hq"])


def flop_per_unit_pairs(cfg):
    """Mask-adjusted FLOP of one (batch, q-head): 4 * d * #unmasked pairs (M query rows, default N)."""
    N, D = cfg["N"], cfg["D"]
    M = cfg.get("M", N)
    mask = block_mask_for(cfg)
    if mask is None:
        if cfg["causal"]:  # top-left: row qi sees keys 0..min(qi, N - 1)
            pairs = M * (M + 1) // 2 if M <= N else N * (N + 1) // 2 + (M - N) * N
        else:
            pairs = M * N
    else:
        # element-level: allowed block and (causal) kj <= qi
        pairs = 0
        nb = mask.shape[0]
        for qb in range(nb):
            for kb in range(nb):
                if not mask[qb, kb]:
                    continue
                if cfg["causal"] and kb == qb:
                    pairs += 128 * 129 // 2
                elif not cfg["causal"] or kb < qb:
                    pairs += 128 * 128
    return 4 * D * pairs


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
        except (OSError, ValueError):
            pass
    return 1590.0, 1400.0, 6650.0, "fallback"


def profiled_traffic(config, seq_len=None):
    """DRAM bytes per launch from the committed ncu summary of this kernel/config, if any
    (profiles/flash_fwd_<config>.md; none for a --seq-len override)."""
    if seq_len is not None:
        return None
    path = ROOT / "profiles" / f"flash_fwd_{config}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU, sampled every 20 ms with timestamps.

    nvidia-smi takes a moment to start, and a timed region can be shorter than that (c5 on 8 GPUs:
    about 40 ms), so the sampler starts before the warm-up and the summary keeps the samples whose
    timestamps fall inside the timed region (mark_start .. mark_end, host wall clock).  The GPU is
    addressed by UUID, so a rank's local device maps to the right physical GPU."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 20

    def __init__(self, local):
        import torch

        self.target = str(local)
        try:
            uuid = str(torch.cuda.get_device_properties(local).uuid)
            if uuid:
                self.target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except (AttributeError, RuntimeError):
            pass
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        import atexit

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                 str(self.INTERVAL_MS), "-i", self.target], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            atexit.register(self.stop)  # never leave the sampling loop behind, whatever happens next
            time.sleep(0.3)  # let it start sampling before the work it is to watch
        except OSError:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
            self.proc = None

    def summary(self):
        import datetime

        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]),
                             {n for n, v in zip(names, parts[6:10]) if v.lower().startswith("active")}))
            except ValueError:
                continue
        inside = rows
        note = None
        if self.t0 is not None and self.t1 is not None:
            lo, hi = self.t0 - 0.5 * self.INTERVAL_MS / 1e3, self.t1 + 0.5 * self.INTERVAL_MS / 1e3
            inside = [r for r in rows if lo <= r[0] <= hi]
            if not inside and rows:  # nothing landed inside: the samples around the region
                near = sorted(rows, key=lambda r: min(abs(r[0] - self.t0), abs(r[0] - self.t1)))[:2]
                inside, note = near, "no sample inside the timed region; the two nearest"
        out = {"sm_mhz": statistics.median(r[1] for r in inside) if inside else None,
               "sm_max_mhz": inside[0][2] if inside else None,
               "reasons": sorted(set().union(*[r[3] for r in inside])) if inside else [],
               "samples": len(inside), "interval_ms": self.INTERVAL_MS,
               "timed_region_s": (self.t1 - self.t0) if self.t0 is not None and self.t1 is not None else None}
        if note:
            out["note"] = note
        return out


def shard_config(cfg, rank, world, scaling):
    """The rank's share of the workload and its input seed.

    weak:   every rank runs the whole configuration on its own inputs (batch element
            `rank` of a global batch of `world`), so per-GPU work is fixed.
    strong: the configuration's (batch, kv-head group) units are split contiguously
            across ranks; a rank keeps whole GQA groups, so no K/V crosses ranks.
    """
    if scaling == "weak":
        return dict(cfg), 1234 + rank
    units = cfg["B"] * cfg["Hkv"]
    if units % world != 0:
        raise ValueError(f"{units} (batch x kv-head) units do not split over {world} ranks")
    per = units // world
    group = cfg["Hq"] // cfg["Hkv"]
    out = dict(cfg)
    if per % cfg["Hkv"] == 0:          # whole batch elements per rank
        out["B"] = per // cfg["Hkv"]
    elif cfg["Hkv"] % per == 0:        # a slice of one batch element's kv heads
        out["B"] = 1
        out["Hkv"] = per
        out["Hq"] = per * group
    else:
        raise ValueError(f"{per} units per rank do not form a [B, H] block")
    return out, 1234 + rank


def reduce_max(values, dist):
    """Element-wise max over ranks of a list of floats (device timing is max over GPUs)."""
    import torch

    if dist is None:
        return [float(v) for v in values]
    backend = dist.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def gpu_numa_cpus(local):
    """(NUMA node, its CPUs usable here) of GPU `local`, from sysfs; (reason, None) when the
    platform gives no node for the GPU."""
    import torch

    props = torch.cuda.get_device_properties(local)
    try:
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
        if node < 0:
            return f"sysfs reports no NUMA node for {bus}", None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        return (node, cpus) if cpus else (f"no CPU of node {node} is usable here", None)
    except (AttributeError, OSError, ValueError) as exc:
        return f"{type(exc).__name__}: {exc}", None


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference_sample(cfg, rows, steps, warmup, use_ref=True):
    """Times the reference's own CPU path on a bounded sample of the workload.

    Sample: every (batch, q-head) of the config restricted to query/key prefix
    [0, rows) -- for a causal mask the prefix rows are an exact sub-problem.
    The reference's per-head flash_attention_qk_pv_tile_ws runs on every host
    core through oracle/_ref's (batch x head) thread pool, with the TensorFlow
    op's default tiles (query_block_size=16, key_block_size=32).
    """
    import numpy as np

    import oracle

    B, Hq, Hkv, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"]
    rng = np.random.default_rng(7)
    R = rows
    q = oracle.round_bf16(rng.standard_normal((B, Hq, R, D)).astype(np.float32) * cfg["in_scale"])
    k = oracle.round_bf16(rng.standard_normal((B, Hkv, R, D)).astype(np.float32) * cfg["in_scale"])
    v = oracle.round_bf16(rng.standard_normal((B, Hkv, R, D)).astype(np.float32) * cfg["in_scale"])
    cores = os.cpu_count() or 1
    kind = "reference" if (use_ref and oracle.ref_available()) else "port"
    kw = dict(causal=cfg["causal"], q_block=16, k_block=32, nthreads=cores)
    if cfg["alibi"]:
        kw["alibi_slopes"] = oracle.alibi_slopes(Hq)
    if kind == "reference" and cfg["softcap"] > 0:
        kind = "port"  # the reference has no soft-cap
    if kind == "port":
        kw["softcap"] = cfg["softcap"]
    if cfg.get("bias"):  # the reference's ScoreBiasFn path reads the same values
        shape = (1, 1, R, R) if cfg["bias"] == "broadcast" else (B, Hq, R, R)
        kw["bias"] = rng.standard_normal(shape).astype(np.float32)
    sub = dict(cfg, N=R, M=R, mask=None)
    flop = flop_per_unit_pairs(sub) * B * Hq
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        if kind == "reference":
            oracle.ref_fwd("flash_ws", q, k, v, **kw)
        else:
            oracle.flash_fwd(q, k, v, want_lse=False, **kw)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    t = statistics.mean(times)
    return {
        "value": flop / t / 1e12,
        "unit": "TFLOP/s",
        "cores": min(cores, B * Hq),
        "kind": kind,
        "sample": f"{B}x{Hq} (batch x q-head) units on query/key prefix [0,{R}) of the workload, "
                  f"{flop / 1e9:.1f} GFLOP per step, tiles 16x32, {kw['nthreads']} threads, mean of {len(times)}",
        "seconds_per_step": t,
    }


def shipped_cpu_bench(timeout_s=120):
    """The reference's own CPU benchmark as shipped (benchmarks/bench_attention.cpp, built unmodified
    into oracle/_ref/onednn_flash_bench): a fixed M=N=128, d=64 causal shape; its exit code is its
    own parity verdict (tiled == standard within 1e-5).  Returns its timings in ms."""
    exe = ROOT / "oracle" / "_ref" / "onednn_flash_bench"
    if not exe.exists():
        return {"available": False, "why": "oracle/_ref/onednn_flash_bench not built"}
    try:
        r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=timeout_s)
    except (OSError, subprocess.TimeoutExpired) as exc:
        return {"available": False, "why": f"{type(exc).__name__}: {exc}"}
    out = {"available": True, "exit_code": r.returncode, "parity_ok": r.returncode == 0}
    for line in r.stdout.splitlines():
        key, _, val = line.partition(":")
        if key.startswith("shape"):
            out["shape"] = val.strip()
        elif key.endswith("_ms"):
            try:
                out[key.strip()] = float(val)
            except ValueError:
                pass
    return out


def batched_single_thread_sample(cfg, rows):
    """The reference's flash_attention_batched_qk_pv_tile as shipped (serial over (batch x head), one
    thread) on a head subset of the workload: one query head per kv-head group of batch 0 (the
    reference has no GQA, so each sampled head gets its group's K/V), causal prefix [0, rows),
    tiles 16x32.  ALiBi and soft-cap are left out (the batched entry takes no bias functor)."""
    import numpy as np

    import oracle

    if not oracle.ref_available():
        return None
    Hq, Hkv, D = cfg["Hq"], cfg["Hkv"], cfg["D"]
    G = Hq // Hkv
    rng = np.random.default_rng(8)
    R = rows
    q = oracle.round_bf16(rng.standard_normal((1, Hkv, R, D)).astype(np.float32) * cfg["in_scale"])
    k = oracle.round_bf16(rng.standard_normal((1, Hkv, R, D)).astype(np.float32) * cfg["in_scale"])
    v = oracle.round_bf16(rng.standard_normal((1, Hkv, R, D)).astype(np.float32) * cfg["in_scale"])
    sub = dict(cfg, N=R, M=R, mask=None)
    flop = flop_per_unit_pairs(sub) * Hkv
    t0 = time.perf_counter()
    oracle.ref_fwd("batched", q, k, v, causal=cfg["causal"], q_block=16, k_block=32)
    dt = time.perf_counter() - t0
    return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "seconds": dt,
            "sample": f"{Hkv} q-heads (head g*{G} of each kv group, batch 0), causal prefix [0,{R}), "
                      f"{flop / 1e9:.2f} GFLOP, tiles 16x32, score mods off"}


def run_reference_arm(args, cfg, workload):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    rows = args.ref_rows
    base = cpu_reference_sample(cfg, rows, args.steps, args.warmup)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": base["value"],
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": base["seconds_per_step"] * 1e3,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload, "sample_rows": rows, "same_config": False,
                   "sample": f"every (batch, q-head) unit of the workload on its causal prefix [0,{rows}): "
                             "an exact sub-problem (causal rows < R see only keys < R), timed at its own "
                             "size; value = its mask-adjusted FLOP / time, not extrapolated to N",
                   "note": f"CPU reference on host cores ({cpu_model()})"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, cfg, workload):
    import numpy as np
    import torch

    import odf_b200

    world, rank, local = dist_setup()
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    cfg, seed = shard_config(cfg, rank, world, args.scaling)
    B, Hq, Hkv, N, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["N"], cfg["D"]
    M = cfg.get("M", N)  # query rows
    out_dtype = torch.bfloat16 if cfg["out"] == "bf16" else torch.float32
    g = torch.Generator(device=dev).manual_seed(seed)
    s = cfg["in_scale"]
    q = (torch.randn((B, Hq, M, D), generator=g, device=dev) * s).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, N, D), generator=g, device=dev) * s).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, N, D), generator=g, device=dev) * s).to(torch.bfloat16)
    o = torch.empty((B, Hq, M, D), dtype=out_dtype, device=dev)
    lse = torch.empty((B, Hq, M), dtype=torch.float32, device=dev)
    mask = block_mask_for(cfg)
    bias = None
    if cfg.get("bias"):
        bshape = (1, 1, M, N) if cfg["bias"] == "broadcast" else (B, Hq, M, N)
        bias = torch.randn(bshape, generator=g, device=dev)
    flop_rank = flop_per_unit_pairs(cfg) * B * Hq
    # the library's own kernels per step: the block-mask tile lists, or for causal ALiBi at d = 128
    # the tile norms and the far-tile bound, then the forward kernel
    far_bound = cfg["alibi"] and cfg["causal"] and D == 128 and mask is None
    launches_per_step = 2 if mask is not None else (3 if far_bound else 1)
    # launches that split their key range (workspace room beyond the 256-byte counter, no block
    # mask, no far-tile bound) add the merge kernel
    kv_splits = mask is None and not far_bound and kv_split_room(q, k, v, o, lse, cfg) > 0
    launches_per_step += 1 if kv_splits else 0

    stream = torch.cuda.current_stream(dev)

    def step():
        odf_b200.flash_fwd(q, k, v, causal=cfg["causal"], alibi=cfg["alibi"], softcap=cfg["softcap"],
                           block_mask=mask, out=o, lse_out=lse, bias=bias)

    # algorithmic bytes: Q, K, V read once, O and LSE written once
    out_es = 2 if out_dtype == torch.bfloat16 else 4
    alg_bytes = (B * Hq * M * D * 2 + 2 * B * Hkv * N * D * 2 + B * Hq * M * D * out_es + B * Hq * M * 4)
    alg_bytes += unmasked_pairs(cfg) * 4 * bias_planes(cfg)  # the bias values the mask keeps, read once
    # Working sets under twice the 126 MB L2 get an L2 flush (a 256 MB write) between timed steps;
    # the value then sums the per-step event times, which exclude the flushes.
    l2_bytes = 126 * 2 ** 20
    flush = torch.empty(64 * 2 ** 20, dtype=torch.float32, device=dev) if alg_bytes < 2 * l2_bytes else None

    clocks = ClockSampler(local).start()
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    # With per-step events (small configs) the GPU would otherwise sit idle while the host enqueues
    # the launch after the start event, and that host time would be counted: a spin kernel
    # (torch's, ~1 ms) after the flush keeps the GPU busy until the launch is queued.
    spin_cycles = 2_000_000 if flush is not None else 0
    clocks.mark_start()
    t_begin.record(stream)
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
            torch.cuda._sleep(spin_cycles)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clocks.mark_end()
    clocks.stop()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    per_launch_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    total_ms = sum(per_launch_ms) if flush is not None else t_begin.elapsed_time(t_end)
    status = odf_b200.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: an in-kernel wait timed out")
    visited = None
    if far_bound:
        # one untimed launch with the tile-visit record: the share of the causal tiles that the
        # kernel visits once the norm bound has left out the far ones
        n_t = -(-N // 128)
        vis = torch.zeros((B * Hq, n_t, n_t), dtype=torch.uint8, device=dev)
        odf_b200.flash_fwd(q, k, v, causal=True, alibi=True, softcap=cfg["softcap"], out=o, lse_out=lse,
                           visits=vis)
        torch.cuda.synchronize(dev)
        visited = int(vis.sum().item()) / (B * Hq * n_t * (n_t + 1) // 2)

    # e2e through the host entry (pinned host buffers, H2D + D2H inside the timed region).  The
    # rank's thread runs on its GPU's NUMA node while it fills the pinned buffers (first touch
    # places the pages there) and while it drives the copies.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    numa_node, numa_cpus = gpu_numa_cpus(local)
    saved_affinity = os.sched_getaffinity(0)
    if numa_cpus:
        os.sched_setaffinity(0, numa_cpus)
    hq = q.cpu().pin_memory()
    hk = k.cpu().pin_memory()
    hv = v.cpu().pin_memory()
    ho = torch.empty(o.shape, dtype=out_dtype).pin_memory()
    hl = torch.empty(lse.shape, dtype=torch.float32).pin_memory()
    hqn, hkn, hvn = (t.view(torch.int16).numpy().view(np.uint16) for t in (hq, hk, hv))
    hon = ho.view(torch.int16).numpy().view(np.uint16) if out_dtype == torch.bfloat16 else ho.numpy()
    hln = hl.numpy()
    hb = bias.cpu().pin_memory() if bias is not None else None
    hbn = hb.numpy() if hb is not None else None

    def e2e_step():
        odf_b200.flash_fwd_host(hqn, hkn, hvn, causal=cfg["causal"], alibi=cfg["alibi"], softcap=cfg["softcap"],
                                block_mask=mask, out=hon, lse_out=hln, bias=hbn)

    e2e_step()  # warm the host-entry pool
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    os.sched_setaffinity(0, saved_affinity)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv) + ((hb,) if hb is not None else ()))
    d2h = ho.numel() * ho.element_size() + hl.numel() * 4

    total_ms, e2e_s = reduce_max([total_ms, e2e_s], dist)

    peak, peak_sus, hbm, peak_kind = measured_peaks()
    value = world * flop_rank * args.steps / (total_ms * 1e-3) / 1e12  # every rank runs the same FLOP
    avg_launch_ms = statistics.mean(per_launch_ms)
    achieved = flop_rank / (avg_launch_ms * 1e-3) / 1e12
    mod = (1 if cfg["alibi"] else 0) | (2 if cfg["softcap"] > 0 else 0) | (4 if cfg.get("bias") else 0)
    if mod == 0 and D == 128 and cfg["mask"] is None and -(-N // 128) >= 16:
        mod = 8  # the library's launch picks the variant that skips the row-max pass (kModSkipMax)
    if flop_rank / alg_bytes >= peak * 1e12 / (hbm * 1e9):  # above the ridge point: tensor-bound
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_kind": f"{peak_kind} bf16 burst (cuBLAS); sustained {peak_sus}",
                "frac_of_sustained": achieved / peak_sus}
    else:  # below it (short, small shapes): algorithmic bytes against the measured copy bandwidth
        gbs = alg_bytes / (avg_launch_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                "peak_kind": f"{peak_kind} HBM copy bandwidth", "tflops": achieved}
    roof.update({"traffic": profiled_traffic(args.config, args.seq_len), "algorithmic_bytes": alg_bytes,
                 "kernel": f"flash_fwd_kernel<{D},{mod}>" + (" + split_combine_kernel" if kv_splits else ""),
                 "avg_launch_ms": avg_launch_ms})
    if visited is not None:
        # causal ALiBi: far tiles (every score 48 (log2) below the row max by the norm bound) are
        # left out, so the tensor pipe runs only on the visited share of the algorithmic FLOP
        roof.update({"tiles_visited_frac": visited, "achieved_on_visited_tiles": achieved * visited,
                     "frac_on_visited_tiles": achieved * visited / peak})
    l2_note = ("L2 flushed (256 MB write) between timed steps, then a ~1 ms spin kernel so the launch is "
               "queued before its start event; value from per-step events" if flush is not None
               else f"inputs and outputs ({alg_bytes / 2 ** 20:.0f} MiB) larger than twice L2; no flush needed")
    result = None
    if rank == 0:
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": workload,
                "batch_per_gpu": B, "global_batch": B * world if args.scaling == "weak" else CONFIGS[args.config]["B"],
                "heads_q_per_gpu": Hq, "heads_kv_per_gpu": Hkv, "seq_len": N, "query_rows": M,
                "kv_splits": bool(kv_splits),
                "head_dim": D, "causal": cfg["causal"], "alibi": cfg["alibi"], "softcap": cfg["softcap"],
                "block_mask": cfg["mask"], "bias": cfg.get("bias"), "out_dtype": cfg["out"], "lse": True,
                "parallelism": f"(batch x head) shards, {world} GPU(s), no collective on the data path",
                "flop_per_gpu_step": flop_rank,
                "l2": l2_note,
            },
            "roofline": roof,
            "e2e": {"value": world * flop_rank / e2e_s / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "path": "odf_flash_fwd_host (pinned host buffers)",
                    "host_numa": ({"node": numa_node, "cpus": len(numa_cpus)} if numa_cpus
                                  else f"not bound ({numa_node})")},
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                base = cpu_reference_sample(cfg, args.cpu_rows, 1, 0)
                result["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
            except Exception as exc:  # the CPU checker is optional for the GPU number
                result["cpu_baseline"] = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "unavailable",
                                          "sample": f"{type(exc).__name__}: {exc}"}
            result["cpu_baseline"]["cpu_model"] = cpu_model()
            result["cpu_baseline"]["host_cores"] = os.cpu_count()
            try:
                result["cpu_baseline"]["batched_single_thread"] = batched_single_thread_sample(cfg, args.cpu_rows // 3)
            except Exception as exc:
                result["cpu_baseline"]["batched_single_thread"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
            result["cpu_baseline"]["shipped_bench"] = shipped_cpu_bench()
        print(json.dumps(result), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c5")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-rows", type=int, default=3072, help="prefix rows of the CPU baseline sample")
    ap.add_argument("--ref-rows", type=int, default=1536, help="prefix rows per step of the reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong",
                    help="strong (default): the config's (batch, kv-head) groups split over the GPUs; "
                         "weak: the whole config on every GPU")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="override N (profiling of a smaller case only; the BASELINE config is the default)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    workload = WORKLOAD_NAMES[args.config]
    if args.seq_len is not None:
        cfg["N"] = args.seq_len
        workload = f"{workload}_seq{args.seq_len}"
    if args.impl == "reference":
        return run_reference_arm(args, cfg, workload)
    return run_ours(args, cfg, workload)


if __name__ == "__main__":
    sys.exit(main())
