#!/usr/bin/env python
"""Benchmark of the b200attn hot path (driver contract: one JSON line on rank 0).

Default workload: config 3 -- causal prefill forward, B=4, H=32, N=8192,
D=128, bf16, returning O and L: the shape the "% of BF16 tensor peak" target
is stated on.  Its 128 (b, h) units shard across torchrun ranks with no
collective.  The same line carries a `secondary` object with config 2 (the
reference's headline shape, B=1 H=8 N=4096 D=64 fp16 non-causal, which
bench/bench_fa3_headline.py of the reference times as forward()+L) and config 4
(split-KV GQA decode), timed in the same process.  A step is one forward over
one batch.  Other main configs: --config 1|2|3m|3s|4|4s|5a|5b|6|6s|7|7s|7m.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): configs 1/2 run independent replicas
(weak scaling); config 3 shards its 128 (b, h) units and configs 4/5a shard
batch rows across ranks with no collective (strong scaling); config 5b shards
the KV sequence and all-gathers the partials over NCCL.  Time is device
time over the K timed steps (CUDA events on the launching stream), max over
ranks.  Inputs: seeded synthetic data of the configs' shapes; steps rotate over
enough input sets that the bytes touched between reuses exceed the 126 MB L2.

`--impl reference` times the reference's CPU path for the same metric: its
naive attention (ref/naive_attn.py:10-38, restated in oracle/attention.py) in
fp32 numpy on the host cores, one bounded sample of the workload per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from types import SimpleNamespace

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flashattn-cuda_b200"))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 2 ** 20
METRIC = "prefill fwd TFLOP/s & % B200 BF16 peak; decode KV GB/s & % HBM; 1/2/4/8 GPU"


# ------------------------------------------------------------------ workloads
CONFIGS = {
    "1": dict(kind="prefill", B=1, H=8, Hkv=8, N=1024, D=64, dtype="float16", causal=False,
              shard=False, name="config1: prefill fwd B=1 H=8 N=1024 D=64 fp16 non-causal"),
    "2": dict(kind="prefill", B=1, H=8, Hkv=8, N=4096, D=64, dtype="float16", causal=False,
              shard=False, name="config2: prefill fwd B=1 H=8 N=4096 D=64 fp16 non-causal"),
    "3": dict(kind="prefill", B=4, H=32, Hkv=32, N=8192, D=128, dtype="bfloat16", causal=True,
              shard=True, name="config3: prefill fwd B=4 H=32 N=8192 D=128 bf16 causal"),
    # config 3 at half the batch (403 MB of Q/K/V): 1024 pair items on 148 SMs, the schedule
    # config 3 itself runs (pairs); the case ncu section captures of that schedule run on
    "3m": dict(kind="prefill", B=2, H=32, Hkv=32, N=8192, D=128, dtype="bfloat16", causal=True,
               shard=True, name="config3-half: prefill fwd B=2 H=32 N=8192 D=128 bf16 causal"),
    # config 3 at 1/4 of the batch (201 MB of Q/K/V, still > L2): 32 heads per GPU, the
    # share of config 3 at 4 GPUs (heaviest-first single-block schedule)
    "3s": dict(kind="prefill", B=1, H=32, Hkv=32, N=8192, D=128, dtype="bfloat16", causal=True,
               shard=True, name="config3-small: prefill fwd B=1 H=32 N=8192 D=128 bf16 causal"),
    "4": dict(kind="decode", B=64, H=32, Hkv=8, L=16384, D=128, dtype="float16", splits=16,
              shard=True, name="config4: split-KV GQA decode B=64 H=32 Hkv=8 L=16384 D=128 fp16"),
    # config 4 at 1/8 batch (537 MB of KV, still > L2): the case ncu section captures run on
    "4s": dict(kind="decode", B=8, H=32, Hkv=8, L=16384, D=128, dtype="float16", splits=16,
               shard=True, name="config4-small: split-KV GQA decode B=8 H=32 Hkv=8 L=16384 D=128 fp16"),
    "5b": dict(kind="kvshard", B=1, H=32, Hkv=8, L=131072, D=128, dtype="bfloat16", splits=32,
               shard=True, name="config5b: KV-sharded decode B=1 H=32 Hkv=8 L=131072 D=128 bf16, "
                                "NCCL all-gather of partials"),
    "5a": dict(kind="paged", B=128, H=32, Hkv=8, D=128, page=16, lmin=512, lmax=32768,
               dtype="float16", pps=64, shard=True,
               name="config5a: paged decode B=128 H=32 Hkv=8 D=128 fp16 page=16 len U[512,32768]"),
    # training counterparts: the backward (dQ, dK, dV) at the config 3 / config 2 shapes
    "7": dict(kind="backward", B=4, H=32, Hkv=32, N=8192, D=128, dtype="bfloat16", causal=True,
              shard=True, name="backward B=4 H=32 N=8192 D=128 bf16 causal (config 3 shape)"),
    "7s": dict(kind="backward", B=1, H=8, Hkv=8, N=4096, D=64, dtype="float16", causal=False,
               shard=False, name="backward B=1 H=8 N=4096 D=64 fp16 (config 2 shape)"),
    # config 7 at 1/16 of the heads (128 MB of inputs and gradients): the case ncu captures run on
    "7m": dict(kind="backward", B=1, H=8, Hkv=8, N=8192, D=128, dtype="bfloat16", causal=True,
               shard=True, name="backward B=1 H=8 N=8192 D=128 bf16 causal (config 7, small)"),
    "6": dict(kind="varlen", B=16, H=32, Hkv=8, D=128, lmin=256, lmax=8192, dtype="bfloat16",
              causal=True, shard=True,
              name="varlen prefill fwd: 16 packed sequences len U[256,8192] H=32 Hkv=8 D=128 "
                   "bf16 causal"),
    # config 6 with 4 sequences (~230 MB of Q/K/V, > L2): the case ncu captures run on
    "6s": dict(kind="varlen", B=4, H=32, Hkv=8, D=128, lmin=256, lmax=8192, dtype="bfloat16",
               causal=True, shard=True,
               name="varlen prefill fwd: 4 packed sequences len U[256,8192] H=32 Hkv=8 D=128 "
                    "bf16 causal (config 6, small)"),
}


def varlen_lengths(c):
    rng = np.random.default_rng(66)
    return rng.integers(c["lmin"], c["lmax"] + 1, size=c["B"]).astype(np.int64)


def prefill_flops(c, units):
    """Algorithmic FLOPs: 4*N^2*D per (b,h) unit; causal counts 2*D*N*(N+1)."""
    N, D = c["N"], c["D"]
    per = 2 * D * N * (N + 1) if c["causal"] else 4 * N * N * D
    return per * units


def paged_lengths(c):
    rng = np.random.default_rng(55)
    return rng.integers(c["lmin"], c["lmax"] + 1, size=c["B"]).astype(np.int64)


# ---------------------------------------------------------------- clock probe
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while the GPU runs the
    workload: from the warm-up, across the timed region, to one sample after it."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def count(self) -> int:
        """Samples written so far."""
        try:
            with open(self.path) as f:
                return sum(1 for line in f if line.strip())
        except Exception:
            return 0

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]),
                "reasons": sorted(reasons), "samples": len(rows)}


def read_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def read_traffic(key: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(key)
    return None


# -------------------------------------------------------------- CPU baselines
def cpu_sample(cfg_key: str, steps: int, warmup: int):
    """Time the reference's CPU path (oracle port, fp32 numpy) on bounded samples.

    Returns (value, unit, sample description, cores).
    """
    from oracle import attention as ora
    c = CONFIGS[cfg_key]
    cores = os.cpu_count() or 1
    if c["kind"] == "backward":
        # one (b, h) head at a bounded length per step
        N, D = min(c["N"], 2048), c["D"]
        q, k, v, do = (ora.seeded_normal((1, 1, N, D), s) for s in (1, 2, 3, 4))
        for i in range(warmup + steps):
            if i == warmup:
                start = time.perf_counter()
            ora.attention_backward(q, k, v, do, None, c["causal"], np.float32)
        el = time.perf_counter() - start
        flops = 10 * D * N * N * (0.5 if c["causal"] else 1.0) * steps
        return flops / el / 1e12, "TFLOP/s", \
            f"one (b,h) head, N={N}, fp32 numpy naive backward, per step", cores
    if c["kind"] in ("prefill", "varlen"):
        # one (b, h) head per step (rows limited for the causal N=8192 case);
        # varlen: one head of a sequence of the median length
        N = c["N"] if c["kind"] == "prefill" else int(np.median(varlen_lengths(c)))
        D = c["D"]
        rows = min(N, 2048)
        q = ora.seeded_normal((rows, D), 1)
        k = ora.seeded_normal((N, D), 2)
        v = ora.seeded_normal((N, D), 3)
        off = N - rows
        for i in range(warmup + steps):
            if i == warmup:
                start = time.perf_counter()
            ora.attention_head(q, k, v, D ** -0.5, c["causal"], off, np.float32)
        el = time.perf_counter() - start
        # 4*D FLOPs per (query row, visible key); causal row g sees g+1 keys
        keys = sum(off + r + 1 for r in range(rows)) if c["causal"] else rows * N
        flops = 4 * D * keys * steps
        return flops / el / 1e12, "TFLOP/s", \
            f"one (b,h) head, {rows} query rows x {N} keys, fp32 numpy, per step", cores
    # decode: one batch row per step
    if c["kind"] == "decode":
        L, D, Hkv, H = c["L"], c["D"], c["Hkv"], c["H"]
    elif c["kind"] == "kvshard":
        L, D, Hkv, H = c["L"] // 8, c["D"], c["Hkv"], c["H"]
    else:
        L, D, Hkv, H = int(paged_lengths(c).mean()), c["D"], c["Hkv"], c["H"]
    q = ora.seeded_normal((1, H, D), 1)
    k = ora.seeded_normal((1, Hkv, L, D), 2)
    v = ora.seeded_normal((1, Hkv, L, D), 3)
    for i in range(warmup + steps):
        if i == warmup:
            start = time.perf_counter()
        ora.decode(q, k, v, None, np.float32)
    el = time.perf_counter() - start
    byts = 2 * Hkv * L * D * 2 * steps  # fp16 K+V bytes of the sample
    return byts / el / 1e9, "GB/s", f"one batch row (KV length {L}), fp32 numpy, per step", cores


# ------------------------------------------------------------------ GPU arm
def make_workload(cfg_key, args, rank, world, dev):
    """Device-resident inputs and the step function of one workload on this rank
    (plus the host buffers and call of its end-to-end form)."""
    import torch
    import b200attn

    c = CONFIGS[cfg_key]
    tdt = torch.float16 if c["dtype"] == "float16" else torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    if c["kind"] == "prefill":
        units = c["B"] * c["H"]
        B = c["B"]
        if c["shard"]:
            assert c["B"] * c["H"] % world == 0
            units //= world
            Bl, Hl = (1, units) if units < c["H"] else (units // c["H"], c["H"])
        else:
            Bl, Hl = c["B"], c["H"]
        shape = (Bl, Hl, c["N"], c["D"])
        set_bytes = 4 * np.prod(shape) * 2
        nsets = max(1, int(np.ceil(1.5 * L2_BYTES / set_bytes))) if set_bytes < L2_BYTES else 1
        sets = [[torch.randn(shape, device=dev, generator=gen).to(tdt) for _ in range(3)]
                for _ in range(nsets)]
        flops = prefill_flops(c, Bl * Hl)
        work_per_step = flops
        unit = "TFLOP/s"

        def step(i):
            q, k, v = sets[i % nsets]
            return b200attn.forward(q, k, v, causal=c["causal"])

        kernel_regex = "prefill_d64_kernel" if c["D"] == 64 else "prefill_fwd_kernel"
        bound, peak = "tensor", None
        h2d = 3 * int(np.prod(shape)) * 2
        d2h = int(np.prod(shape)) * 2 + int(np.prod(shape[:3])) * 4
        host_in = [torch.randn(shape, generator=torch.Generator().manual_seed(rank)).to(tdt)
                   .pin_memory() for _ in range(3)]
        host_out = (torch.empty(shape, dtype=tdt).pin_memory(),
                    torch.empty(shape[:3], dtype=torch.float32).pin_memory())

        e2e_in = host_in
        static_out = False

        def e2e_run(q, k, v):
            return b200attn.forward(q, k, v, causal=c["causal"])

        workload = dict(workload=c["name"], B=Bl, H=Hl, N=c["N"], D=c["D"],
                        causal=c["causal"], dtype=c["dtype"], units_per_rank=Bl * Hl)
    elif c["kind"] == "backward":
        units = c["B"] * c["H"]
        if c["shard"]:
            assert units % world == 0
            units //= world
            Bl, Hl = (1, units) if units < c["H"] else (units // c["H"], c["H"])
        else:
            Bl, Hl = c["B"], c["H"]
        shape = (Bl, Hl, c["N"], c["D"])
        set_bytes = 8 * np.prod(shape) * 2  # q k v O dO + dq dk dv
        nsets = max(1, int(np.ceil(1.5 * L2_BYTES / set_bytes))) if set_bytes < L2_BYTES else 1
        sets = []
        for _ in range(nsets):
            q, k, v, do = (torch.randn(shape, device=dev, generator=gen).to(tdt) for _ in range(4))
            O, L = b200attn.forward(q, k, v, causal=c["causal"])
            sets.append((q, k, v, O, do, L))
        # 5 products of 2*N*N*D FLOPs each (S, dP, dV, dK, dQ); causal: the unmasked half
        work_per_step = 10 * c["N"] * c["N"] * c["D"] * Bl * Hl * (0.5 if c["causal"] else 1.0)
        unit = "TFLOP/s"

        def step(i):
            return b200attn.backward(*sets[i % nsets], causal=c["causal"])

        kernel_regex = "bwd_main_kernel"
        bound, peak = "tensor", None
        n_el = int(np.prod(shape))
        h2d = 5 * n_el * 2 + int(np.prod(shape[:3])) * 4
        d2h = 3 * n_el * 2
        hg = torch.Generator().manual_seed(rank)
        host_in = [torch.randn(shape, generator=hg).to(tdt).pin_memory() for _ in range(5)]
        host_in.append(torch.randn(shape[:3], generator=hg).abs().pin_memory())
        host_out = tuple(torch.empty(shape, dtype=tdt).pin_memory() for _ in range(3))

        e2e_in = host_in
        static_out = False

        def e2e_run(q, k, v, O, do, L):
            return b200attn.backward(q, k, v, O, do, L, causal=c["causal"])

        workload = dict(workload=c["name"], B=Bl, H=Hl, N=c["N"], D=c["D"], causal=c["causal"],
                        dtype=c["dtype"], units_per_rank=Bl * Hl,
                        flops="10*N^2*D per (b,h) (x0.5 causal): S, dP, dV, dK, dQ")
    elif c["kind"] == "varlen":
        lens_all = varlen_lengths(c)
        # greedy balance of sequences over ranks by attention work (~ n^2)
        order = np.argsort(-lens_all)
        loads = [0] * world
        mine = []
        for idx in order:
            r = int(np.argmin(loads))
            loads[r] += int(lens_all[idx]) ** 2
            if r == rank:
                mine.append(idx)
        lens = lens_all[sorted(mine)]
        H, Hkv, D = c["H"], c["Hkv"], c["D"]
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
        T, maxlen = int(lens.sum()), int(lens.max())
        q = torch.randn(T, H, D, device=dev, generator=gen).to(tdt)
        k = torch.randn(T, Hkv, D, device=dev, generator=gen).to(tdt)
        v = torch.randn(T, Hkv, D, device=dev, generator=gen).to(tdt)
        cud = cu.to(dev)
        nsets = 1  # 550 MB of Q/K/V per step on one rank, well past L2
        # causal with Nk == N: each (sequence, head) does 2*D*n*(n+1) FLOPs
        work_per_step = sum(2 * D * int(n) * (int(n) + 1) for n in lens) * H
        unit = "TFLOP/s"

        def step(i):
            return b200attn.forward_varlen(q, k, v, cud, cud, maxlen, causal=c["causal"])

        kernel_regex = "prefill_fwd_kernel"
        bound, peak = "tensor", None
        h2d = (T * H * D + 2 * T * Hkv * D) * 2 + 2 * cu.numel() * 4
        d2h = T * H * D * 2 + H * T * 4
        hg = torch.Generator().manual_seed(rank)
        host_in = [torch.randn(T, H, D, generator=hg).to(tdt).pin_memory(),
                   torch.randn(T, Hkv, D, generator=hg).to(tdt).pin_memory(),
                   torch.randn(T, Hkv, D, generator=hg).to(tdt).pin_memory(),
                   cu.pin_memory(), cu.clone().pin_memory()]
        host_out = (torch.empty(T, H, D, dtype=tdt).pin_memory(),
                    torch.empty(H, T, dtype=torch.float32).pin_memory())

        e2e_in = host_in
        static_out = False

        def e2e_run(q, k, v, cq, ck):
            return b200attn.forward_varlen(q, k, v, cq, ck, maxlen, causal=c["causal"])

        workload = dict(workload=c["name"], sequences=len(lens), total_tokens=T,
                        max_seqlen=maxlen, H=H, Hkv=Hkv, D=D, causal=c["causal"],
                        dtype=c["dtype"])
    elif c["kind"] == "decode":
        B = c["B"] // world if c["shard"] else c["B"]
        H, Hkv, L, D = c["H"], c["Hkv"], c["L"], c["D"]
        q = torch.randn(B, H, 1, D, device=dev, generator=gen).to(tdt)
        k = torch.randn(B, Hkv, L, D, device=dev, generator=gen).to(tdt)
        v = torch.randn(B, Hkv, L, D, device=dev, generator=gen).to(tdt)
        work_per_step = 2 * B * Hkv * L * D * 2  # K+V bytes (fp16)
        unit = "GB/s"
        nsets = 1  # 4.3 GB of KV per step >> L2

        def step(i):
            return b200attn.decode(q, k, v, splits=c["splits"])

        if args.graph:
            from b200attn.graphs import CapturedDecode
            cap = CapturedDecode(q, k, v, splits=c["splits"])

            def step(i):  # noqa: F811
                return cap()

        kernel_regex = "decode_kernel"
        bound = "hbm"
        h2d = B * H * D * 2
        d2h = B * H * D * 2 + B * H * 4
        host_q = torch.randn(B, H, 1, D).to(tdt).pin_memory()
        host_out = (torch.empty(B, H, 1, D, dtype=tdt).pin_memory(),
                    torch.empty(B, H, 1, dtype=torch.float32).pin_memory())

        e2e_in = [host_q]
        static_out = bool(args.graph)

        def e2e_run(qd):
            return cap(qd) if args.graph else b200attn.decode(qd, k, v, splits=c["splits"])

        workload = dict(workload=c["name"], B=B, H=H, Hkv=Hkv, L=L, D=D, splits=c["splits"],
                        dtype=c["dtype"], kv_cache="resident (4.3 GB/step > L2)")
    elif c["kind"] == "kvshard":
        from b200attn.sharded import decode_kv_sharded
        B, H, Hkv, D = c["B"], c["H"], c["Hkv"], c["D"]
        assert c["L"] % world == 0
        Ll = c["L"] // world  # this rank's contiguous slice of the sequence
        q = torch.randn(B, H, 1, D, generator=torch.Generator().manual_seed(5)).to(tdt).to(dev)
        k = torch.randn(B, Hkv, Ll, D, device=dev, generator=gen).to(tdt)
        v = torch.randn(B, Hkv, Ll, D, device=dev, generator=gen).to(tdt)
        work_per_step = 2 * B * Hkv * Ll * D * 2  # this rank's K+V bytes
        unit = "GB/s"
        nsets = 1

        def step(i):
            return decode_kv_sharded(q, k, v, splits=c["splits"])

        if args.graph:
            from b200attn.graphs import CapturedDecode
            cap = CapturedDecode(q, k, v, splits=c["splits"], sharded=True)

            def step(i):  # noqa: F811
                return cap()

        kernel_regex = "decode_kernel"
        bound = "hbm"
        h2d = B * H * D * 2
        d2h = B * H * D * 2 + B * H * 4
        host_q = torch.randn(B, H, 1, D).to(tdt).pin_memory()
        host_out = (torch.empty(B, H, 1, D, dtype=tdt).pin_memory(),
                    torch.empty(B, H, 1, dtype=torch.float32).pin_memory())

        e2e_in = [host_q]
        static_out = bool(args.graph)

        def e2e_run(qd):
            return cap(qd) if args.graph else decode_kv_sharded(qd, k, v, splits=c["splits"])

        workload = dict(workload=c["name"], B=B, H=H, Hkv=Hkv, L=c["L"], L_per_rank=Ll, D=D,
                        splits_per_rank=c["splits"], dtype=c["dtype"],
                        collective="merged partials exchanged by one kernel over NVLink peer memory (B*H*(D+1) floats per rank)"
                                   if world > 1 else "none (1 rank)",
                        cuda_graph=bool(args.graph))
    else:  # paged
        lens_all = paged_lengths(c)
        # greedy balance of sequences over ranks by total length
        order = np.argsort(-lens_all)
        loads = [0] * world
        mine = []
        for idx in order:
            r = int(np.argmin(loads))
            loads[r] += lens_all[idx]
            if r == rank:
                mine.append(idx)
        lens = lens_all[sorted(mine)]
        B, H, Hkv, D, page = len(lens), c["H"], c["Hkv"], c["D"], c["page"]
        npages = -(-lens // page)
        P = int(npages.sum())
        perm = torch.randperm(P, generator=torch.Generator().manual_seed(77 + rank)).to(torch.int32)
        bt = torch.zeros(B, int(npages.max()), dtype=torch.int32)
        pos = 0
        for b in range(B):
            bt[b, :npages[b]] = perm[pos:pos + npages[b]]
            pos += npages[b]
        bt = bt.to(dev)
        kl = torch.tensor(lens, dtype=torch.int32, device=dev)
        kp = torch.randn(P, Hkv, page, D, device=dev, generator=gen).to(tdt)
        vp = torch.randn(P, Hkv, page, D, device=dev, generator=gen).to(tdt)
        q = torch.randn(B, H, 1, D, device=dev, generator=gen).to(tdt)
        work_per_step = int(lens.sum()) * Hkv * D * 2 * 2
        unit = "GB/s"
        nsets = 1

        def step(i):
            return b200attn.decode_paged(q, kp, vp, bt, kl, pages_per_split=c["pps"])

        kernel_regex = "decode_kernel"
        bound = "hbm"
        h2d = B * H * D * 2
        d2h = B * H * D * 2 + B * H * 4
        host_q = torch.randn(B, H, 1, D).to(tdt).pin_memory()
        host_out = (torch.empty(B, H, 1, D, dtype=tdt).pin_memory(),
                    torch.empty(B, H, 1, dtype=torch.float32).pin_memory())

        e2e_in = [host_q]
        static_out = False

        def e2e_run(qd):
            return b200attn.decode_paged(qd, kp, vp, bt, kl, pages_per_split=c["pps"])

        workload = dict(workload=c["name"], B=B, total_tokens=int(lens.sum()),
                        pages=P, pages_per_split=c["pps"], dtype=c["dtype"])

    return SimpleNamespace(c=c, step=step, nsets=nsets, work_per_step=work_per_step,
                           unit=unit, kernel_regex=kernel_regex, bound=bound, h2d=h2d,
                           d2h=d2h, e2e_in=e2e_in, host_out=host_out,
                           static_out=static_out, e2e_run=e2e_run, workload=workload)


def roofline_of(w, cfg_key, kernel_ms, clocks, peaks) -> dict:
    """Roofline object of a workload: algorithmic work per step over the median
    per-step device time, against the measured peak of its bound."""
    scale = 1e12 if w.unit == "TFLOP/s" else 1e9
    achieved = w.work_per_step / (kernel_ms / 1e3) / scale
    if w.bound == "tensor":
        # the burst GEMM figure for a kernel running at full clock, the sustained
        # one when the timed region ran under the power cap
        capped = "sw_power_cap" in clocks.get("reasons", []) or (
            clocks.get("sm_mhz") and clocks.get("sm_max_mhz")
            and clocks["sm_mhz"] < 0.9 * clocks["sm_max_mhz"])
        sustained = capped and peaks.get("bf16_tflops_sustained")
        pk = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
        peak_kind = " (sustained)" if sustained else " (burst)"
        runit = "TFLOP/s"
    else:
        pk = peaks["hbm_gbs"]
        peak_kind = ""
        runit = "GB/s"
    return {"bound": w.bound, "achieved": round(achieved, 2), "peak": pk, "unit": runit,
            "frac": round(achieved / pk, 4), "traffic": read_traffic(f"config{cfg_key}"),
            "traffic_source": "profiles/traffic.json: dram__bytes_read.sum + "
                              "dram__bytes_write.sum of one ncu capture, bytes per launch "
                              "(a stored figure, not measured by this run)",
            "peak_source": peaks["source"] + peak_kind,
            "kernel": w.kernel_regex, "launch_ms_median": round(kernel_ms, 5),
            "note": "achieved = algorithmic work per step / median per-step device time "
                    "(CUDA events on the launching stream, steps queued behind a GPU sleep so "
                    "that host launch gaps are not counted)"}


def kernel_step_times(torch, step, stream, first: int, n: int) -> list:
    """Device time of each of n steps, CUDA events around each on `stream`.  The
    launches queue behind a GPU-side sleep first, so the events measure the GPU
    work of a step and not the host's launch gaps."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    torch.cuda._sleep(int(min(n, 200) * 40e-6 * 2e9))   # ~40 us of host time per step
    for i in range(n):
        evs[i][0].record(stream)
        step(first + i)
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


SECONDARY = ("2", "4", "5a", "5b")


def run_secondary(args, rank, world, dev, clocks, peaks) -> dict:
    """Value and roofline of the other headline workloads -- config 2 (the
    reference's own headline shape), config 4 (split-KV decode, batch-sharded),
    config 5a (paged decode, sequences balanced over ranks) and config 5b (the
    KV-sharded decode with its NCCL all-gather) -- timed in the same process on
    the same box: warm-up, then K device-timed steps (max over ranks), then the
    per-step kernel time for the roofline."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    out = {}
    for key in SECONDARY:
        if key == args.config:
            continue
        w = make_workload(key, args, rank, world, dev)
        steps = 50 if w.c["kind"] in ("prefill", "kvshard") else 20
        for i in range(max(args.warmup, 3)):
            w.step(i)
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            w.step(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        kms = statistics.median(kernel_step_times(torch, w.step, stream, 0, steps))
        scale = 1e12 if w.unit == "TFLOP/s" else 1e9
        out[f"config{key}"] = {
            "workload": w.workload["workload"],
            "value": round(w.work_per_step * steps * world / (ms / 1e3) / scale, 3),
            "unit": w.unit, "steps": steps, "ms_per_step": round(ms / steps, 5),
            "scaling": "weak" if not w.c["shard"] else "strong",
            "parallelism": ("replicas" if not w.c["shard"] else "sharded") + f" x{world}",
            "l2": f"{w.nsets} rotating input sets" if w.nsets > 1 else "inputs larger than L2",
            "roofline": roofline_of(w, key, kms, clocks, peaks)}
        if "collective" in w.workload:
            out[f"config{key}"]["collective"] = w.workload["collective"]
        del w
        torch.cuda.empty_cache()
    return out



def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)
    w = make_workload(args.config, args, rank, world, dev)
    c, step, nsets, work_per_step, unit = w.c, w.step, w.nsets, w.work_per_step, w.unit
    kernel_regex, bound, h2d, d2h = w.kernel_regex, w.bound, w.h2d, w.d2h
    e2e_in, host_out, static_out, e2e_run = w.e2e_in, w.host_out, w.static_out, w.e2e_run
    workload = w.workload

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def keep_busy(samples_wanted: int):
        """Run untimed steps until the clock sampler has `samples_wanted` more
        samples (at most ~3 s).  Every rank runs the same number of steps: a
        step may contain a collective (KV-sharded decode), so the ranks agree on
        each round through a one-element MAX all-reduce instead of deciding
        from their own sampler."""
        t_end = time.time() + 3.0
        n = sampler.count()
        while True:
            more = (sampler.proc is not None and sampler.count() < n + samples_wanted
                    and time.time() < t_end)
            if world > 1:
                flag = torch.tensor([1 if more else 0], dtype=torch.int32, device=dev)
                dist.all_reduce(flag, op=dist.ReduceOp.MAX)
                more = bool(flag.item())
            if not more:
                return
            for i in range(4):
                step(i)
            torch.cuda.synchronize(dev)

    # ---- warm-up, started after the clock sampler so that the GPU is not left
    # idle between the warm-up and the timed region
    sampler = ClockSampler(local_rank)
    sampler.start()
    for i in range(args.warmup):
        step(i)
    keep_busy(2)  # until the sampler is producing samples

    # ---- timed device-resident region (barrier + synchronize on both sides)
    barrier()
    torch.cuda.synchronize(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = ev0.elapsed_time(ev1)
    # and keep it busy (untimed) until a sample after the timed region lands
    keep_busy(1)
    clocks = sampler.stop()

    # ---- per-step device time of the dominant kernel(s), for the roofline: a
    # separate pass, because events between steps add a few microseconds each
    step_ms = kernel_step_times(torch, step, stream, args.warmup, args.steps)

    # ---- end-to-end through the public API with host buffers.  Every step copies
    # its inputs host->device and its outputs device->host inside the timed
    # region; the copies run on their own streams, double-buffered, so that
    # step i+1's upload and step i-1's download overlap step i's compute.
    cp_in = torch.cuda.Stream(dev)
    cp_out = torch.cuda.Stream(dev)
    slots = [[torch.empty_like(h, device=dev) for h in e2e_in] for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_loop(n):
        for i in range(n):
            sl = i % 2
            with torch.cuda.stream(cp_in):
                if i >= 2:
                    cp_in.wait_event(ev_done[sl])  # slot's inputs consumed by step i-2
                for d, hsrc in zip(slots[sl], e2e_in):
                    d.copy_(hsrc, non_blocking=True)
                ev_in[sl].record(cp_in)
            stream.wait_event(ev_in[sl])
            if static_out and i >= 1:
                stream.wait_event(ev_out[(i - 1) % 2])  # graph outputs are reused
            outs = e2e_run(*slots[sl])
            ev_done[sl].record(stream)
            with torch.cuda.stream(cp_out):
                cp_out.wait_event(ev_done[sl])
                for o, hdst in zip(outs, host_out):
                    hdst.copy_(o, non_blocking=True)
                    o.record_stream(cp_out)
                ev_out[sl].record(cp_out)
        stream.wait_stream(cp_in)
        stream.wait_stream(cp_out)

    e2e_loop(3)
    torch.cuda.synchronize(dev)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    cp_in.wait_event(e0)
    cp_out.wait_event(e0)
    e2e_loop(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)

    # ---- max over ranks
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])

    scale = 1e12 if unit == "TFLOP/s" else 1e9
    total_work = work_per_step * args.steps * world
    value = total_work / (ms / 1e3) / scale
    e2e_value = total_work / (e2e_ms / 1e3) / scale

    peaks = read_peaks()
    kernel_ms = statistics.median(step_ms)
    roofline = roofline_of(w, args.config, kernel_ms, clocks, peaks)

    secondary = None
    if not args.no_secondary:
        secondary = run_secondary(args, rank, world, dev, clocks, peaks)

    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, u, sample, cores = cpu_sample(args.config, steps=2, warmup=1)
            cpu = {"value": round(v, 6), "unit": u, "cores": cores, "kind": "port",
                   "sample": sample}
        per_step = {"prefill": 1, "varlen": 1, "backward": 3}.get(c["kind"], 2)
        kernel_launches = args.steps * per_step  # timed region only
        out = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": unit,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak" if not c["shard"] else "strong",
            "vs_baseline": None,
            "dtype": "f16" if c["dtype"] == "float16" else "bf16",
            "data": "synthetic (seeded N(0,1), generated on device)",
            "config": {**workload,
                       "l2": f"{nsets} rotating input sets" if nsets > 1 else
                             "inputs larger than L2",
                       "parallelism": ("replicas" if not c["shard"] else "sharded") +
                                      f" x{world}"},
            "e2e": {"value": round(e2e_value, 3), "unit": unit,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": kernel_launches,
            "secondary": secondary,
            "clocks": clocks,
        }
    return out


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU naive attention (oracle port) on rank 0 only."""
    if rank != 0:
        return None
    c = CONFIGS[args.config]
    v, unit, sample, cores = cpu_sample(args.config, steps=args.steps, warmup=args.warmup)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 6),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak" if not c["shard"] else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": c["name"], "sample": sample},
        "cpu_baseline": {"value": round(v, 6), "unit": unit, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 6), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config 2 / config 4 lines timed after the main workload")
    ap.add_argument("--graph", action="store_true",
                    help="decode configs: replay each step as one captured CUDA graph")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    # Libraries (NCCL's version banner at communicator set-up) may write to fd 1;
    # keep stdout for the one JSON line by sending everything else to stderr.
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)

    if args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        if world > 1:
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        out = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if out is not None:
        sys.stdout.flush()
        json_out.write(json.dumps(out) + "\n")
        json_out.flush()


if __name__ == "__main__":
    main()
