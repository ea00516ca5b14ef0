"""Benchmark of the B200 paged-KV decode path (BASELINE.json metric:
paged-decode KV GB/s and decode tokens/s).

Default workload = BASELINE.json configs[1], "Llama-3-8B-shape batched decode":
bf16, 32 layers each with its own paged pool, batch 256, 32 q / 8 kv heads,
head_dim 128, block_size 16, context lengths uniform in [512, 4096] (seeded),
K/V ~ N(0, 1).  One step = for every layer, append one new token per sequence
through reshape_and_cache, then paged_attention_v1 over context + 1 tokens.
A step emits 256 tokens (one per sequence).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5]
    python bench.py --impl reference ...     # CPU reference arm

Multi-GPU (torchrun, one process per GPU): the KV pool is sharded by KV head
(rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their q heads); block tables
and lengths are replicated; no collective runs in the data path.  Total work
is fixed, so scaling is strong.  Timing: CUDA events on the launching stream,
barrier + synchronize around the timed region, max over ranks.

The per-layer KV cache (2.4 GB) is far larger than L2 (126 MB), so no L2
flush is needed between iterations.  Inputs are synthetic (seeded N(0,1));
torch fills the device caches (plumbing); every timed kernel is libkvcache's.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sglang-mlx_b200"))
sys.path.insert(0, ROOT)

METRIC = "paged-decode KV GB/s (% of HBM peak) and decode tokens/s"


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one decode launch, from the ncu captures
# summarised in profiles/ (config 2: captured at batch 64 and scaled by KV bytes to the full launch).
TRAFFIC_PER_LAUNCH = {
    2: (2.289e9 + 0.016e9, "profiles/paged_decode_mma_bs16_small.md (batch-64 capture scaled to batch 256)"),
    3: (537.1e6 + 9.8e6, "profiles/paged_decode_mma_bs32_config3.md (partition kernel; reduce adds 8.6e6)"),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
CONFIGS = {
    2: dict(name="llama3-8b-batched-decode", layers=32, batch=256, hq=32, hkv=8, d=128, bs=16, lo=512, hi=4096,
            dtype="bfloat16", partition=0),
    3: dict(name="128k-batch1-splitk-decode", layers=1, batch=1, hq=64, hkv=8, d=128, bs=32, lo=131072,
            hi=131072, dtype="bfloat16", partition=512),
}


def context_lengths(cfg, seed=2024):
    rng = np.random.default_rng(seed)
    return rng.integers(cfg["lo"], cfg["hi"] + 1, size=cfg["batch"]).astype(np.int64)


def build_tables(lens_after, bs, seed=7):
    """Seeded random permutation of the pool's blocks, ceil((C+1)/bs) per sequence."""
    rng = np.random.default_rng(seed)
    nblk = [(-(-int(c) // bs)) for c in lens_after]
    total = int(sum(nblk))
    perm = rng.permutation(total).astype(np.int32)
    mb = max(nblk)
    tables = np.zeros((len(lens_after), mb), np.int32)
    o = 0
    for b, n in enumerate(nblk):
        tables[b, :n] = perm[o:o + n]
        tables[b, n:] = perm[o]  # padding never read
        o += n
    return tables, total


def algorithmic_bytes(lens_after, hq, hkv, d, bs, s_cache=2, s_q=2, s_out=2):
    """Decode bytes per launch (per layer): KV read + q read + out write + table
    entries + lengths."""
    kv = int(np.sum(lens_after)) * hkv * d * s_cache * 2
    qo = len(lens_after) * hq * d * (s_q + s_out)
    tab = int(np.sum(-(-lens_after // bs))) * 4 + len(lens_after) * 4
    return kv + qo + tab


# ---------------------------------------------------------------------------
# clocks sampling
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"kvc_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port, C + OpenMP, float64 gather + SDPA)
# ---------------------------------------------------------------------------
def cpu_sample(cfg, lens_after, tables, kcache_np_fn, vcache_np_fn, q_np, hkv_local, n_seq, budget_s=10.0):
    """Times the oracle on `n_seq` sequences of one layer, repeated up to
    `budget_s`; returns seconds per (one layer, n_seq sequences)."""
    from oracle import c_oracle

    bs = cfg["bs"]
    sel = np.arange(n_seq)
    nblk = [(-(-int(lens_after[b]) // bs)) for b in sel]
    blocks = np.concatenate([tables[b, :n] for b, n in zip(sel, nblk)]).astype(np.int64)
    kc = kcache_np_fn(blocks)
    vc = vcache_np_fn(blocks)
    mb = max(nblk)
    t2 = np.zeros((n_seq, mb), np.uint32)
    o = 0
    for i, n in enumerate(nblk):
        t2[i, :n] = np.arange(o, o + n)
        o += n
    lens = lens_after[sel].astype(np.uint32)
    q = q_np[sel]
    threads = c_oracle.num_threads()
    reps, t0 = 0, time.perf_counter()
    while True:
        c_oracle.paged_attention(q, "bfloat16", kc, vc, "bfloat16", t2, lens, hkv_local, 1.0 / math.sqrt(cfg["d"]),
                                 int(mb * bs), threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 2000:
            break
    return el / reps, threads


def lscpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, cfg, rank, world):
    """The reference's own CPU path is MLX (gather + mx.fast.scaled_dot_product_attention),
    not installed here; the oracle port (same dataflow, float64, all host cores) runs
    instead on a bounded sample of the same workload, scaled to the full step."""
    if rank != 0:
        return
    from oracle import c_oracle

    lens = context_lengths(cfg)
    lens_after = lens + 1
    tables, total_blocks = build_tables(lens_after, cfg["bs"])
    n_seq = 8 if cfg["batch"] >= 8 else cfg["batch"]
    rng = np.random.default_rng(99)
    bs, d, hkv, hq = cfg["bs"], cfg["d"], cfg["hkv"], cfg["hq"]
    sel_blocks = sum(-(-int(lens_after[b]) // bs) for b in range(n_seq))

    def rand_bits(shape):
        return rng.standard_normal(shape, dtype=np.float32).view(np.uint32).__rshift__(16).astype(np.uint16)

    kc = rand_bits((sel_blocks, hkv, d // 8, bs, 8))
    vc = rand_bits((sel_blocks, hkv, d, bs))
    q = rand_bits((n_seq, hq, d))
    t2 = np.zeros((n_seq, tables.shape[1]), np.uint32)
    o = 0
    for b in range(n_seq):
        n = -(-int(lens_after[b]) // bs)
        t2[b, :n] = np.arange(o, o + n)
        o += n
    threads = c_oracle.num_threads()
    scale_factor = (cfg["batch"] / n_seq) * cfg["layers"]
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        c_oracle.paged_attention(q, "bfloat16", kc, vc, "bfloat16", t2, lens_after[:n_seq].astype(np.uint32), hkv,
                                 1.0 / math.sqrt(d), int(tables.shape[1] * bs), threads=threads)
        el = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(el)
    step_s = float(np.mean(times)) * scale_factor
    toks = cfg["batch"] / step_s
    sample = (f"{n_seq} of {cfg['batch']} sequences x 1 of {cfg['layers']} layers per step, scaled x"
              f"{scale_factor:g}; C oracle port (float64 gather+SDPA), {threads} threads, {lscpu_model()}")
    line = {"metric": METRIC, "value": toks, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["name"], "global_batch": cfg["batch"], "layers": cfg["layers"],
                       "heads": f"{hq}q/{hkv}kv", "head_dim": d, "block_size": bs,
                       "context": f"U[{cfg['lo']},{cfg['hi']}]"},
            "cpu_baseline": {"value": toks, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": toks, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, cfg, rank, world, local_rank):
    import torch

    from sglang_mlx_b200 import _lib
    from sglang_mlx_b200 import metal_kernels as mk
    from sglang_mlx_b200.device_array import DeviceArray, Event, HostBuffer

    dev = local_rank
    _lib.set_device(dev)
    torch.cuda.set_device(dev)
    tdev = torch.device("cuda", dev)
    from sglang_mlx_b200 import sharding

    L, B_all, HQ, HKV, D, BS = cfg["layers"], cfg["batch"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"]
    lens_all = context_lengths(cfg)
    plan = sharding.plan(HQ, HKV, world, rank, lens_all + 1)
    hkv, hq = plan.num_kv_heads, plan.num_q_heads
    lens = lens_all[plan.seqs]
    B = len(lens)
    lens_after = lens + 1
    tables, total_blocks = build_tables(lens_after, BS)
    max_seq_len = int(tables.shape[1] * BS)
    slots = (tables[np.arange(B), lens // BS].astype(np.int64) * BS + lens % BS).astype(np.int32)

    g = torch.Generator(device=tdev)
    g.manual_seed(1234 + rank)
    tdt = torch.bfloat16
    kc_t, vc_t, kc, vc = [], [], [], []
    for _ in range(L):
        k = torch.randn((total_blocks, hkv, D // 8, BS, 8), generator=g, device=tdev, dtype=tdt)
        v = torch.randn((total_blocks, hkv, D, BS), generator=g, device=tdev, dtype=tdt)
        kc_t.append(k)
        vc_t.append(v)
        kc.append(DeviceArray.from_dlpack(k))
        vc.append(DeviceArray.from_dlpack(v))
    q_t = torch.randn((L, B, hq, D), generator=g, device=tdev, dtype=tdt)
    kn_t = torch.randn((L, B, hkv, D), generator=g, device=tdev, dtype=tdt)
    vn_t = torch.randn((L, B, hkv, D), generator=g, device=tdev, dtype=tdt)
    q = [DeviceArray.from_dlpack(q_t[i]) for i in range(L)]
    kn = [DeviceArray.from_dlpack(kn_t[i]) for i in range(L)]
    vn = [DeviceArray.from_dlpack(vn_t[i]) for i in range(L)]
    out = [DeviceArray.empty((B, hq, D), "bfloat16", dev) for _ in range(L)]
    tables_d = DeviceArray.from_numpy(tables, device=dev)
    lens_d = DeviceArray.from_numpy(lens_after.astype(np.int32), device=dev)
    slots_d = DeviceArray.from_numpy(slots, device=dev)
    scale = 1.0 / math.sqrt(D)
    # config 3 fixes 512-token partitions; otherwise the shim's heuristic decides
    # (single pass at N = 1 for config 2, split-K once head sharding leaves too few CTAs)
    psize = cfg["partition"] or mk.choose_decode(B, hkv, max_seq_len, BS)
    if args.decode == "v1":
        psize = 0
    elif args.decode == "v2":
        psize = args.partition or psize or 512
    if args.partition and psize:
        psize = args.partition
    split = psize > 0
    ws = mk.splitk_workspace(B, hq, D, max_seq_len, psize, dev) if split else None
    torch.cuda.synchronize()

    def decode(i, o=None):
        if split:
            return mk.paged_attention_v2(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len,
                                         partition_size=psize, workspace=ws, out=o or out[i])
        return mk.paged_attention_v1(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len,
                                     out=o or out[i])

    def step(ev=None):
        for i in range(L):
            mk.reshape_and_cache(kn[i], vn[i], kc[i], vc[i], slots_d)
            if ev is not None:
                ev[i][0].record()
            decode(i)
            if ev is not None:
                ev[i][1].record()

    dist = None
    if world > 1:
        import torch.distributed as dist
    def barrier():
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    _lib.synchronize()

    # ---- timed region (device-resident inputs) ----
    evs = [[[Event(), Event()] for _ in range(L)] for _ in range(args.steps)]
    start, end = Event(), Event()
    sampler = ClockSampler(dev)
    barrier()
    _lib.synchronize()
    sampler.start()
    launches0 = _lib.launch_count()
    start.record()
    for s in range(args.steps):
        step(evs[s])
    end.record()
    end.synchronize()
    _lib.synchronize()
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop()
    total_ms = start.elapsed_ms(end)
    dec_ms = [evs[s][i][0].elapsed_ms(evs[s][i][1]) for s in range(args.steps) for i in range(L)]
    barrier()

    # ---- e2e through the public API with pinned host buffers ----
    h_q = [HostBuffer((B, hq, D), "bfloat16") for _ in range(L)]
    h_k = [HostBuffer((B, hkv, D), "bfloat16") for _ in range(L)]
    h_v = [HostBuffer((B, hkv, D), "bfloat16") for _ in range(L)]
    h_o = [HostBuffer((B, hq, D), "bfloat16") for _ in range(L)]
    rng = np.random.default_rng(5 + rank)
    for i in range(L):
        for hb in (h_q[i], h_k[i], h_v[i]):
            hb.array[...] = rng.integers(0x3c00, 0x4000, size=hb.shape, dtype=np.uint16)
    h_lens = HostBuffer((B,), "int32")
    h_lens.array[...] = lens_after
    h_slots = HostBuffer((B,), "int32")
    h_slots.array[...] = slots

    def e2e_step():
        lens_d.copy_from_host(h_lens)
        slots_d.copy_from_host(h_slots)
        for i in range(L):
            q[i].copy_from_host(h_q[i])
            kn[i].copy_from_host(h_k[i])
            vn[i].copy_from_host(h_v[i])
            mk.reshape_and_cache(kn[i], vn[i], kc[i], vc[i], slots_d)
            decode(i)
            out[i].copy_to_host(h_o[i])

    e2e_ms = float("nan")
    if not args.no_e2e:
        for _ in range(max(1, args.warmup)):
            e2e_step()
        _lib.synchronize()
        barrier()
        e0, e1 = Event(), Event()
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        e1.synchronize()
        e2e_ms = e0.elapsed_ms(e1)
    h2d = (B * 4 * 2) + L * (B * hq * D * 2 + 2 * B * hkv * D * 2)
    d2h = L * B * hq * D * 2

    # ---- reduce over ranks (max time; KV bytes summed) ----
    step_ms = total_ms / args.steps
    e2e_step_ms = e2e_ms / args.steps
    mean_dec_ms = float(np.mean(dec_ms))
    alg = algorithmic_bytes(lens_after, hq, hkv, D, BS)
    alg_all = float(alg)
    if dist is not None:
        t = torch.tensor([step_ms, e2e_step_ms, mean_dec_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_step_ms, mean_dec_ms_max = [float(x) for x in t]
        s = torch.tensor([float(alg)], dtype=torch.float64)
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        alg_all = float(s[0])
    else:
        mean_dec_ms_max = mean_dec_ms

    if rank != 0:
        return
    peak, peak_kind = load_peaks()
    # the capture is of the default workload on one GPU; other shapes report null
    traffic = TRAFFIC_PER_LAUNCH.get(args.config) if (world == 1 and not (args.layers or args.batch)) else None
    achieved = alg / (mean_dec_ms * 1e-3) / 1e9
    toks = B_all / (step_ms * 1e-3)
    kv_bytes_step = L * alg_all
    line = {
        "metric": METRIC,
        "value": toks,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": cfg["name"], "global_batch": B_all, "layers": L, "heads": f"{HQ}q/{HKV}kv",
                   "head_dim": D, "block_size": BS, "context": f"U[{cfg['lo']},{cfg['hi']}] (seeded)",
                   "parallelism": f"kv-head-shard{world}", "l2": "inputs larger than L2 (KV per layer "
                   f"{alg * world / 1e9:.2f} GB); no flush",
                   "kernel": f"split-K v2, {psize}-token partitions" if split else "paged_attention_v1"},
        "kv_gbs": kv_bytes_step / (step_ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic[0] if traffic else None,
                     "traffic_source": traffic[1] if traffic else None,
                     "peak_kind": peak_kind, "kernel": "paged decode (per layer launch)",
                     "algorithmic_bytes_per_launch": alg, "mean_launch_ms": mean_dec_ms},
        "e2e": None if args.no_e2e else {"value": B_all / (e2e_step_ms * 1e-3), "unit": "tokens/s",
                                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        n_seq = 8
        sel_lens = lens_after

        def kfn(blocks):
            idx = torch.from_numpy(blocks).to(tdev)
            return kc_t[0].index_select(0, idx).view(torch.int16).cpu().numpy().view(np.uint16)

        def vfn(blocks):
            idx = torch.from_numpy(blocks).to(tdev)
            return vc_t[0].index_select(0, idx).view(torch.int16).cpu().numpy().view(np.uint16)

        q_np = q_t[0].view(torch.int16).cpu().numpy().view(np.uint16)
        t_sample, threads = cpu_sample(cfg, sel_lens, tables, kfn, vfn, q_np, hkv, n_seq)
        scale_factor = (B / n_seq) * L
        cpu_step = t_sample * scale_factor
        line["cpu_baseline"] = {"value": B / cpu_step, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{n_seq} of {B} sequences x 1 of {L} layers, scaled x{scale_factor:g}; "
                                          f"C oracle (float64 gather+SDPA, OpenMP), {lscpu_model()}"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--decode", default="auto", choices=["auto", "v1", "v2"],
                    help="decode form: the shim's choice (default), single pass, or split-K")
    ap.add_argument("--partition", type=int, default=0, help="split-K partition size (tokens) when split")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling cases only)")
    ap.add_argument("--batch", type=int, default=0, help="override the batch (profiling cases only)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    cfg = dict(CONFIGS[args.config])
    if args.layers or args.batch:
        cfg["layers"] = args.layers or cfg["layers"]
        cfg["batch"] = args.batch or cfg["batch"]
        cfg["name"] += f" (reduced: {cfg['layers']} layers, batch {cfg['batch']})"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            run_reference(args, cfg, rank, world)
        else:
            run_ours(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
