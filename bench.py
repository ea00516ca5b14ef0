"""Benchmark of the B200 paged-KV decode path (BASELINE.json metric:
paged-decode KV GB/s and decode tokens/s).

Default workload = BASELINE.json configs[1], "Llama-3-8B-shape batched decode":
bf16, 32 layers each with its own paged pool, batch 256, 32 q / 8 kv heads,
head_dim 128, block_size 16, context lengths uniform in [512, 4096] (seeded),
K/V ~ N(0, 1).  One step = for every layer, append one new token per sequence
through reshape_and_cache, then the decode over context + 1 tokens.  A step
emits 256 tokens (one per sequence).  On one GPU the same JSON line also
carries configs 3, 4 and 5 (`other_configs`), each timed the same way.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5]
    python bench.py --impl reference ...     # CPU reference arm

--config 3: 128k batch-1 decode, split-K with 512-token partitions + LSE reduce.
--config 4: 64 sequences sharing one 2048-token prefix (same block ids) + 256
            unique tail tokens; the unique footprint (75.5 MB) fits in L2, so L2
            is flushed between steps and the roofline counts unique bytes.
--config 5: mixed continuous-batch step: 16 prefill chunks of 512 tokens
            appended together with 512 decode tokens, then the decode of 512
            sequences with lognormal lengths (block 32, 28 q / 4 kv heads).

Multi-GPU (torchrun, one process per GPU): the KV pool is sharded by KV head
(sglang_mlx_b200.sharding; heads x sequences when there are fewer KV heads than
GPUs); block tables and lengths are replicated; no collective runs in the data
path.  Total work is fixed, so scaling is strong.  Timing: CUDA events on the
launching stream, barrier + synchronize around the timed region, max over ranks.
After timing, every rank checks a sample of its own outputs against the CPU
oracle (float64 gather + SDPA) and the run fails if any rank is off.

Inputs are synthetic (seeded N(0,1)); torch fills the device caches
(plumbing); every timed kernel is libkvcache's.
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
for _p in (os.path.join(ROOT, "tests", "golden"), os.path.join(ROOT, "sglang-mlx_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import cases  # noqa: E402  (seeded BASELINE workloads)

METRIC = "paged-decode KV GB/s (% of HBM peak) and decode tokens/s"

CONTEXT_DESC = {
    2: "U[512,4096] (seeded)",
    3: "131072",
    4: "2048-token shared prefix + 256 unique",
    5: "lognormal(median 1500, sigma 1.0) clipped to [16, 32768] (seeded)",
}

# ncu-measured DRAM traffic per decode launch (the profiles/ summaries name the commands)
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "dram_traffic_per_launch.json")

L2_FLUSH_BYTES = 512 << 20  # > 4x the 126 MB L2

ATOL, RTOL = 2e-3, 1e-2  # north-star tolerance of bf16 attention outputs


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(config: int, kernel_key: str):
    """(bytes per launch, description) of an ncu capture of this workload's decode, or None."""
    try:
        with open(TRAFFIC_FILE) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return None
    e = d.get(f"config{config}/{kernel_key}")
    if not e:
        return None
    return float(e["bytes_per_launch"]), e["how"]


def host_threads() -> int:
    """Host threads for the CPU legs: every core this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def decode_bytes(tables, lens_after, hq, hkv, d, bs, shared: bool, s=2, s_kv=None):
    """Algorithmic bytes of one decode launch: K/V read (distinct blocks once when
    blocks are shared), q read, output write, table entries, lengths.  Also
    returns the logical K/V bytes (every sequence's tokens counted).  `s_kv` is
    the cache element size (1 for FP8 caches), `s` that of q and out."""
    s_kv = s if s_kv is None else s_kv
    logical = int(np.sum(lens_after)) * hkv * d * s_kv * 2
    kv = cases.unique_kv_bytes(tables, lens_after, hkv, d, bs, s_kv) if shared else logical
    qo = len(lens_after) * hq * d * (s + s)
    tab = int(np.sum(-(-np.asarray(lens_after) // bs))) * 4 + len(lens_after) * 4
    return kv + qo + tab, logical


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
        self.path = os.path.join("/tmp", f"kvc_clocks_{os.getpid()}_{index}.csv")

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


def lscpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# CPU legs: the reference's serving dataflow (gather the sequence's K/V token
# rows out of the pool, then scaled-dot-product attention) restated on the host
# ---------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    u = bits.astype(np.uint32)
    np.left_shift(u, np.uint32(16), out=u)  # in place: a Python-int shift is far slower here
    return u.view(np.float32)


def numpy_gather_sdpa(q_bits, kc_bits, vc_bits, tables, lens, hkv, scale, bs, threads):
    """fp32 gather + SDPA of a batch, the dataflow of the reference's
    gather-then-mx.fast.scaled_dot_product_attention path
    (bench_paged_vs_gather.py:83-103; PooledKVCache.update_and_fetch + SDPA):
    per sequence, its blocks' K/V token rows are gathered out of the paged
    cache into token-major fp32 arrays, then softmax(q K^T * scale) V with the
    GQA broadcast, as batched BLAS matmuls.  Sequences are spread over
    `threads` worker threads (NumPy releases the GIL in the copies and BLAS
    calls, which run single-threaded each)."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    B, Hq, D = q_bits.shape
    G = Hq // hkv
    qf = bf16_bits_to_f32(q_bits)
    out = np.empty((B, Hq, D), np.float32)

    def rows(b0, b1):
        for b in range(b0, b1):
            C = int(lens[b])
            nb = -(-C // bs)
            blk = tables[b, :nb]
            K = bf16_bits_to_f32(kc_bits[blk]).transpose(1, 0, 3, 2, 4).reshape(hkv, nb * bs, D)[:, :C]
            V = bf16_bits_to_f32(vc_bits[blk]).transpose(1, 0, 3, 2).reshape(hkv, nb * bs, D)[:, :C]
            s = np.matmul(qf[b].reshape(hkv, G, D), K.transpose(0, 2, 1))
            s *= np.float32(scale)
            s -= s.max(axis=-1, keepdims=True)
            np.exp(s, out=s)
            l_ = s.sum(axis=-1, keepdims=True)
            out[b] = (np.matmul(s, V) / l_).reshape(Hq, D)

    cuts = np.linspace(0, B, num=min(B, 4 * threads) + 1).astype(int)
    with threadpool_limits(1), ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda i: rows(cuts[i], cuts[i + 1]), range(len(cuts) - 1)))
    return out


def c_float64_gather_sdpa(q_bits, kc_bits, vc_bits, tables, lens, hkv, scale, bs, threads):
    """The C oracle (float64 gather + SDPA, OpenMP over sequences)."""
    from oracle import c_oracle

    return c_oracle.paged_attention(q_bits, "bfloat16", kc_bits, vc_bits, "bfloat16", tables,
                                    np.asarray(lens).astype(np.uint32), hkv, scale, int(tables.shape[1] * bs),
                                    threads=threads)


def mlx_probe():
    """The reference's own CPU path needs MLX (mx.fast.scaled_dot_product_attention)."""
    try:
        import mlx.core  # noqa: F401
        return "importable"
    except Exception as e:  # noqa: BLE001
        return f"not importable ({type(e).__name__})"


def workload(args, config=None):
    config = config or args.config
    w = cases.baseline_workload(config, batch=args.batch or None)
    cfg = dict(w["cfg"])
    if args.layers and config == args.config:
        cfg["layers"] = args.layers
    if (args.layers or args.batch or args.kv_heads) and config == args.config:
        cfg["name"] += f" (reduced: {cfg['layers']} layers, batch {cfg['batch']}, kv heads {args.kv_heads or cfg['hkv']})"
    return w, cfg


def config_json(cfg, config, world, extra=None):
    d = {"workload": cfg["name"], "global_batch": cfg["batch"], "layers": cfg["layers"],
         "heads": f"{cfg['hq']}q/{cfg['hkv']}kv", "head_dim": cfg["d"], "block_size": cfg["bs"],
         "context": CONTEXT_DESC[config], "parallelism": f"kv-head-shard{world}"}
    if cfg.get("prefill_chunks"):
        d["prefill"] = f"{cfg['prefill_chunks']} chunks x {cfg['chunk']} tokens appended per step"
    if extra:
        d.update(extra)
    return d


def random_bf16_bits(rng, shape, chunk=1 << 24):
    """N(0, 1) values as bf16 bits, generated in chunks."""
    out = np.empty(int(np.prod(shape)), np.uint16)
    for o in range(0, out.size, chunk):
        n = min(chunk, out.size - o)
        out[o:o + n] = rng.standard_normal(n, dtype=np.float32).view(np.uint32) >> 16
    return out.reshape(shape)


def cpu_legs(cfg, w, threads, reps=1):
    """Times both host legs over one full layer of the workload (all sequences):
    (fp32 NumPy/BLAS seconds, float64 C seconds), means over `reps`."""
    lens_after = w["lens"] + 1
    bs, d, hkv, hq, B = cfg["bs"], cfg["d"], cfg["hkv"], cfg["hq"], cfg["batch"]
    tables = np.ascontiguousarray(w["tables"])
    rng = np.random.default_rng(99)
    kc = random_bf16_bits(rng, (w["num_blocks"], hkv, d // 8, bs, 8))
    vc = random_bf16_bits(rng, (w["num_blocks"], hkv, d, bs))
    q = random_bf16_bits(rng, (B, hq, d))
    scale = 1.0 / math.sqrt(d)
    t_np, t_c = [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        numpy_gather_sdpa(q, kc, vc, tables, lens_after, hkv, scale, bs, threads)
        t1 = time.perf_counter()
        c_float64_gather_sdpa(q, kc, vc, tables, lens_after, hkv, scale, bs, threads)
        t2 = time.perf_counter()
        t_np.append(t1 - t0)
        t_c.append(t2 - t1)
    return float(np.mean(t_np)), float(np.mean(t_c))


def cpu_baseline_entry(cfg, w, threads, reps):
    """The faster of the two host legs as the baseline (tokens/s), the other beside it."""
    L, B = cfg["layers"], cfg["batch"]
    t_np, t_c = cpu_legs(cfg, w, threads, reps)
    legs = {"numpy_fp32_blas": B / (t_np * L), "c_float64_openmp": B / (t_c * L)}
    best = max(legs, key=legs.get)
    what = {"numpy_fp32_blas": "fp32 NumPy/BLAS gather + SDPA", "c_float64_openmp": "float64 C gather + SDPA (OpenMP)"}
    return {"value": legs[best], "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"all {B} sequences x 1 of {L} layers per rep ({reps} reps), scaled x{L}; the faster of two "
                      f"restatements of the reference's gather-then-SDPA dataflow: {what[best]} "
                      f"(legs: {', '.join(f'{k} {v:.3g}' for k, v in legs.items())} tokens/s); {lscpu_model()}",
            "leg": best, "legs_tokens_per_s": legs}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The reference's own CPU path is MLX's gather + mx.fast.scaled_dot_product_attention;
    MLX is not installed on these hosts (probed: `mlx` below), so its dataflow is
    restated twice, an fp32 NumPy/BLAS gather + SDPA and the float64 C port, both
    on every host thread, each step one full layer of the workload (all
    sequences) scaled to the step's layers; `value` is the faster leg."""
    if rank != 0:
        return
    w, cfg = workload(args)
    B = cfg["batch"]
    threads = host_threads()
    if args.warmup:
        cpu_legs(cfg, w, threads, 1)
    entry = cpu_baseline_entry(cfg, w, threads, max(1, args.steps))
    toks = entry["value"]
    step_s = B / toks
    line = {"metric": METRIC, "value": toks, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": min(args.warmup, 1), "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": config_json(cfg, args.config, world), "cpu_baseline": entry, "mlx": mlx_probe(),
            "e2e": {"value": toks, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def check_outputs(torch, q_t, kc_t, vc_t, out, tables, lens_after, hkv, D, bs, mode, fmt=None):
    """A sample of this rank's sequences (first, middle, last) of one layer
    against the CPU oracle: float64 gather + SDPA over the rank's own caches.
    Returns (ok, max |err|, rows checked)."""
    from oracle import c_oracle, kv_oracle

    B = len(lens_after)
    rows = sorted({0, B // 2, B - 1})
    dev = kc_t.device
    got = out.to_numpy()[rows]
    nb = [(-(-int(lens_after[b]) // bs)) for b in rows]
    ids = np.concatenate([tables[b, :n] for b, n in zip(rows, nb)]).astype(np.int64)
    t2 = np.zeros((len(rows), max(nb)), np.uint32)
    o = 0
    for i, n in enumerate(nb):
        t2[i, :n] = np.arange(o, o + n)
        o += n
    idx = torch.from_numpy(ids).to(dev)
    kg, vg = kc_t.index_select(0, idx), vc_t.index_select(0, idx)
    qr = q_t.index_select(0, torch.tensor(rows, device=dev))
    scale = 1.0 / math.sqrt(D)

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    if mode == "fp8":
        kq = kv_oracle.dequantize(kg.cpu().numpy(), 0.05, fmt)
        vq = kv_oracle.dequantize(vg.cpu().numpy(), 0.05, fmt)
        ref = kv_oracle.paged_attention_v1(bf16_bits_to_f32(bits(qr)), kq, vq, t2, lens_after[rows], hkv, scale, bs,
                                           int(t2.shape[1] * bs))
    else:
        kb, vb = bits(kg), bits(vg)
        if mode == "pool":  # token rows [n, H, D] = paged pages of one token
            kb = kb.reshape(kb.shape[0], hkv, D // 8, 1, 8)
            vb = vb.reshape(vb.shape[0], hkv, D, 1)
        ref = c_oracle.paged_attention(bits(qr), "bfloat16", kb, vb, "bfloat16", t2, lens_after[rows], hkv, scale,
                                       int(t2.shape[1] * bs))
    ok, err, _ = kv_oracle.allclose_report(got, ref, ATOL, RTOL)
    return bool(ok and np.isfinite(got).all()), float(err), len(rows)


def measure_decode(args, config, rank, world, local_rank, top=True):
    """Times `config` on this rank's share; returns the JSON line (rank 0) or None.
    top=False (the other configs of a one-GPU run): no e2e, no CPU baseline."""
    import torch

    from sglang_mlx_b200 import _lib, sharding
    from sglang_mlx_b200 import metal_kernels as mk
    from sglang_mlx_b200.device_array import DeviceArray, Event, Graph, HostBuffer, Stream

    dev = local_rank
    tdev = torch.device("cuda", dev)
    w, cfg = workload(args, config)
    L, B_all, HQ, HKV, D, BS = cfg["layers"], cfg["batch"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"]
    if args.kv_heads and top:  # profiling: one rank's share of a head-sharded run, on one GPU
        HQ, HKV = HQ * args.kv_heads // HKV, args.kv_heads
        cfg["hq"], cfg["hkv"] = HQ, HKV
    plan = sharding.plan(HQ, HKV, world, rank, w["lens"] + 1)
    hkv, hq = plan.num_kv_heads, plan.num_q_heads
    lens = w["lens"][plan.seqs]
    B = len(lens)
    lens_after = lens + 1
    tables = np.ascontiguousarray(w["tables"][plan.seqs])
    max_seq_len = w["max_seq_len"]
    num_blocks = w["num_blocks"]
    # new tokens appended this step: this rank's share of the prefill chunks, then one per decode sequence
    pre = w["prefill_slots"]
    if len(pre) and HKV < world:
        group = world // HKV
        chunk = cfg["chunk"]
        mine = [c for c in range(cfg["prefill_chunks"]) if c % group == rank % group]
        pre = np.concatenate([pre[c * chunk:(c + 1) * chunk] for c in mine]) if mine else pre[:0]
    slots = np.concatenate([pre, w["decode_slots"][plan.seqs]]).astype(np.int32)
    T_new = len(slots)
    shared = config == 4
    pool = args.layout in ("pool", "pool-pages") and top
    pool_pages = args.layout == "pool-pages" and top  # the pool read through page tables (page_size = block size)
    fp8 = args.kv_dtype.startswith("fp8") and top
    fmt = args.kv_dtype[4:] if fp8 else None
    if fp8 and (pool or args.decode == "cascade"):
        raise SystemExit("--kv-dtype fp8 runs on the paged layout with the single-pass / split-K / planned decode")
    page_tables = tables
    if pool:
        # MHATokenPool layout: block b's tokens are slots b*BS+1 .. b*BS+BS (slot 0 is
        # the pool's padding slot), i.e. block b is page b of a page-granular pool; the
        # slot-list form of the tables lists every token's slot
        t = np.arange(tables.shape[1] * BS)
        blk = tables[:, t // BS].astype(np.int64)
        tables = np.ascontiguousarray(np.where(blk >= 0, blk * BS + t % BS + 1, 0).astype(np.int32))
        slots = (slots.astype(np.int64) + 1).astype(np.int32)
    tab_bs = 1 if pool else BS

    g = torch.Generator(device=tdev)
    g.manual_seed(1234 + rank)
    tdt = torch.bfloat16
    kc_t, vc_t, kc, vc = [], [], [], []
    for _ in range(L):
        if pool:
            k = torch.randn((num_blocks * BS + 1, hkv, D), generator=g, device=tdev, dtype=tdt)
            v = torch.randn((num_blocks * BS + 1, hkv, D), generator=g, device=tdev, dtype=tdt)
        elif fp8:
            # finite codes only (exponent field below all-ones), random sign
            top_code = 0x78 if fmt == "e4m3" else 0x7C
            k = (torch.randint(0, top_code, (num_blocks, hkv, D // 16, BS, 16), generator=g, device=tdev,
                               dtype=torch.int32)
                 | (torch.randint(0, 2, (1,), generator=g, device=tdev, dtype=torch.int32) << 7)).to(torch.uint8)
            v = (torch.randint(0, top_code, (num_blocks, hkv, D, BS), generator=g, device=tdev, dtype=torch.int32)
                 | (torch.randint(0, 2, (1,), generator=g, device=tdev, dtype=torch.int32) << 7)).to(torch.uint8)
        else:
            k = torch.randn((num_blocks, hkv, D // 8, BS, 8), generator=g, device=tdev, dtype=tdt)
            v = torch.randn((num_blocks, hkv, D, BS), generator=g, device=tdev, dtype=tdt)
        kc_t.append(k)
        vc_t.append(v)
        kc.append(DeviceArray.from_dlpack(k))
        vc.append(DeviceArray.from_dlpack(v))
    q_t = torch.randn((L, B, hq, D), generator=g, device=tdev, dtype=tdt)
    kn_t = torch.randn((L, T_new, hkv, D), generator=g, device=tdev, dtype=tdt)
    vn_t = torch.randn((L, T_new, hkv, D), generator=g, device=tdev, dtype=tdt)
    q = [DeviceArray.from_dlpack(q_t[i]) for i in range(L)]
    kn = [DeviceArray.from_dlpack(kn_t[i]) for i in range(L)]
    vn = [DeviceArray.from_dlpack(vn_t[i]) for i in range(L)]
    out = [DeviceArray.empty((B, hq, D), "bfloat16", dev) for _ in range(L)]
    tables_d = DeviceArray.from_numpy(page_tables if pool_pages else tables, device=dev)
    if pool_pages:  # page view of each layer's pool buffers: [num_blocks, BS, kv heads, D] from slot 1
        kview = [a[1:].reshape(num_blocks, BS, hkv, D) for a in kc]
        vview = [a[1:].reshape(num_blocks, BS, hkv, D) for a in vc]
    lens_d = DeviceArray.from_numpy(lens_after.astype(np.int32), device=dev)
    slots_d = DeviceArray.from_numpy(slots, device=dev)
    flush = DeviceArray.empty((L2_FLUSH_BYTES,), "int32", dev) if cfg.get("l2_flush") else None
    scale = 1.0 / math.sqrt(D)

    # decode form.  auto: config 3 runs BASELINE's 512-token split-K; the paged bf16
    # caches otherwise run the planned split-K (work list longest first, one plan per
    # step) with the shim's partition choice; the token pool and FP8 caches, which
    # have no planned entry point, the shim's single-pass / split-K heuristic (the
    # token-pool kernel runs 16-token groups, two CTAs per SM)
    heuristic = mk.choose_decode(B, hkv, max_seq_len, 16 if pool else BS)
    planned_p = mk.choose_planned_partition(B, hkv, max_seq_len, BS, lens_after, head_size=D)
    auto_planned = args.decode == "auto" and not (cfg["partition"] or pool)
    if args.decode == "v1":
        psize = 0
    elif args.decode == "v2":
        psize = args.partition or cfg["partition"] or heuristic or 512
    elif args.decode == "planned" or auto_planned:
        psize = args.partition or planned_p
    else:
        psize = cfg["partition"] or heuristic
    if args.partition and psize and top:
        psize = args.partition
    # config 4 is a radix-cache hit: every table starts with the same prefix, which
    # the serving stack knows, so the default decode is the shared-prefix (cascade) one
    cascade = (args.decode == "cascade" or (args.decode == "auto" and shared)) and not pool and not fp8
    if cascade:
        prefix = cfg["prefix"]
        pp, pt = mk.cascade_partitions(B, hq, hkv, max_seq_len, prefix, BS)
        if top:
            pp, pt = args.partition_prefix or pp, args.partition or pt
        cws = mk.cascade_workspace(B, hq, D, max_seq_len, prefix, pp, pt, dev)
        psize = 0
    split = psize > 0
    planned = split and (args.decode == "planned" or auto_planned) and not pool
    # the step's append folded into the planned decode (one launch per layer) where
    # the step appends one token per sequence to a paged 16-bit cache
    can_fold = planned and not fp8 and not pool and not cascade and T_new == B
    if args.append == "folded" and not can_fold:
        raise SystemExit("--append folded needs the planned paged decode and one new token per sequence")
    folded = can_fold and args.append != "separate"
    ws = mk.splitk_workspace(B, hq, D, max_seq_len, psize, dev) if split else None
    dplan = mk.DecodePlan(B, hkv, max_seq_len, psize, dev) if planned else None
    torch.cuda.synchronize()
    st = Stream()  # all work of the step runs on this stream (graph-capturable)

    def append(i, stream=st):
        if fp8:
            return mk.reshape_and_cache_fp8(kn[i], vn[i], kc[i], vc[i], slots_d, 0.05, 0.05, fmt, stream=stream)
        if pool:
            return mk.reshape_and_cache_flash(kn[i], vn[i], kc[i], vc[i], slots_d, stream=stream)
        return mk.reshape_and_cache(kn[i], vn[i], kc[i], vc[i], slots_d, stream=stream)

    def make_plan(stream=st):
        # one work list per step (every layer has the same lengths)
        if planned:
            mk.make_decode_plan(lens_d, hkv, max_seq_len, psize, plan=dplan, stream=stream)

    def decode(i, stream=st):
        if folded:  # the append and the decode in one launch
            return mk.paged_attention_append(q[i], kn[i], vn[i], kc[i], vc[i], slots_d, tables_d, lens_d, hkv, scale,
                                             BS, max_seq_len, workspace=ws, out=out[i], stream=stream, plan=dplan)
        if fp8:
            return mk.paged_attention_fp8(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len,
                                          k_scale=0.05, v_scale=0.05, fp8_format=fmt, partition_size=psize,
                                          workspace=ws, out=out[i], stream=stream, plan=dplan)
        if cascade:
            return mk.paged_attention_cascade(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len, prefix,
                                              prefix_partition_size=pp, partition_size=pt, workspace=cws, out=out[i],
                                              stream=stream)
        if pool_pages:
            return mk.paged_attention_flash(q[i], kview[i], vview[i], tables_d, lens_d, hkv, scale, BS, max_seq_len,
                                            partition_size=psize, workspace=ws, out=out[i], stream=stream)
        if pool:
            return mk.paged_attention_flash(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, 1, max_seq_len,
                                            partition_size=psize, workspace=ws, out=out[i], stream=stream)
        if split:
            return mk.paged_attention_v2(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len,
                                         partition_size=psize, workspace=ws, out=out[i], stream=stream, plan=dplan)
        return mk.paged_attention_v1(q[i], kc[i], vc[i], tables_d, lens_d, hkv, scale, BS, max_seq_len, out=out[i],
                                     stream=stream)

    def step(ev=None):
        make_plan()
        for i in range(L):
            if not folded:
                append(i)
            if ev is not None:
                ev[i][0].record(st)
            decode(i)
            if ev is not None:
                ev[i][1].record(st)

    def l2_flush():
        if flush is not None:
            flush.fill_zero(stream=st)

    dist = None
    if world > 1 and top:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        l2_flush()
        step()
    st.synchronize()

    # ---- timed region (device-resident inputs); L2 flushed between steps, outside the events ----
    evs = [[[Event(), Event()] for _ in range(L)] for _ in range(args.steps)]
    sev = [[Event(), Event()] for _ in range(args.steps)]

    graph = None
    if args.graph:
        # one step (all layers) as one CUDA graph; replayed between events below
        launches0 = _lib.launch_count()
        graph = Graph.capture(st, step)
        graph_launches = _lib.launch_count() - launches0
        for _ in range(args.warmup):
            l2_flush()
            graph.replay(st)
        st.synchronize()

    def timed_region(with_layer_events):
        for s in range(args.steps):
            l2_flush()
            sev[s][0].record(st)
            if graph is not None and not with_layer_events:
                graph.replay(st)
            else:
                step(evs[s] if with_layer_events else None)
            sev[s][1].record(st)

    sampler = ClockSampler(dev)
    barrier()
    _lib.synchronize()
    sampler.start()
    launches0 = _lib.launch_count()
    timed_region(with_layer_events=graph is None)
    st.synchronize()
    launches = (_lib.launch_count() - launches0) if graph is None else graph_launches * args.steps
    clocks = sampler.stop()
    total_ms = sum(a.elapsed_ms(b) for a, b in sev)
    if graph is not None:
        # per-launch decode times come from an eager pass of the same launches
        timed_region(with_layer_events=True)
        st.synchronize()
    dec_ms = [evs[s][i][0].elapsed_ms(evs[s][i][1]) for s in range(args.steps) for i in range(L)]
    barrier()

    # ---- e2e through the public API with pinned host buffers ----
    # Every step copies its inputs (q, the new K/V rows, lengths, slots) from pinned
    # host memory and its outputs back.  Copies run on two side streams (host ->
    # device, device -> host), ordered with events, so layer i + 1's inputs land
    # while layer i computes and layer i's output leaves while layer i + 1 does.
    e2e_ms = float("nan")
    h2d = d2h = 0
    if not args.no_e2e and top:
        h_q = [HostBuffer((B, hq, D), "bfloat16") for _ in range(L)]
        h_k = [HostBuffer((T_new, hkv, D), "bfloat16") for _ in range(L)]
        h_v = [HostBuffer((T_new, hkv, D), "bfloat16") for _ in range(L)]
        h_o = [HostBuffer((B, hq, D), "bfloat16") for _ in range(L)]
        rng = np.random.default_rng(5 + rank)
        for i in range(L):
            for hb in (h_q[i], h_k[i], h_v[i]):
                hb.array[...] = random_bf16_bits(rng, hb.shape)
        h_lens = HostBuffer((B,), "int32")
        h_lens.array[...] = lens_after
        h_slots = HostBuffer((T_new,), "int32")
        h_slots.array[...] = slots
        up, down = Stream(), Stream()
        ev_in = [Event() for _ in range(L)]    # layer i's inputs are on the device
        ev_dec = [Event() for _ in range(L)]   # layer i's decode is done (inputs free, output ready)
        ev_out = [Event() for _ in range(L)]   # layer i's output is on the host (output buffer free)
        ev_meta = Event()

        def e2e_step(first):
            if not first:
                up.wait(ev_dec[L - 1])  # the previous step's last decode has read lengths and slots
            lens_d.copy_from_host(h_lens, stream=up)
            slots_d.copy_from_host(h_slots, stream=up)
            ev_meta.record(up)
            for i in range(L):
                if not first:
                    up.wait(ev_dec[i])
                q[i].copy_from_host(h_q[i], stream=up)
                kn[i].copy_from_host(h_k[i], stream=up)
                vn[i].copy_from_host(h_v[i], stream=up)
                ev_in[i].record(up)
            st.wait(ev_meta)
            make_plan()
            for i in range(L):
                st.wait(ev_in[i])
                if not first:
                    st.wait(ev_out[i])
                if not folded:
                    append(i)
                decode(i)
                ev_dec[i].record(st)
                down.wait(ev_dec[i])
                out[i].copy_to_host(h_o[i], stream=down)
                ev_out[i].record(down)

        for s in range(max(2, args.warmup)):
            l2_flush()
            e2e_step(first=(s == 0))
        st.synchronize()
        down.synchronize()
        barrier()
        t0, t1 = Event(), Event()
        t0.record(st)
        up.wait(t0)
        for s in range(args.steps):
            e2e_step(first=False)
        st.wait(ev_out[L - 1])
        t1.record(st)
        st.synchronize()
        e2e_ms = t0.elapsed_ms(t1)
        h2d = B * 4 + T_new * 4 + L * (B * hq * D * 2 + 2 * T_new * hkv * D * 2)
        d2h = L * B * hq * D * 2

    # ---- every rank checks a sample of its outputs (the last layer) against the oracle ----
    mode = "fp8" if fp8 else ("pool" if pool else "paged")
    ok, err, nrows = check_outputs(torch, q_t[L - 1], kc_t[L - 1], vc_t[L - 1], out[L - 1], tables, lens_after, hkv,
                                   D, tab_bs, mode, fmt)
    status = _lib.get_status(dev, clear=True)
    ok = ok and status == 0

    # ---- reduce over ranks (max time; bytes summed; worst check) ----
    step_ms = total_ms / args.steps
    e2e_step_ms = e2e_ms / args.steps
    mean_dec_ms = float(np.mean(dec_ms))
    alg, logical = decode_bytes(page_tables if pool_pages else tables, lens_after, hq, hkv, D,
                                BS if pool_pages else tab_bs, shared, s_kv=1 if fp8 else 2)
    if folded:  # the launch also reads the new K/V rows and writes them into the cache
        alg += 2 * 2 * T_new * hkv * D * 2
        logical += 2 * 2 * T_new * hkv * D * 2
    sums = np.array([float(alg), float(logical), float(h2d), float(d2h)])
    if dist is not None:
        t = torch.tensor([step_ms, e2e_step_ms, mean_dec_ms, 0.0 if ok else 1.0, err], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_step_ms, _, bad, err = [float(x) for x in t]
        ok = bad == 0.0
        tt = torch.tensor(np.concatenate([sums, [float(nrows)]]), dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        sums, nrows = tt.numpy()[:4], int(tt.numpy()[4])
    del kc_t, vc_t, kc, vc, q_t, kn_t, vn_t
    if rank != 0:
        if not ok:
            raise SystemExit(f"rank {rank}: outputs differ from the CPU oracle or kernel status flags are set")
        return None
    alg_all, logical_all, h2d_all, d2h_all = sums
    peak, peak_kind = load_peaks()
    kernel_key = ("cascade" if cascade else "pool-pages" if pool_pages else "pool" if pool else f"fp8-{fmt}" if fp8 else
                  f"planned{psize}" if planned else f"splitk{psize}" if split else "v1")
    traffic = (load_traffic(config, kernel_key)
               if (world == 1 and not (args.layers or args.batch or args.kv_heads)) else None)
    achieved = alg / (mean_dec_ms * 1e-3) / 1e9
    toks = B_all / (step_ms * 1e-3)
    kernel = f"split-K v2, {psize}-token partitions" if split else "paged_attention_v1"
    if planned:
        kernel = f"planned split-K, {psize}-token partitions longest first, merge fused"
        if folded:
            kernel += ", the step's append folded in"
    if pool:
        kernel = "token-pool decode (paged_attention_flash, " + (
            f"{BS}-token page tables, tensor copies" if pool_pages else "slot lists") + (
            f", {psize}-token partitions)" if split else ", single pass)")
    if fp8:
        kernel = f"FP8 ({fmt}) cache decode, " + (
            f"planned split-K, {psize}-token partitions longest first" if planned else
            f"{psize}-token partitions" if split else "single pass")
    if cascade:
        kernel = f"shared-prefix cascade ({prefix}-token prefix in {pp}-token chunks, tail partitions of {pt})"
    extra = {"kernel": kernel, "launch": "one CUDA graph per step (decode timing from an eager pass)" if graph is not None else "eager",
             "l2": ("flushed between steps (unique KV fits in L2)" if flush is not None else
                    f"inputs larger than L2 (KV per layer {logical_all / 1e9:.2f} GB); no flush")}
    if pool:
        extra["layout"] = ("MHATokenPool buffers [slots, kv_heads, head_dim], " +
                           (f"page tables ({BS}-slot pages)" if pool_pages else "slot-list tables"))
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
        "dtype": f"{args.kv_dtype} cache, f16 products" if fp8 else "bf16",
        "data": "synthetic",
        "config": config_json(cfg, config, world, extra),
        "kv_gbs": L * alg_all / (step_ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic[0] if traffic else None,
                     "traffic_source": traffic[1] if traffic else None,
                     "peak_kind": peak_kind, "kernel": f"paged decode ({kernel}), per layer launch",
                     "algorithmic_bytes_per_launch": alg, "mean_launch_ms": mean_dec_ms},
        "e2e": None if (args.no_e2e or not top) else {
            "value": B_all / (e2e_step_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d_all),
            "d2h_bytes_per_step": int(d2h_all),
            "how": "public API per layer (append + decode) with pinned host inputs/outputs copied every step on "
                   "two side streams overlapping the compute"},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "output_check": {"ok": bool(ok), "ranks": world, "rows_checked": int(nrows), "max_abs_err": err,
                         "against": "CPU oracle (float64 gather + SDPA) on each rank's own caches, last layer; "
                                    "kernel status word clear",
                         "tolerance": f"{ATOL:g} abs + {RTOL:g} rel"},
    }
    if shared:
        line["effective_kv_gbs"] = L * logical_all / (step_ms * 1e-3) / 1e9
        line["roofline"]["note"] = "achieved counts each shared prefix block once (unique bytes)"
    if len(w["prefill_slots"]):
        line["prefill_tokens_per_s"] = len(w["prefill_slots"]) / (step_ms * 1e-3)
    if not ok:
        print(json.dumps(line), flush=True)
        raise SystemExit("outputs differ from the CPU oracle or kernel status flags are set (output_check)")
    return line


def add_cpu_baseline(line, args, config):
    """The host legs (cpu_baseline_entry) over one full layer of the workload, twice."""
    w, cfg = workload(args, config)
    line["cpu_baseline"] = cpu_baseline_entry(cfg, w, host_threads(), 2)


OTHER_KEYS = ("value", "unit", "ms_per_step", "kv_gbs", "effective_kv_gbs", "prefill_tokens_per_s", "roofline",
              "gpu_launches", "clocks", "output_check")


def run_ours(args, rank, world, local_rank):
    import torch

    from sglang_mlx_b200 import _lib

    _lib.set_device(local_rank)
    torch.cuda.set_device(local_rank)
    line = measure_decode(args, args.config, rank, world, local_rank, top=True)
    plain = (world == 1 and args.config == 2 and args.layout == "paged" and args.kv_dtype == "bf16"
             and args.decode == "auto" and not (args.layers or args.batch or args.kv_heads or args.partition))
    if rank != 0:
        return
    if plain and not args.no_other_configs:
        torch.cuda.empty_cache()
        others = {}
        for c in (3, 4, 5):
            sub = argparse.Namespace(**vars(args))
            sub.config, sub.steps, sub.warmup = c, max(args.steps, 20), max(args.warmup, 3)
            lc = measure_decode(sub, c, 0, 1, local_rank, top=False)
            entry = {k: lc[k] for k in OTHER_KEYS if k in lc}
            entry["config"] = lc["config"]
            entry["steps"] = sub.steps
            others[str(c)] = entry
            torch.cuda.empty_cache()
        line["other_configs"] = others
    if not args.no_cpu_baseline and world == 1 and args.layout == "paged" and args.kv_dtype == "bf16":
        add_cpu_baseline(line, args, args.config)
    print(json.dumps(line), flush=True)


PREFILL_METRIC = "paged prefill/extend attention TFLOP/s (visible keys only) and prefill tokens/s"


def prefill_flops(prefixes, qlens, hq, d):
    """4 * d FLOPs (Q.K^T and P.V multiply-adds) per (query row, visible key):
    new token t of a sequence with prefix p sees p + t + 1 keys."""
    vis = sum(int(n) * int(p) + int(n) * (int(n) + 1) // 2 for p, n in zip(prefixes, qlens))
    return 4.0 * d * hq * vis


def run_prefill(args, rank, world, local_rank):
    """--mode prefill: the chunked prefill of BASELINE config 5 (16 chunks of 512
    new tokens, each on a prefix drawn from config 5's seeded lognormal context
    lengths; 28 q / 4 kv heads, head_dim 128, block 32, bf16) through
    paged_prefill_attention, per layer.  Tensor-bound: the roofline is TFLOP/s
    of visible-key FLOPs against the measured bf16 GEMM peak."""
    import torch

    from sglang_mlx_b200 import _lib, sharding
    from sglang_mlx_b200 import metal_kernels as mk
    from sglang_mlx_b200.device_array import DeviceArray, Event, HostBuffer, Stream

    dev = local_rank
    _lib.set_device(dev)
    torch.cuda.set_device(dev)
    tdev = torch.device("cuda", dev)
    w = cases.baseline_workload(5)
    cfg = dict(w["cfg"])
    L = args.layers or cfg["layers"]
    HQ, HKV, D, BS = cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"]
    n_chunks, chunk = cfg["prefill_chunks"], cfg["chunk"]
    prefixes_all = np.asarray(w["lens"][:n_chunks], np.int64)
    qlens_all = np.full(n_chunks, chunk, np.int64)
    plan = sharding.plan(HQ, HKV, world, rank, prefixes_all + qlens_all)
    hkv, hq = plan.num_kv_heads, plan.num_q_heads
    prefixes, qlens = prefixes_all[plan.seqs], qlens_all[plan.seqs]
    B = len(prefixes)
    kvl = prefixes + qlens
    pool = args.layout == "pool"
    rng = np.random.default_rng(77 + rank)
    nbs = [-(-int(n) // BS) for n in kvl]
    num_blocks = sum(nbs) + 8
    perm = rng.permutation(num_blocks)
    tables = np.zeros((B, max(nbs)), np.int64)
    o = 0
    for b, nb in enumerate(nbs):
        tables[b, :nb] = perm[o:o + nb]
        o += nb
    if pool:  # token-pool slot lists (slot 0 is the pool's padding slot)
        t = np.arange(tables.shape[1] * BS)
        tables = tables[:, t // BS] * BS + t % BS + 1
    tables = np.ascontiguousarray(tables.astype(np.int32))
    indptr = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    T = int(indptr[-1])
    max_q = int(qlens.max())

    g = torch.Generator(device=tdev)
    g.manual_seed(4321 + rank)
    tdt = torch.bfloat16
    kc, vc, q, out, keep = [], [], [], [], []
    for _ in range(L):
        if pool:
            k = torch.randn((num_blocks * BS + 1, hkv, D), generator=g, device=tdev, dtype=tdt)
            v = torch.randn((num_blocks * BS + 1, hkv, D), generator=g, device=tdev, dtype=tdt)
        else:
            k = torch.randn((num_blocks, hkv, D // 8, BS, 8), generator=g, device=tdev, dtype=tdt)
            v = torch.randn((num_blocks, hkv, D, BS), generator=g, device=tdev, dtype=tdt)
        qq = torch.randn((T, hq, D), generator=g, device=tdev, dtype=tdt)
        keep += [k, v, qq]
        kc.append(DeviceArray.from_dlpack(k))
        vc.append(DeviceArray.from_dlpack(v))
        q.append(DeviceArray.from_dlpack(qq))
        out.append(DeviceArray.empty((T, hq, D), "bfloat16", dev))
    tables_d = DeviceArray.from_numpy(tables, device=dev)
    indptr_d = DeviceArray.from_numpy(indptr, device=dev)
    kvl_d = DeviceArray.from_numpy(kvl.astype(np.int32), device=dev)
    flush = DeviceArray.empty((L2_FLUSH_BYTES,), "int32", dev)
    scale = 1.0 / math.sqrt(D)
    torch.cuda.synchronize()
    st = Stream()
    tab_bs = 1 if pool else BS

    def layer(i):
        mk.paged_prefill_attention(q[i], kc[i], vc[i], tables_d, indptr_d, kvl_d, hkv, scale, tab_bs, max_q_len=max_q,
                                   out=out[i], stream=st)

    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        flush.fill_zero(stream=st)
        for i in range(L):
            layer(i)
    st.synchronize()
    if _lib.get_status(clear=True):
        raise SystemExit("prefill kernel status flags set in warm-up")
    evs = [[[Event(), Event()] for _ in range(L)] for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    barrier()
    _lib.synchronize()
    sampler.start()
    launches0 = _lib.launch_count()
    for s in range(args.steps):
        flush.fill_zero(stream=st)  # between steps, outside the events
        for i in range(L):
            evs[s][i][0].record(st)
            layer(i)
            evs[s][i][1].record(st)
    st.synchronize()
    launches = _lib.launch_count() - launches0  # prefill kernels (the L2 flush memsets are not counted)
    clocks = sampler.stop()
    # the timed launches' results: status word, and the last layer against the oracle
    status = _lib.get_status(clear=True)
    ok, err, nrows = check_prefill(torch, keep[3 * (L - 1) + 2], keep[3 * (L - 1)], keep[3 * (L - 1) + 1],
                                   out[L - 1], tables, indptr, kvl, hkv, D, BS, pool)
    ok = ok and status == 0
    lay_ms = [evs[s][i][0].elapsed_ms(evs[s][i][1]) for s in range(args.steps) for i in range(L)]
    step_ms = float(np.sum(lay_ms)) / args.steps
    mean_ms = float(np.mean(lay_ms))

    # e2e through the public API: queries from pinned host memory, outputs back
    e2e_ms = float("nan")
    h2d = d2h = 0
    if not args.no_e2e:
        hq_buf = [HostBuffer((T, hq, D), "bfloat16") for _ in range(L)]
        ho_buf = [HostBuffer((T, hq, D), "bfloat16") for _ in range(L)]
        for hb in hq_buf:
            hb.array[...] = rng.integers(0x3c00, 0x4000, size=hb.shape, dtype=np.uint16)

        def e2e_step():
            for i in range(L):
                q[i].copy_from_host(hq_buf[i], stream=st)
                layer(i)
                out[i].copy_to_host(ho_buf[i], stream=st)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        st.synchronize()
        eev = [[Event(), Event()] for _ in range(args.steps)]
        for s in range(args.steps):
            flush.fill_zero(stream=st)
            eev[s][0].record(st)
            e2e_step()
            eev[s][1].record(st)
        st.synchronize()
        e2e_ms = sum(a.elapsed_ms(b) for a, b in eev) / args.steps
        h2d = d2h = L * T * hq * D * 2

    flops = prefill_flops(prefixes, qlens, hq, D)
    sums = np.array([flops, float(T), float(h2d), float(d2h)])
    if dist is not None:
        t = torch.tensor([step_ms, e2e_ms, mean_ms, 0.0 if ok else 1.0, err], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms, mean_ms = [float(x) for x in t[:3]]
        ok, err = bool(t[3] == 0.0), float(t[4])  # every rank's sample passed; the largest error
        tt = torch.tensor(sums, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        sums = tt.numpy()
    if rank != 0:
        return
    flops_all, _, h2d_all, d2h_all = sums
    peak, peak_kind = load_tensor_peak()
    achieved = flops / (mean_ms * 1e-3) / 1e12
    tokens = n_chunks * chunk  # new tokens of the whole job per layer pass
    line = {
        "metric": PREFILL_METRIC,
        "value": L * flops_all / (step_ms * 1e-3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "config5-chunked-prefill", "chunks": f"{n_chunks} x {chunk} new tokens",
                   "prefixes": "config 5 lognormal lengths of sequences 0..15 (seeded)", "layers": L,
                   "heads": f"{HQ}q/{HKV}kv", "head_dim": D, "block_size": BS,
                   "layout": "MHATokenPool slot lists" if pool else "paged (vLLM layout)",
                   "parallelism": f"kv-head-shard{world}", "kernel": "paged_prefill_attention",
                   "l2": "flushed between steps (512 MB write, outside the events)"},
        "prefill_tokens_per_s": tokens * 1.0 / (step_ms * 1e-3 / L) if L else None,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": peak_kind, "kernel": "prefill_kernel, per layer launch",
                     "algorithmic_flops_per_launch": flops, "mean_launch_ms": mean_ms},
        "e2e": None if args.no_e2e else {"value": L * flops_all / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                                         "h2d_bytes_per_step": int(h2d_all), "d2h_bytes_per_step": int(d2h_all)},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "output_check": {"ok": bool(ok), "ranks": world, "rows_checked": int(nrows), "max_abs_err": err,
                         "against": "CPU oracle (float64 gather + masked SDPA) on the last 8 new tokens of 3 "
                                    "sequences of the last layer; kernel status word clear",
                         "tolerance": f"{ATOL:g} abs + {RTOL:g} rel"},
    }
    if not ok:
        print(json.dumps(line), flush=True)
        raise SystemExit("prefill outputs differ from the CPU oracle or kernel status flags are set (output_check)")
    if not args.no_cpu_baseline and world == 1:
        from oracle import kv_oracle
        from threadpoolctl import threadpool_limits

        n_s = min(8, B)
        kb = keep[0].float().cpu().numpy()
        vb = keep[1].float().cpu().numpy()
        qb = keep[2][: int(indptr[n_s])].float().cpu().numpy()
        with threadpool_limits(1):
            t0 = time.perf_counter()
            kv_oracle.paged_prefill(qb, kb, vb, tables[:n_s], indptr[: n_s + 1], kvl[:n_s], hkv, scale)
            dt = time.perf_counter() - t0
        sample_flops = prefill_flops(prefixes[:n_s], qlens[:n_s], hq, D)
        line["cpu_baseline"] = {"value": sample_flops / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                                "sample": f"{n_s} of {B} sequences x 1 of {L} layers (float64 gather + masked SDPA, "
                                          f"NumPy, 1 thread), {lscpu_model()}"}
    print(json.dumps(line), flush=True)


def check_prefill(torch, q_t, kc_t, vc_t, out, tables, indptr, kvl, hkv, D, bs, pool, n_last=8):
    """The last n_last new tokens of a sample of this rank's sequences (first,
    middle, last) of one layer against the CPU oracle (float64 gather + masked
    SDPA over the rank's own caches).  Returns (ok, max |err|, rows checked)."""
    from oracle import kv_oracle

    B = len(kvl)
    seqs = sorted({0, B // 2, B - 1})
    dev = kc_t.device
    got, qs, ind, ids, t2, lens = [], [], [0], [], [], []
    o = 0
    for b in seqs:
        q1 = int(indptr[b + 1])
        q0 = max(int(indptr[b]), q1 - n_last)
        got.append(out.to_numpy()[q0:q1])
        qs.append(q_t[q0:q1].float().cpu().numpy())
        ind.append(ind[-1] + q1 - q0)
        n = int(kvl[b]) if pool else -(-int(kvl[b]) // bs)  # slots, or pages
        ids.append(tables[b, :n].astype(np.int64))
        t2.append(np.arange(o, o + n))
        lens.append(int(kvl[b]))
        o += n
    width = max(len(t) for t in t2)
    tab = np.zeros((len(seqs), width), np.int64)
    for i, t in enumerate(t2):
        tab[i, :len(t)] = t
    idx = torch.from_numpy(np.concatenate(ids)).to(dev)
    kg = kc_t.index_select(0, idx).float().cpu().numpy()
    vg = vc_t.index_select(0, idx).float().cpu().numpy()
    ref = kv_oracle.paged_prefill(np.concatenate(qs), kg, vg, tab, np.asarray(ind), np.asarray(lens), hkv,
                                  1.0 / math.sqrt(D))
    got = np.concatenate(got)
    ok, err, _ = kv_oracle.allclose_report(got, ref, ATOL, RTOL)
    return bool(ok and np.isfinite(got).all()), float(err), int(got.shape[0])


def load_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=sorted(cases.BASELINE))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="one-GPU default run: skip the nested measurements of configs 3, 4 and 5")
    ap.add_argument("--kv-dtype", default="bf16", choices=["bf16", "fp8-e4m3", "fp8-e5m2"],
                    help="cache element type: bf16 (default) or one-byte FP8 codes (half the KV bytes)")
    ap.add_argument("--layout", default="paged", choices=["paged", "pool", "pool-pages"],
                    help="cache layout: the vLLM paged layout (default), the MHATokenPool token pool read through "
                         "slot lists, or the same pool read through page tables (a page-granular allocator)")
    ap.add_argument("--decode", default="auto", choices=["auto", "v1", "v2", "planned", "cascade"],
                    help="decode form: the shim's choice (default; shared-prefix cascade for config 4), single pass, "
                         "split-K, planned split-K (work list longest first, merge fused), or cascade")
    ap.add_argument("--partition", type=int, default=0, help="split-K partition size (tokens) when split")
    ap.add_argument("--append", default="auto", choices=["auto", "separate", "folded"],
                    help="the step's append: folded into the planned decode where it applies (default), or its own "
                         "launch before each decode")
    ap.add_argument("--partition-prefix", type=int, default=0,
                    help="cascade: shared-prefix chunk size (tokens); default from cascade_partitions")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling cases only)")
    ap.add_argument("--batch", type=int, default=0, help="override the batch (profiling cases only)")
    ap.add_argument("--kv-heads", type=int, default=0,
                    help="override the KV head count, keeping the group size (profiling cases only)")
    ap.add_argument("--mode", default="decode", choices=["decode", "prefill"],
                    help="decode (the BASELINE metric) or the config-5 chunked prefill through paged_prefill_attention")
    ap.add_argument("--graph", action=argparse.BooleanOptionalAction, default=True,
                    help="replay each timed step as one CUDA graph (removes host launch overhead)")
    args = ap.parse_args()
    if args.impl == "ours":
        args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference" and args.mode == "prefill":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "prefill mode: the reference runs prefill as mlx "
                                  "SDPA (not installed); the --impl ours line carries the CPU oracle as cpu_baseline"}))
        elif args.impl == "reference":
            run_reference(args, rank, world)
        elif args.mode == "prefill":
            run_prefill(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
