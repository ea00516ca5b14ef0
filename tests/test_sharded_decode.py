"""The multi-GPU decode layout checked through the real kernels.

Every rank's share of BASELINE configs 2 and 5 at full size (one layer) is
cut out exactly as a rank of `bench.py --gpus N` holds it: its KV heads of the
pool (a dense copy), its query heads, and for config 5 at N = 8 (4 KV heads on
8 ranks) its token-balanced half of the sequences (sharding.plan).  Each share
is decoded on one GPU, one rank after another, with the form the shim's
default decode runs for that share (metal_kernels.paged_attention: the planned
split-K, partition size from choose_planned_partition on the share's lengths).
The shares assembled by sharding.assemble must equal the unsharded decode
within the north-star tolerance, and a sample of sequences of every rank is
checked against the CPU oracle (float64 gather + SDPA)."""

import math

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close
from oracle import c_oracle
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200 import sharding

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _oracle_rows(q, kc, vc, tables, lens, rows, hkv, scale, bs):
    """c_oracle decode of sequences `rows` of one share (blocks renumbered densely)."""
    dev = kc.device
    nb = [(-(-int(lens[b]) // bs)) for b in rows]
    blocks = np.concatenate([tables[b, :n] for b, n in zip(rows, nb)]).astype(np.int64)
    t2 = np.zeros((len(rows), max(nb)), np.uint32)
    o = 0
    for i, n in enumerate(nb):
        t2[i, :n] = np.arange(o, o + n)
        o += n
    idx = torch.from_numpy(blocks).to(dev)
    return c_oracle.paged_attention(_bits(q[torch.from_numpy(np.asarray(rows)).to(dev)]), "bfloat16",
                                    _bits(kc.index_select(0, idx)), _bits(vc.index_select(0, idx)), "bfloat16", t2,
                                    lens[rows].astype(np.uint32), hkv, scale, int(t2.shape[1] * bs))


@pytest.fixture(scope="module", params=[2, 5])
def full_config(request):
    config = request.param
    w = cases.baseline_workload(config)
    cfg = w["cfg"]
    B, HQ, HKV, D, BS = cfg["batch"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(300 + config)
    kc = torch.randn((w["num_blocks"], HKV, D // 8, BS, 8), generator=g, device=dev, dtype=torch.bfloat16)
    vc = torch.randn((w["num_blocks"], HKV, D, BS), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((B, HQ, D), generator=g, device=dev, dtype=torch.bfloat16)
    lens = (w["lens"] + 1).astype(np.int32)
    scale = 1.0 / math.sqrt(D)
    full = mk.paged_attention_v1(q, kc, vc, w["tables"], lens, HKV, scale, BS, w["max_seq_len"]).to_numpy()
    yield dict(config=config, w=w, cfg=cfg, kc=kc, vc=vc, q=q, lens=lens, scale=scale, full=full)
    del kc, vc, q
    torch.cuda.empty_cache()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_matches_unsharded(gpu, full_config, world):
    fc = full_config
    w, cfg = fc["w"], fc["cfg"]
    B, HQ, HKV, BS = cfg["batch"], cfg["hq"], cfg["hkv"], cfg["bs"]
    outs, plans = [], []
    for rank in range(world):
        p = sharding.plan(HQ, HKV, world, rank, fc["lens"])
        k0, k1 = p.kv_heads
        q0, q1 = p.q_heads
        seqs = torch.from_numpy(p.seqs).to(fc["q"].device)
        kc = fc["kc"][:, k0:k1].contiguous()  # the rank's own pool: its KV heads only
        vc = fc["vc"][:, k0:k1].contiguous()
        q = fc["q"].index_select(0, seqs)[:, q0:q1].contiguous()
        tables = np.ascontiguousarray(w["tables"][p.seqs])
        lens = fc["lens"][p.seqs]
        psize = mk.choose_planned_partition(len(lens), p.num_kv_heads, w["max_seq_len"], BS, lens,
                                           head_size=fc["q"].shape[-1])
        out = mk.paged_attention(q, kc, vc, tables, lens, p.num_kv_heads, fc["scale"], BS,
                                 w["max_seq_len"]).to_numpy()
        assert np.isfinite(out).all()
        # a sample of this rank's sequences (first, middle, last) against the CPU oracle
        rows = sorted({0, len(lens) // 2, len(lens) - 1})
        ref = _oracle_rows(q, kc, vc, tables, lens, rows, p.num_kv_heads, fc["scale"], BS)
        assert_close(out[rows], ref, ATOL_NS, RTOL_NS,
                     f"config {fc['config']} N={world} rank {rank} (partitions {psize}) vs oracle")
        outs.append(out)
        plans.append(p)
        del kc, vc
    assembled = sharding.assemble(outs, plans, B, HQ)
    assert_close(assembled, fc["full"], ATOL_NS, RTOL_NS, f"config {fc['config']} N={world}: assembled vs unsharded")
    assert gpu.get_status(clear=True) == 0
