"""Host-side multi-GPU logic on CPU: KV-head (and head x sequence) sharding with
2 and 4 gloo ranks.  Each rank computes its shard with the CPU oracle; the
all-gathered shards must equal the unsharded result.  No GPU."""

import os
import socket

import numpy as np
import pytest

import cases
from oracle import kv_oracle
from sglang_mlx_b200 import sharding


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(Hq, Hkv, lens):
    c = cases.paged_batch(77, "bfloat16", len(lens), Hq, Hkv, 64, 16, lens)
    kc = np.zeros(c["k_cache"].shape, np.float32)
    vc = np.zeros(c["v_cache"].shape, np.float32)
    kv_oracle.reshape_and_cache(c["k"], c["v"], kc, vc, c["slot_mapping"])
    return c, kc, vc


def _rank_main(rank, world, port, Hq, Hkv, lens, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c, kc, vc = _case(Hq, Hkv, lens)
        p = sharding.plan(Hq, Hkv, world, rank, c["context_lens"])
        # this rank's slice of the pool (its kv heads), tables/lengths of its sequences
        k0, k1 = p.kv_heads
        out = kv_oracle.paged_attention_v1(c["q"][p.seqs][:, p.q_heads[0]:p.q_heads[1]], kc[:, k0:k1], vc[:, k0:k1],
                                           c["block_tables"][p.seqs], c["context_lens"][p.seqs], p.num_kv_heads,
                                           c["scale"], 16, c["max_seq_len"])
        # pad to a fixed shape for the gather
        buf = np.zeros((len(lens), Hq, 64))
        buf[p.seqs, p.q_heads[0]:p.q_heads[1]] = out
        t = torch.from_numpy(buf)
        dist.all_reduce(t)  # disjoint slices: the sum is the concatenation
        if rank == 0:
            full = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], Hkv,
                                                c["scale"], 16, c["max_seq_len"])
            q.put(float(np.abs(t.numpy() - full).max()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,Hq,Hkv", [(2, 16, 8), (2, 8, 1), (4, 28, 2)])
def test_sharded_decode_equals_unsharded(world, Hq, Hkv):
    import torch.multiprocessing as mp

    lens = [100, 900, 37, 512, 1, 260]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, Hq, Hkv, lens, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) < 1e-12


def test_plans_cover_every_head_and_sequence_once():
    lens = np.array([5, 100, 2000, 30, 30, 900, 7, 64])
    for Hq, Hkv, world in ((32, 8, 8), (32, 8, 2), (28, 4, 8), (28, 4, 4), (64, 8, 1)):
        seen = np.zeros((len(lens), Hq), int)
        for r in range(world):
            p = sharding.plan(Hq, Hkv, world, r, lens)
            seen[np.ix_(p.seqs, np.arange(*p.q_heads))] += 1
        assert (seen == 1).all(), (Hq, Hkv, world)


def test_sequence_split_balances_tokens():
    lens = np.random.default_rng(0).lognormal(np.log(1500), 1.0, 512).clip(16, 32768).astype(int)
    parts = sharding.split_by_tokens(lens, 2)
    a, b = lens[parts[0]].sum(), lens[parts[1]].sum()
    assert abs(a - b) <= lens.max()


def test_bad_shapes_rejected():
    with pytest.raises(ValueError):
        sharding.plan(32, 8, 3, 0, [1])
    with pytest.raises(ValueError):
        sharding.plan(30, 8, 2, 0, [1])
