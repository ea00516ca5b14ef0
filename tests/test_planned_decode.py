"""GPU tests of the planned split-K decode (kvc_decode_plan +
kvc_paged_attention_planned): the work list the plan kernel writes (every
(sequence, partition) item exactly once, sizes non-increasing, counters zero),
and the decode against the float64 oracle and the plain split-K decode, over
dtypes, head and block sizes, group sizes, ALiBi, the zero-output edge rules,
many partitions (the separate-reduce form), a plan reused by many layers,
CUDA-graph capture and a mismatched plan."""

import math

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close, fill_cache, oracle_fill, upload_case
from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray, Graph, Stream

pytestmark = pytest.mark.gpu


def expected_items(lens, max_seq_len, P):
    """(sequence, partition, size) of every item the plan must hold."""
    items = []
    for b, C in enumerate(int(x) for x in lens):
        if C == 0 or C > max_seq_len:
            items.append((b, 0, 0))
            continue
        n = -(-C // P)
        items += [(b, k, P) for k in range(n - 1)]
        items.append((b, n - 1, C - (n - 1) * P))
    return items


@pytest.mark.parametrize("P,lens", [
    (512, [1, 512, 513, 4097, 0, 9000, 1500, 2048]),
    (2048, list(np.random.default_rng(3).integers(0, 6000, size=300))),
    (32, [31, 32, 33, 64, 1000]),
])
def test_plan_holds_every_item_longest_first(gpu, P, lens):
    lens = np.asarray(lens, np.int32)
    max_seq_len = 8192
    hkv = 3
    plan = mk.make_decode_plan(DeviceArray.from_numpy(lens), hkv, max_seq_len, P)
    raw = plan.array.to_numpy().view(np.uint32)
    want = expected_items(lens, max_seq_len, P)
    assert raw[0] == 0x4E4C5044 and list(raw[1:5]) == [len(lens), hkv, max_seq_len, P]
    n = int(raw[5])
    assert n == len(want)
    items = raw[8:8 + n]
    got = [(int(i & 0xFFFF), int(i >> 16)) for i in items]
    assert sorted(got) == sorted((b, k) for b, k, _ in want)
    size = {(b, k): s for b, k, s in want}
    sizes = [size[x] for x in got]
    assert all(a >= b for a, b in zip(sizes, sizes[1:])), "items must be ordered longest first"
    max_items = mk.decode_plan_size(len(lens), hkv, max_seq_len, P) - 8 - len(lens) * hkv
    counters = raw[8 + max_items:8 + max_items + len(lens) * hkv]
    assert not counters.any()


def _run(c, d, P, alibi=None, plan=None, max_seq_len=None):
    msl = max_seq_len or c["max_seq_len"]
    if plan is None:
        plan = mk.make_decode_plan(d["context_lens"], c["num_kv_heads"], msl, P)
    return mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                 c["num_kv_heads"], c["scale"], c["block_size"], msl, alibi, partition_size=P,
                                 plan=plan).to_numpy()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_planned_matches_oracle(gpu, dtype, D, bs):
    lens = [1, 37, 300, 1025, 2048, 2049, 5000, 640]
    c = cases.paged_batch(7000 + D + bs, dtype, len(lens), 8, 2, D, bs, lens)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], bs,
                                       c["max_seq_len"])
    for P in (256, 1024):
        out = _run(c, d, P)
        assert_close(out, ref, ATOL_NS, RTOL_NS, f"planned P={P}")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("Hq,Hkv", [(4, 1), (16, 2), (28, 4), (64, 8), (32, 2)])
def test_planned_group_sizes_and_v2_agreement(gpu, Hq, Hkv):
    rng = np.random.default_rng(Hq)
    lens = rng.integers(1, 3000, size=40)
    c = cases.paged_batch(7100 + Hq, "bfloat16", len(lens), Hq, Hkv, 128, 16, lens)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    out = _run(c, d, 512)
    v2 = mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], Hkv,
                               c["scale"], 16, c["max_seq_len"], partition_size=512).to_numpy()
    assert_close(out, v2, ATOL_NS, RTOL_NS, "planned vs v2")
    pick = [0, len(lens) // 2, len(lens) - 1]
    ref = kv_oracle.paged_attention_v1(c["q"][pick], kc, vc, c["block_tables"][pick], c["context_lens"][pick], Hkv,
                                       c["scale"], 16, c["max_seq_len"])
    assert_close(out[pick], ref, ATOL_NS, RTOL_NS, "planned vs oracle")
    assert gpu.get_status(clear=True) == 0


def test_planned_alibi_and_zero_rules(gpu):
    lens = [0, 100, 700, 2000, 1500]
    c = cases.paged_batch(7200, "float16", len(lens), 8, 2, 128, 16, lens)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "float16")
    slopes = np.linspace(-0.5, 0.25, 8).astype(np.float32)
    out = _run(c, d, 512, alibi=DeviceArray.from_numpy(slopes))
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16,
                                       c["max_seq_len"], slopes)
    assert_close(out, ref, ATOL_NS, RTOL_NS, "alibi")
    assert not out[0].any()
    # lengths past max_seq_len give zeros (paged_attention_kernels.metal:45-50)
    out = _run(c, d, 512, max_seq_len=1024)
    assert not out[0].any() and not out[3].any() and not out[4].any()
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16, 1024)
    assert_close(out, ref, ATOL_NS, RTOL_NS, "max_seq_len")
    assert gpu.get_status(clear=True) == 0


def test_many_partitions_use_the_reduce_kernel(gpu):
    """Over 32 partitions per sequence the partials go through the reduce kernel."""
    lens = [40000, 5, 17000]
    c = cases.paged_batch(7300, "bfloat16", len(lens), 8, 1, 64, 32, lens)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    out = _run(c, d, 512)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 1, c["scale"], 32,
                                       c["max_seq_len"])
    assert_close(out, ref, ATOL_NS, RTOL_NS, "80 partitions")
    assert gpu.get_status(clear=True) == 0


def test_plan_reused_by_layers_and_graph_capture(gpu):
    """One plan serves many decodes (the counters return to zero), also when the
    plan and the decodes are replayed as one CUDA graph."""
    lens = list(np.random.default_rng(9).integers(100, 4000, size=64))
    c = cases.paged_batch(7400, "bfloat16", len(lens), 4, 1, 128, 16, lens)
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 1, c["scale"], 16,
                                       c["max_seq_len"])
    plan = mk.make_decode_plan(d["context_lens"], 1, c["max_seq_len"], 1024)
    ws = mk.splitk_workspace(len(lens), 4, 128, c["max_seq_len"], 1024)
    outs = [DeviceArray.empty((len(lens), 4, 128), "bfloat16") for _ in range(4)]
    st = Stream()

    def step():
        mk.make_decode_plan(d["context_lens"], 1, c["max_seq_len"], 1024, plan=plan, stream=st)
        for o in outs:
            mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 1,
                                  c["scale"], 16, c["max_seq_len"], partition_size=1024, workspace=ws, out=o,
                                  stream=st, plan=plan)

    step()
    st.synchronize()
    for o in outs:
        assert_close(o.to_numpy(), ref, ATOL_NS, RTOL_NS, "eager layer")
        o.fill_zero()
    _lib.synchronize()
    g = Graph.capture(st, step)
    for _ in range(3):
        g.replay(st)
    st.synchronize()
    for o in outs:
        assert_close(o.to_numpy(), ref, ATOL_NS, RTOL_NS, "graph replay")
    assert gpu.get_status(clear=True) == 0


def test_mismatched_plan_writes_nothing_and_flags(gpu):
    lens = [300, 900]
    c = cases.paged_batch(7500, "bfloat16", 2, 8, 2, 128, 16, lens)
    d = upload_case(c)
    fill_cache(d)
    # a plan for another max_seq_len: large enough to pass the size check, so the kernel must catch it
    big = mk.make_decode_plan(d["context_lens"], 2, 2 * c["max_seq_len"], 256)
    out = DeviceArray.from_numpy(np.full((2, 8, 128), 3.0, np.float32), dtype="bfloat16")
    mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 2, c["scale"], 16,
                          c["max_seq_len"], partition_size=256, out=out, plan=big)
    assert (out.to_numpy() == 3.0).all()
    assert gpu.get_status(clear=True) & _lib.STATUS_PLAN_MISMATCH


def test_config2_eight_way_share(gpu):
    """The share of one rank of an 8-GPU run of BASELINE config 2 (one KV head,
    256 sequences of U[512, 4096] tokens) with 2048-token partitions, against
    the plain split-K decode, plus a sample against the CPU oracle."""
    torch = pytest.importorskip("torch")
    from oracle import c_oracle

    w = cases.baseline_workload(2)
    lens = (w["lens"] + 1).astype(np.int32)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    kc = torch.randn((w["num_blocks"], 1, 16, 16, 8), generator=g, device=dev, dtype=torch.bfloat16)
    vc = torch.randn((w["num_blocks"], 1, 128, 16), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((256, 4, 128), generator=g, device=dev, dtype=torch.bfloat16)
    tables = DeviceArray.from_numpy(w["tables"])
    lens_d = DeviceArray.from_numpy(lens)
    scale = 1.0 / math.sqrt(128)
    plan = mk.make_decode_plan(lens_d, 1, w["max_seq_len"], 2048)
    out = mk.paged_attention_v2(q, kc, vc, tables, lens_d, 1, scale, 16, w["max_seq_len"], partition_size=2048,
                                plan=plan).to_numpy()
    v2 = mk.paged_attention_v2(q, kc, vc, tables, lens_d, 1, scale, 16, w["max_seq_len"],
                               partition_size=2048).to_numpy()
    assert_close(out, v2, ATOL_NS, RTOL_NS, "planned vs v2")
    rows = [0, 100, 255]
    nb = [(-(-int(lens[b]) // 16)) for b in rows]
    ids = np.concatenate([w["tables"][b, :n] for b, n in zip(rows, nb)]).astype(np.int64)
    t2 = np.zeros((3, max(nb)), np.uint32)
    o = 0
    for i, n in enumerate(nb):
        t2[i, :n] = np.arange(o, o + n)
        o += n
    idx = torch.from_numpy(ids).to(dev)

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    ref = c_oracle.paged_attention(bits(q[torch.tensor(rows, device=dev)]), "bfloat16", bits(kc.index_select(0, idx)),
                                   bits(vc.index_select(0, idx)), "bfloat16", t2, lens[rows], 1, scale,
                                   int(t2.shape[1] * 16))
    assert_close(out[rows], ref, ATOL_NS, RTOL_NS, "planned vs oracle")
    assert gpu.get_status(clear=True) == 0


# ---- the step's append folded into the decode (kvc_paged_attention_planned_append) ----

def _step_case(seed, dtype, lens, hq, hkv, D, bs):
    """A paged case whose caches hold every token but each sequence's last one,
    plus that last token (key/value [B, hkv, D], its slot) as the step's append."""
    c = cases.paged_batch(seed, dtype, len(lens), hq, hkv, D, bs, lens)
    ends = np.cumsum(c["context_lens"].astype(np.int64))
    last = [int(e) - 1 if n > 0 else -1 for e, n in zip(ends, c["context_lens"])]
    keep = np.ones(len(c["slot_mapping"]), bool)
    keep[[i for i in last if i >= 0]] = False
    B, dk = len(lens), c["k"].shape[1:]
    key = np.zeros((B,) + dk, c["k"].dtype)
    val = np.zeros((B,) + dk, c["v"].dtype)
    slot = np.full(B, -1, np.int64)
    for b, i in enumerate(last):
        if i >= 0:
            key[b], val[b], slot[b] = c["k"][i], c["v"][i], c["slot_mapping"][i]
    return c, keep, key, val, slot


def _caches(c, keep):
    """Fresh device caches holding the tokens of `keep` (every token but the step's)."""
    dt = c["dtype"]
    kc = DeviceArray.from_numpy(c["k_cache"], dtype=dt)
    vc = DeviceArray.from_numpy(c["v_cache"], dtype=dt)
    mk.reshape_and_cache(DeviceArray.from_numpy(c["k"][keep], dtype=dt), DeviceArray.from_numpy(c["v"][keep], dtype=dt),
                         kc, vc, DeviceArray.from_numpy(c["slot_mapping"][keep]))
    return kc, vc


def _both(c, keep, key, val, slot, msl, P, slot_dtype=np.int64):
    """(out, k_cache, v_cache) of append + planned decode, and of the folded call."""
    dt = c["dtype"]
    q = DeviceArray.from_numpy(c["q"], dtype=dt)
    bt, cl = DeviceArray.from_numpy(c["block_tables"]), DeviceArray.from_numpy(c["context_lens"])
    kd, vd, sd = (DeviceArray.from_numpy(key, dtype=dt), DeviceArray.from_numpy(val, dtype=dt),
                  DeviceArray.from_numpy(slot.astype(slot_dtype)))
    plan = mk.make_decode_plan(cl, c["num_kv_heads"], msl, P)
    kc, vc = _caches(c, keep)
    mk.reshape_and_cache(kd, vd, kc, vc, sd)
    two = mk.paged_attention_v2(q, kc, vc, bt, cl, c["num_kv_heads"], c["scale"], c["block_size"], msl,
                                partition_size=P, plan=plan).to_numpy()
    sep = (two, kc.to_numpy(), vc.to_numpy())
    kc2, vc2 = _caches(c, keep)
    one = mk.paged_attention_append(q, kd, vd, kc2, vc2, sd, bt, cl, c["num_kv_heads"], c["scale"], c["block_size"],
                                    msl, plan=plan).to_numpy()
    return sep, (one, kc2.to_numpy(), vc2.to_numpy())


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_folded_append_equals_append_then_decode(gpu, dtype, D, bs):
    """The folded call leaves the caches bit-identical to the append kernel's
    and gives the same output as the planned decode after it; both agree with
    the oracle.  Lengths put the new token first in a block, last in a block,
    and in sequences of one to many partitions."""
    lens = [1, bs, bs + 1, 300, 1025, 2048, 2049, 5000]
    c, keep, key, val, slot = _step_case(7600 + D + bs, dtype, lens, 8, 2, D, bs)
    (two, k2, v2), (one, k1, v1) = _both(c, keep, key, val, slot, c["max_seq_len"], 512)
    np.testing.assert_array_equal(k1, k2)
    np.testing.assert_array_equal(v1, v2)
    np.testing.assert_array_equal(one, two)
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], bs,
                                       c["max_seq_len"])
    assert_close(one, ref, ATOL_NS, RTOL_NS, f"folded append {dtype} D{D} bs{bs}")
    assert gpu.get_status(clear=True) == 0


def test_folded_append_edge_rules(gpu):
    """Padding slots (-1) skip their token, sequences of length 0 or past
    max_seq_len still get their token written (as the append kernel does) and
    produce zeros, an int32 slot mapping, one partition per sequence and the
    separate-reduce form (over 32 partitions) all match append + decode; a slot
    past the cache is skipped and flagged."""
    lens = [0, 5, 64, 5000, 700, 1, 33, 4096]
    c, keep, key, val, slot = _step_case(7700, "bfloat16", lens, 32, 8, 128, 16, )
    slot[2] = -1  # a padding token
    # sequence 0 (length 0) still appends a token, to the first slot of a block no table uses
    spare = sorted(set(range(c["k_cache"].shape[0])) - set(c["block_tables"].ravel().tolist()))[0]
    key[0], val[0], slot[0] = c["k"][0], c["v"][0], spare * 16
    for msl, P, sdt in ((4096, 512, np.int64), (c["max_seq_len"], 4096, np.int32), (c["max_seq_len"], 32, np.int64)):
        (two, k2, v2), (one, k1, v1) = _both(c, keep, key, val, slot, msl, P, sdt)
        np.testing.assert_array_equal(k1, k2)
        np.testing.assert_array_equal(v1, v2)
        np.testing.assert_array_equal(one, two)
        assert not one[0].any()
        if msl == 4096:
            assert not one[3].any()
    assert gpu.get_status(clear=True) == 0
    slot[4] = 10 ** 9  # past the cache: the folded call alone flags it
    dt = c["dtype"]
    kc, vc = _caches(c, keep)
    mk.paged_attention_append(DeviceArray.from_numpy(c["q"], dtype=dt), DeviceArray.from_numpy(key, dtype=dt),
                              DeviceArray.from_numpy(val, dtype=dt), kc, vc, DeviceArray.from_numpy(slot),
                              DeviceArray.from_numpy(c["block_tables"]), DeviceArray.from_numpy(c["context_lens"]), 8,
                              c["scale"], 16, c["max_seq_len"])
    assert gpu.get_status(clear=True) & _lib.STATUS_SLOT_OOB


def test_folded_append_replays_as_graph(gpu):
    """Captured once and replayed: every replay rewrites the same token and
    gives the eager result."""
    lens = [100, 2000, 3000, 17]
    c, keep, key, val, slot = _step_case(7800, "bfloat16", lens, 16, 4, 128, 16)
    dt = c["dtype"]
    q = DeviceArray.from_numpy(c["q"], dtype=dt)
    bt, cl = DeviceArray.from_numpy(c["block_tables"]), DeviceArray.from_numpy(c["context_lens"])
    kd, vd, sd = DeviceArray.from_numpy(key, dtype=dt), DeviceArray.from_numpy(val, dtype=dt), DeviceArray.from_numpy(slot)
    kc, vc = _caches(c, keep)
    st = Stream()
    plan = mk.make_decode_plan(cl, 4, c["max_seq_len"], 512, stream=st)
    ws = mk.splitk_workspace(len(lens), 16, 128, c["max_seq_len"], 512, 0)
    o = DeviceArray.empty(q.shape, dt)

    def work():
        mk.paged_attention_append(q, kd, vd, kc, vc, sd, bt, cl, 4, c["scale"], 16, c["max_seq_len"], plan=plan,
                                  workspace=ws, out=o, stream=st)

    work()
    st.synchronize()
    eager, keager = o.to_numpy(), kc.to_numpy()
    g = Graph.capture(st, work)
    for _ in range(2):
        o.fill_zero(stream=st)
        g.replay(st)
        st.synchronize()
        np.testing.assert_array_equal(o.to_numpy(), eager)
        np.testing.assert_array_equal(kc.to_numpy(), keager)


def test_folded_append_refuses_other_caches(gpu):
    """FP8 and float32 caches, a key of another dtype, a key without one row
    per sequence and rows off a 4-byte boundary are refused before anything runs."""
    lens = [40, 50]
    c, keep, key, val, slot = _step_case(7900, "float16", lens, 8, 2, 128, 16)
    q = DeviceArray.from_numpy(c["q"], dtype="float16")
    bt, cl = DeviceArray.from_numpy(c["block_tables"]), DeviceArray.from_numpy(c["context_lens"])
    kc, vc = _caches(c, keep)
    sd = DeviceArray.from_numpy(slot)
    with pytest.raises(NotImplementedError, match="dtype"):
        mk.paged_attention_append(q, DeviceArray.from_numpy(key, dtype="float32"),
                                  DeviceArray.from_numpy(val, dtype="float32"), kc, vc, sd, bt, cl, 2, c["scale"], 16,
                                  c["max_seq_len"])
    with pytest.raises(ValueError, match="one new token per sequence"):
        mk.paged_attention_append(q, DeviceArray.from_numpy(key[:1], dtype="float16"),
                                  DeviceArray.from_numpy(val[:1], dtype="float16"), kc, vc, sd, bt, cl, 2, c["scale"],
                                  16, c["max_seq_len"])
    wide = np.zeros(key.shape[:-1] + (key.shape[-1] + 1,), np.float32)
    wide[..., 1:] = key
    kw = DeviceArray.from_numpy(wide, dtype="float16")[:, :, 1:]  # odd offset and strides
    with pytest.raises(NotImplementedError):
        mk.paged_attention_append(q, kw, DeviceArray.from_numpy(val, dtype="float16"), kc, vc, sd, bt, cl, 2,
                                  c["scale"], 16, c["max_seq_len"])
    c32 = cases.paged_batch(7901, "float32", 2, 8, 2, 128, 16, lens)
    q32 = DeviceArray.from_numpy(c32["q"], dtype="float32")
    k32 = DeviceArray.from_numpy(c32["k_cache"], dtype="float32")
    v32 = DeviceArray.from_numpy(c32["v_cache"], dtype="float32")
    with pytest.raises(NotImplementedError):
        mk.paged_attention_append(q32, DeviceArray.from_numpy(key, dtype="float32"),
                                  DeviceArray.from_numpy(val, dtype="float32"), k32, v32, sd, bt, cl, 2, c["scale"],
                                  16, c["max_seq_len"])


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("bs", [8, 16])
def test_whole_sequence_partitions_on_ten_warps(gpu, dtype, bs, monkeypatch):
    """Few (sequence, KV head) pairs per SM and whole sequences of up to 4096
    tokens per partition: the decode runs on 10-warp CTAs (one per SM).  Its
    output matches the oracle and, within the tolerance, the 4-warp CTAs on the
    same plan (forced through KVC_MMA_CONFIG)."""
    lens = [1, bs - 1, bs, bs + 1, 300, 2049, 4000, 4096, 1025, 777]
    c = cases.paged_batch(7700 + bs, dtype, len(lens), 8, 2, 128, bs, lens)
    assert c["max_seq_len"] <= 4096 + 2 * bs
    assert mk.choose_planned_partition(len(lens), 2, c["max_seq_len"], bs, lens) == 4096
    d = upload_case(c)
    fill_cache(d)
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], bs,
                                       c["max_seq_len"])
    wide = _run(c, d, 4096)
    assert_close(wide, ref, ATOL_NS, RTOL_NS, f"10-warp planned {dtype} bs{bs}")
    monkeypatch.setenv("KVC_MMA_CONFIG", "4x3x16")
    four = _run(c, d, 4096)
    assert_close(wide, four, ATOL_NS, RTOL_NS, "10-warp vs 4-warp CTAs")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_folded_append_on_ten_warps(gpu, dtype):
    """The folded append in the 10-warp form: caches bit-identical to the append
    kernel's, output equal to the planned decode after it, and the oracle."""
    lens = [1, 16, 17, 300, 2048, 2049, 4096, 3000]
    c, keep, key, val, slot = _step_case(7800, dtype, lens, 8, 2, 128, 16)
    assert c["max_seq_len"] <= 4096 + 32
    (two, k2, v2), (one, k1, v1) = _both(c, keep, key, val, slot, c["max_seq_len"], 4096)
    np.testing.assert_array_equal(k1, k2)
    np.testing.assert_array_equal(v1, v2)
    np.testing.assert_array_equal(one, two)
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], 2, c["scale"], 16,
                                       c["max_seq_len"])
    assert_close(one, ref, ATOL_NS, RTOL_NS, f"folded append, 10 warps, {dtype}")
    assert gpu.get_status(clear=True) == 0
