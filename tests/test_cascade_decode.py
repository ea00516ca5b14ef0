"""GPU parity tests of the shared-prefix ("cascade") decode,
kvc_paged_attention_cascade.  The result must equal paged_attention_v1 on the
same inputs, so the oracle is kv_oracle.paged_attention_v1 (float64, pinned to
the reference's own oracle).  Cases: every dtype / head size / block size of
the tensor-core path, group sizes, sequences shorter than the prefix and rows
the reference zeroes, every partition layout, the prefix-mismatch flag, the
BASELINE config 4 shape, and graph replay."""

import math

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close, fill_cache, oracle_fill, upload_case
from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray

pytestmark = pytest.mark.gpu


def cascade_case(seed, dtype, num_seqs, hq, hkv, d, bs, prefix, lens):
    """A batch whose tables all start with the same prefix // bs blocks; sequence b
    has context lens[b] (shorter than the prefix, or the prefix plus its own tail)."""
    rng = np.random.default_rng(seed)
    pb = prefix // bs
    tails = [max(0, int(n) - prefix) for n in lens]
    tb = [-(-t // bs) for t in tails]
    num_blocks = pb + sum(tb) + 3
    perm = rng.permutation(num_blocks).astype(np.int32)
    max_blocks = max(pb + max(tb), 1)
    tables = np.full((num_seqs, max_blocks), -1, np.int32)
    pos = pb
    for b in range(num_seqs):
        tables[b, :pb] = perm[:pb]
        tables[b, pb:pb + tb[b]] = perm[pos:pos + tb[b]]
        pos += tb[b]
    # tokens: the prefix once, then every tail
    ntok = prefix + sum(tails)
    slots = np.empty(ntok, np.int64)
    t = np.arange(prefix)
    slots[:prefix] = perm[t // bs].astype(np.int64) * bs + t % bs
    o = prefix
    for b in range(num_seqs):
        t = np.arange(prefix, prefix + tails[b])
        slots[o:o + tails[b]] = tables[b, t // bs].astype(np.int64) * bs + t % bs
        o += tails[b]
    q = cases.cast(rng.standard_normal((num_seqs, hq, d), dtype=np.float32), dtype)
    k = cases.cast(rng.standard_normal((ntok, hkv, d), dtype=np.float32), dtype)
    v = cases.cast(rng.standard_normal((ntok, hkv, d), dtype=np.float32), dtype)
    store = np.float16 if dtype == "float16" else np.float32
    x = 8
    return dict(q=q, k=k, v=v, k_cache=np.zeros((num_blocks, hkv, d // x, bs, x), store),
                v_cache=np.zeros((num_blocks, hkv, d, bs), store), context_lens=np.asarray(lens, np.int32),
                block_tables=tables, slot_mapping=slots.astype(np.int32), num_kv_heads=hkv,
                scale=1.0 / math.sqrt(d), block_size=bs, max_seq_len=max_blocks * bs, dtype=dtype, prefix=prefix)


def ref_of(c, max_seq_len=None):
    kc, vc = oracle_fill(c, c["dtype"])
    return kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                        c["scale"], c["block_size"], max_seq_len or c["max_seq_len"])


def run_cascade(d, c, max_seq_len=None, **kw):
    return mk.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                      c["num_kv_heads"], c["scale"], c["block_size"], max_seq_len or c["max_seq_len"],
                                      c["prefix"], **kw).to_numpy()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_dtype_headsize_blocksize_matrix(gpu, dtype, D, bs):
    c = cascade_case(5000 + D + bs, dtype, 6, 16, 4, D, bs, 256, [256, 257, 273, 356, 556, 261])
    d = upload_case(c)
    fill_cache(d)
    assert_close(run_cascade(d, c), ref_of(c), ATOL_NS, RTOL_NS, f"{dtype} D{D} bs{bs}")
    assert gpu.get_status(clear=True) == 0


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (28, 4), (32, 4), (32, 2), (64, 8), (16, 1), (64, 4), (32, 1)])
def test_group_sizes(gpu, Hq, Hkv):
    c = cascade_case(5100 + Hq + Hkv, "bfloat16", 11, Hq, Hkv, 128, 16, 512, [512 + 37 * i for i in range(11)])
    d = upload_case(c)
    fill_cache(d)
    if Hq // Hkv > 16:  # the tensor-core tiles hold at most 16 query heads of a group
        with pytest.raises(NotImplementedError, match="16 query heads"):
            run_cascade(d, c)
        return
    assert_close(run_cascade(d, c), ref_of(c), ATOL_NS, RTOL_NS, f"G={Hq // Hkv}")


def test_short_and_zero_rows(gpu):
    """Sequences shorter than the prefix attend to their own length; rows the
    reference zeroes (length 0, or past max_seq_len) stay zero."""
    lens = [0, 1, 100, 255, 256, 300, 700, 5000]
    c = cascade_case(5200, "bfloat16", len(lens), 32, 8, 128, 16, 256, [max(x, 1) for x in lens])
    c["context_lens"] = np.asarray(lens, np.int32)
    d = upload_case(c)
    fill_cache(d)
    out = run_cascade(d, c)
    assert not out[0].any()
    assert_close(out, ref_of(c), ATOL_NS, RTOL_NS, "short rows")
    out = run_cascade(d, c, max_seq_len=1024)
    assert not out[7].any()
    assert_close(out, ref_of(c, max_seq_len=1024), ATOL_NS, RTOL_NS, "max_seq_len")


@pytest.mark.parametrize("pp,pt", [(32, 32), (64, 256), (256, 1024), (1024, 64), (96, 160)])
def test_partition_layouts(gpu, pp, pt):
    c = cascade_case(5300 + pp + pt, "float16", 9, 32, 8, 128, 16, 1024, [1024 + 61 * i for i in range(9)])
    d = upload_case(c)
    fill_cache(d)
    assert_close(run_cascade(d, c, prefix_partition_size=pp, partition_size=pt), ref_of(c), ATOL_NS, RTOL_NS,
                 f"pp={pp} pt={pt}")


def test_prefix_mismatch_is_flagged(gpu):
    c = cascade_case(5400, "float16", 4, 16, 4, 128, 16, 256, [300, 300, 300, 300])
    d = upload_case(c)
    fill_cache(d)
    bt = c["block_tables"].copy()
    bt[2, 3] = bt[2, 17]  # sequence 2 no longer starts with the shared blocks (17: one of its tail blocks)
    d["block_tables"] = DeviceArray.from_numpy(bt)
    gpu.get_status(clear=True)
    run_cascade(d, c)
    assert gpu.get_status(clear=True) & _lib.STATUS_PREFIX_MISMATCH


def test_unsupported_inputs_are_refused(gpu):
    c = cascade_case(5500, "float16", 2, 8, 2, 128, 16, 64, [70, 80])
    d = upload_case(c)
    fill_cache(d)
    from sglang_mlx_b200.dlpack import as_dltensor

    es, ml, to = mk.cascade_workspace(2, 8, 128, c["max_seq_len"], 64, 32, 32)
    out = DeviceArray.empty(d["q"].shape, "float16")
    al = DeviceArray.from_numpy(np.ones(8, np.float32))
    args = [as_dltensor(a)[0] for a in (out, es, ml, to, d["q"], d["k_cache"], d["v_cache"], d["block_tables"],
                                         d["context_lens"])]
    with pytest.raises(NotImplementedError, match="alibi"):
        _lib.check(_lib.lib.kvc_paged_attention_cascade(*args, 2, c["scale"], 16, c["max_seq_len"], as_dltensor(al)[0],
                                                        64, 32, 32, None))
    cf = cascade_case(5501, "float16", 2, 8, 2, 128, 16, 64, [70, 80])
    df = upload_case(cf, q_dtype="float32", cache_dtype="float16")
    fill_cache(df)
    with pytest.raises(NotImplementedError, match="float16/bfloat16"):
        run_cascade(df, cf)
    with pytest.raises(ValueError, match="shared_prefix_len"):
        mk.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 2,
                                   c["scale"], 16, c["max_seq_len"], 40)


def test_config4_shape_against_split_k(gpu):
    """64 sequences, 64/8 heads, one 2048-token prefix and a
    256-token tail each (bf16, bs 16): cascade == split-K decode, and the
    oracle on a few sequences."""
    c = cascade_case(5600, "bfloat16", 64, 64, 8, 128, 16, 2048, [2048 + 255] * 64)
    d = upload_case(c)
    fill_cache(d)
    out = run_cascade(d, c)
    v2 = mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 8,
                               c["scale"], 16, c["max_seq_len"], partition_size=512).to_numpy()
    assert_close(out, v2.astype(np.float64), ATOL_NS, RTOL_NS, "cascade vs split-K")
    pick = [0, 31, 63]
    kc, vc = oracle_fill(c, "bfloat16")
    ref = kv_oracle.paged_attention_v1(c["q"][pick], kc, vc, c["block_tables"][pick], c["context_lens"][pick], 8,
                                       c["scale"], 16, c["max_seq_len"])
    assert_close(out[pick], ref, ATOL_NS, RTOL_NS, "oracle subset")
    assert gpu.get_status(clear=True) == 0


def test_replays_as_cuda_graph(gpu):
    from sglang_mlx_b200.device_array import Graph, Stream

    c = cascade_case(5700, "bfloat16", 8, 32, 8, 128, 16, 512, [700] * 8)
    d = upload_case(c)
    fill_cache(d)
    st = Stream()
    pp, pt = mk.cascade_partitions(8, 32, 8, c["max_seq_len"], 512, 16)
    ws = mk.cascade_workspace(8, 32, 128, c["max_seq_len"], 512, pp, pt)
    o = DeviceArray.empty(d["q"].shape, "bfloat16")

    def work():
        mk.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], 8,
                                   c["scale"], 16, c["max_seq_len"], 512, workspace=ws, out=o, stream=st)

    work()
    st.synchronize()
    eager = o.to_numpy()
    g = Graph.capture(st, work)
    for _ in range(2):
        o.fill_zero(stream=st)
        g.replay(st)
        st.synchronize()
        np.testing.assert_array_equal(o.to_numpy(), eager)
    assert_close(eager, ref_of(c), ATOL_NS, RTOL_NS, "graph")


@pytest.mark.parametrize("num_seqs,bs", [(40, 16), (16, 32), (100, 16)])
def test_two_tile_and_one_tile_prefix_forms(gpu, monkeypatch, num_seqs, bs):
    """The shared prefix on the gathered-K tcgen05 kernel runs items of two
    128-row tiles of (sequence, head) rows: 40 x 8 rows = 3 tiles (the second
    pair's tile B empty), 16 x 8 = 1 tile, 100 x 8 = 7 tiles; with sequences
    shorter than the prefix.  The result matches the oracle and the one-tile
    kernel (KVC_PREFILL_PAIR=0); KVC_PREFILL_PAIR=1 forces the two-tile kernel
    (unset, it runs only when its items fill the SMs)."""
    lens = [1024 + 13 * i if i % 5 else 300 + i for i in range(num_seqs)]
    c = cascade_case(5800 + num_seqs + bs, "bfloat16", num_seqs, 64, 8, 128, bs, 1024, lens)
    d = upload_case(c)
    fill_cache(d)
    r = ref_of(c)
    monkeypatch.setenv("KVC_PREFILL_PAIR", "1")
    two = run_cascade(d, c)
    assert_close(two, r, ATOL_NS, RTOL_NS, "two-tile prefix")
    monkeypatch.setenv("KVC_PREFILL_PAIR", "0")
    one = run_cascade(d, c)
    assert_close(one, r, ATOL_NS, RTOL_NS, "one-tile prefix")
    assert gpu.get_status(clear=True) == 0
