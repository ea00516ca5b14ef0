"""BASELINE.json configs 2-5 at full size on the GPU (one layer each).

The caches are filled on the device (seeded N(0,1)); the step's new tokens
(one per decode sequence, plus config 5's prefill chunks) go through
reshape_and_cache.  Checks, size-independent where the oracle cannot follow:
  * every appended slot holds exactly its input row (bit-exact);
  * a sample of sequences agrees with the CPU oracle (float64 gather + SDPA),
    including the sequences that share config 4's prefix blocks;
  * the single-pass and split-K decodes agree on every sequence, and all
    outputs are finite.
"""

import math

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close
from oracle import c_oracle
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf16(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("config", [2, 3, 4, 5])
def test_baseline_config_step(gpu, config):
    w = cases.baseline_workload(config)
    cfg = w["cfg"]
    B, HQ, HKV, D, BS = cfg["batch"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["bs"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(100 + config)
    kc = torch.randn((w["num_blocks"], HKV, D // 8, BS, 8), generator=g, device=dev, dtype=torch.bfloat16)
    vc = torch.randn((w["num_blocks"], HKV, D, BS), generator=g, device=dev, dtype=torch.bfloat16)
    slots = np.concatenate([w["prefill_slots"], w["decode_slots"]]).astype(np.int32)
    kn = torch.randn((len(slots), HKV, D), generator=g, device=dev, dtype=torch.bfloat16)
    vn = torch.randn((len(slots), HKV, D), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((B, HQ, D), generator=g, device=dev, dtype=torch.bfloat16)
    lens_after = (w["lens"] + 1).astype(np.int32)
    tables = DeviceArray.from_numpy(w["tables"])
    lens = DeviceArray.from_numpy(lens_after)

    mk.reshape_and_cache(kn, vn, kc, vc, DeviceArray.from_numpy(slots))
    scale = 1.0 / math.sqrt(D)
    v1 = mk.paged_attention_v1(q, kc, vc, tables, lens, HKV, scale, BS, w["max_seq_len"]).to_numpy()
    psize = cfg["partition"] or 512
    v2 = mk.paged_attention_v2(q, kc, vc, tables, lens, HKV, scale, BS, w["max_seq_len"],
                               partition_size=psize).to_numpy()
    auto = mk.paged_attention(q, kc, vc, tables, lens, HKV, scale, BS, w["max_seq_len"]).to_numpy()
    torch.cuda.synchronize()
    assert np.isfinite(v1).all() and np.isfinite(v2).all()
    assert_close(v2, v1, ATOL_NS, RTOL_NS, f"config {config}: split-K vs single pass")
    assert_close(auto, v1, ATOL_NS, RTOL_NS, f"config {config}: auto vs single pass")
    assert gpu.get_status(clear=True) == 0

    # appended rows, bit-exact (a spread of them)
    pick = np.unique(np.linspace(0, len(slots) - 1, num=min(len(slots), 64)).astype(int))
    knb, vnb = _bits(kn), _bits(vn)
    for t in pick:
        s = int(slots[t])
        blk, off = s // BS, s % BS
        krow = _bits(kc[blk, :, :, off, :]).reshape(HKV, D)
        vrow = _bits(vc[blk, :, :, off]).reshape(HKV, D)
        np.testing.assert_array_equal(krow, knb[t])
        np.testing.assert_array_equal(vrow, vnb[t])

    # sample of sequences against the CPU oracle
    sample = np.unique(np.linspace(0, B - 1, num=min(B, 6)).astype(int))
    nb = [(-(-int(lens_after[b]) // BS)) for b in sample]
    blocks = np.concatenate([w["tables"][b, :n] for b, n in zip(sample, nb)]).astype(np.int64)
    t2 = np.zeros((len(sample), max(nb)), np.uint32)
    o = 0
    for i, n in enumerate(nb):
        t2[i, :n] = np.arange(o, o + n)
        o += n
    idx = torch.from_numpy(blocks).to(dev)
    ref = c_oracle.paged_attention(_bits(q[torch.from_numpy(sample).to(dev)]), "bfloat16",
                                   _bits(kc.index_select(0, idx)), _bits(vc.index_select(0, idx)), "bfloat16", t2,
                                   lens_after[sample], HKV, scale, int(t2.shape[1] * BS))
    assert_close(v1[sample], ref, ATOL_NS, RTOL_NS, f"config {config}: single pass vs oracle")
    assert_close(v2[sample], ref, ATOL_NS, RTOL_NS, f"config {config}: split-K vs oracle")
    if config == 4:
        # every sequence reads the same prefix blocks: the shared pages are really shared
        assert (w["tables"][:, :cfg["prefix"] // BS] == w["tables"][0, :cfg["prefix"] // BS]).all()
