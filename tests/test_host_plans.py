"""Host-side planning helpers of the Python shim (no GPU)."""
import math

import cases

from sglang_mlx_b200 import metal_kernels as mk


def test_cascade_partitions_config4():
    # 64 sequences, 64 / 8 heads, a 2048-token shared prefix and 256 tail tokens, block size 16:
    # 8 tiles of 64 rows x 8 kv heads -> 4 prefix chunks of 512 (one wave), one 256-token tail partition
    assert mk.cascade_partitions(64, 64, 8, 2304, 2048, 16) == (512, 256)


def test_cascade_partitions_units_and_bounds():
    for bs in (8, 16, 32):
        unit = 32 * bs // math.gcd(32, bs)
        for B, Hq, Hkv, prefix, tail in [(1, 8, 8, 100, 0), (3, 28, 4, 4096, 5000), (512, 32, 8, 64, 17),
                                         (7, 16, 1, 33, 1024), (7, 16, 1, 33, 1025)]:
            pp, pt = mk.cascade_partitions(B, Hq, Hkv, prefix + tail, prefix, bs)
            assert pp % unit == 0 and pp >= unit and pp >= -(-prefix // max(1, 2 * 148))
            assert pt % unit == 0 and pt >= unit
            if tail > 1024:
                assert pt == 1024
            else:
                assert pt >= tail
            tiles = -(-B * (Hq // Hkv) // 64)
            chunks = -(-prefix // pp)
            # one wave of the prefix kernel (unless one chunk per kv head and tile already exceeds it)
            assert chunks * tiles * Hkv <= max(2 * 148, tiles * Hkv)



def test_planned_partition_choice():
    """choose_planned_partition: whole sequences of up to 4096 tokens when there
    are at most two (sequence, KV head) pairs per SM (head size 128, blocks of
    up to 16 tokens: the 10-warp decode); otherwise the largest of
    4096/2048/1024/512 tokens whose items fill 1.25x the resident CTA slots
    (296 for 16-token blocks)."""
    from sglang_mlx_b200 import metal_kernels as mk

    lens = cases.baseline_workload(2)["lens"] + 1
    assert mk.choose_planned_partition(256, 1, 4112, 16, lens) == 4096   # one rank of an 8-GPU run: 10-warp CTAs
    assert mk.choose_planned_partition(256, 1, 4112, 16, lens, head_size=64) == 2048   # no 10-warp form: 1.25 slots
    assert mk.choose_planned_partition(256, 2, 4112, 16, lens) == 4096
    assert mk.choose_planned_partition(256, 8, 4112, 16, lens) == 4096
    assert mk.choose_planned_partition(300, 1, 4112, 16) == 2048   # more than two pairs per SM
    assert mk.choose_planned_partition(64, 1, 8192, 16) == 512   # sequences longer than one 4096-token partition
    assert mk.choose_planned_partition(4, 1, 300, 16, [100, 200, 300, 50]) == 4096   # whole sequences
    assert mk.choose_planned_partition(4, 1, 300, 32, [100, 200, 300, 50]) == 512   # too few items for any size
    assert mk.choose_planned_partition(1, 8, 131072, 32) == 512   # one 128k sequence (taken as 64k): 1024 gives 512 items < 555
    for bs in (8, 16, 32):
        p = mk.choose_planned_partition(64, 8, 8192, bs)
        assert p % 32 == 0 and p % bs == 0
