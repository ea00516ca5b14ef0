"""GPU tests of copy_blocks / swap_blocks through the C ABI, bit-exact against
oracle/kv_oracle.py (copy_blocks.metal:9-75).

The first two tests are the reference's own (test_paged_attention_kernel.py:
400-438); the rest cover the paged-cache layouts, every mapping placement
(device int32/int64, host list, host NumPy), host <-> device swaps through
pinned and pageable memory, odd block sizes (each vector width of the copy
kernel), more pairs and layers than one launch carries, and the bounds checks."""

import numpy as np
import pytest

from oracle import kv_oracle
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray, HostBuffer

pytestmark = pytest.mark.gpu


def test_copy_blocks_multiple_layers(gpu):
    """test_paged_attention_kernel.py:400-425."""
    key_caches, value_caches, key_before, value_before = [], [], [], []
    for layer in range(2):
        key_np = np.arange(24, dtype=np.float32).reshape(4, 2, 3) + layer * 100
        value_np = key_np + 1000
        key_before.append(key_np.copy())
        value_before.append(value_np.copy())
        key_caches.append(DeviceArray.from_numpy(key_np))
        value_caches.append(DeviceArray.from_numpy(value_np))
    mapping = DeviceArray.from_numpy(np.array([[0, 2], [1, 3]], dtype=np.int32))
    new_keys, new_values = mk.copy_blocks(key_caches, value_caches, mapping)
    for layer in range(2):
        expected_key = key_before[layer].copy()
        expected_value = value_before[layer].copy()
        expected_key[2] = key_before[layer][0]
        expected_key[3] = key_before[layer][1]
        expected_value[2] = value_before[layer][0]
        expected_value[3] = value_before[layer][1]
        np.testing.assert_array_equal(new_keys[layer].to_numpy(), expected_key)
        np.testing.assert_array_equal(new_values[layer].to_numpy(), expected_value)
        assert new_keys[layer] is key_caches[layer]  # updated in place


def test_swap_blocks_noncontiguous_mapping(gpu):
    """test_paged_attention_kernel.py:427-438."""
    src_np = np.arange(24, dtype=np.float32).reshape(4, 2, 3)
    dst_np = np.full((4, 2, 3), -1, dtype=np.float32)
    out = mk.swap_blocks(DeviceArray.from_numpy(src_np), DeviceArray.from_numpy(dst_np),
                         DeviceArray.from_numpy(np.array([[0, 2], [3, 1]], dtype=np.int32)))
    expected = dst_np.copy()
    expected[2] = src_np[0]
    expected[1] = src_np[3]
    np.testing.assert_array_equal(out.to_numpy(), expected)


@pytest.mark.parametrize("mapping_kind", ["device_i32", "device_i64", "host_list", "host_numpy"])
def test_copy_blocks_paged_layouts_match_oracle(gpu, mapping_kind):
    rng = np.random.default_rng(41)
    layers, nb = 4, 40
    ks = [rng.standard_normal((nb, 8, 16, 16, 8)).astype(np.float16) for _ in range(layers)]
    vs = [rng.standard_normal((nb, 8, 128, 16)).astype(np.float16) for _ in range(layers)]
    dk = [DeviceArray.from_numpy(k) for k in ks]
    dv = [DeviceArray.from_numpy(v) for v in vs]
    src = rng.choice(nb // 2, size=12, replace=False)
    dst = nb // 2 + rng.choice(nb // 2, size=12, replace=False)
    pairs = np.stack([src, dst], axis=1)
    mapping = {"device_i32": DeviceArray.from_numpy(pairs.astype(np.int32)),
               "device_i64": DeviceArray.from_numpy(pairs.astype(np.int64)),
               "host_list": pairs.tolist(),
               "host_numpy": pairs.astype(np.int64)}[mapping_kind]
    mk.copy_blocks(dk, dv, mapping)
    kv_oracle.copy_blocks(ks, vs, pairs)
    for i in range(layers):
        np.testing.assert_array_equal(dk[i].to_numpy(), ks[i])
        np.testing.assert_array_equal(dv[i].to_numpy(), vs[i])
    assert gpu.get_status(clear=True) == 0


def test_copy_blocks_more_pairs_and_layers_than_one_launch(gpu):
    """40 layers (80 planes, three launches) and 300 host pairs (three parameter chunks)."""
    rng = np.random.default_rng(42)
    layers, nb = 40, 700
    ks = [rng.standard_normal((nb, 2, 16)).astype(np.float32) for _ in range(layers)]
    vs = [rng.standard_normal((nb, 2, 16)).astype(np.float32) for _ in range(layers)]
    dk = [DeviceArray.from_numpy(k) for k in ks]
    dv = [DeviceArray.from_numpy(v) for v in vs]
    perm = rng.permutation(nb)
    pairs = np.stack([perm[:300], perm[300:600]], axis=1)
    mk.copy_blocks(dk, dv, pairs)
    kv_oracle.copy_blocks(ks, vs, pairs)
    for i in range(layers):
        np.testing.assert_array_equal(dk[i].to_numpy(), ks[i])
        np.testing.assert_array_equal(dv[i].to_numpy(), vs[i])


@pytest.mark.parametrize("shape,dtype", [((9, 3), "uint8"), ((9, 2, 3), "float16"), ((9, 6), "float32"),
                                         ((9, 2, 4), "float32"), ((9, 16), "uint8")])
def test_odd_block_sizes_use_every_vector_width(gpu, shape, dtype):
    rng = np.random.default_rng(43)
    if dtype == "uint8":
        src = rng.integers(0, 256, size=shape, dtype=np.uint8)
        dst = rng.integers(0, 256, size=shape, dtype=np.uint8)
    else:
        np_dt = {"float16": np.float16, "float32": np.float32}[dtype]
        src = (rng.standard_normal(shape) * 50).astype(np_dt)
        dst = (rng.standard_normal(shape) * 50).astype(np_dt)
    pairs = np.array([[0, 8], [3, 1], [7, 4]], dtype=np.int64)
    out = mk.swap_blocks(DeviceArray.from_numpy(src), DeviceArray.from_numpy(dst), pairs)
    np.testing.assert_array_equal(out.to_numpy(), kv_oracle.swap_blocks(src, dst.copy(), pairs))


def test_swap_between_device_and_pinned_host(gpu):
    """Offload device blocks to pinned host memory and bring them back."""
    rng = np.random.default_rng(44)
    nb, shape = 32, (8, 16, 16, 8)
    dev_np = rng.standard_normal((nb,) + shape).astype(np.float16)
    d = DeviceArray.from_numpy(dev_np)
    host = HostBuffer((nb,) + shape, "float16")
    host.array[...] = 0
    out = [[1, 0], [2, 1], [3, 2], [10, 7], [31, 30]]  # one run of three consecutive pairs
    mk.swap_blocks(d, host, out)
    _lib.synchronize()
    expect = kv_oracle.swap_blocks(dev_np, np.zeros_like(dev_np), out)
    np.testing.assert_array_equal(host.array, expect)
    # back into fresh device blocks
    d2 = DeviceArray.from_numpy(np.zeros_like(dev_np))
    back = [[0, 5], [1, 6], [2, 7], [7, 20], [30, 0]]
    mk.swap_blocks(host, d2, back)
    np.testing.assert_array_equal(d2.to_numpy(), kv_oracle.swap_blocks(expect, np.zeros_like(dev_np), back))


def test_swap_with_pageable_numpy(gpu):
    rng = np.random.default_rng(45)
    src_np = rng.standard_normal((6, 4, 32)).astype(np.float32)
    d = DeviceArray.from_numpy(np.zeros_like(src_np))
    mk.swap_blocks(src_np, d, [[5, 0], [0, 5]])
    host_out = np.zeros_like(src_np)
    mk.swap_blocks(d, host_out, [[0, 1], [5, 2]])
    _lib.synchronize()
    exp = np.zeros_like(src_np)
    exp[1], exp[2] = src_np[5], src_np[0]
    np.testing.assert_array_equal(host_out, exp)


def test_out_of_range_pairs_are_skipped_and_flagged(gpu):
    src_np = np.arange(24, dtype=np.float32).reshape(4, 6)
    dst_np = np.full((4, 6), -1, dtype=np.float32)
    gpu.get_status(clear=True)
    out = mk.swap_blocks(DeviceArray.from_numpy(src_np), DeviceArray.from_numpy(dst_np),
                         np.array([[0, 1], [9, 2], [2, -1], [3, 3]], dtype=np.int64))
    exp = dst_np.copy()
    exp[1], exp[3] = src_np[0], src_np[3]
    np.testing.assert_array_equal(out.to_numpy(), exp)
    assert gpu.get_status(clear=True) & _lib.STATUS_INDEX_OOB


def test_host_path_rejects_out_of_range_pairs(gpu):
    d = DeviceArray.from_numpy(np.zeros((4, 6), np.float32))
    host = np.zeros((4, 6), np.float32)
    with pytest.raises(ValueError, match="out of range"):
        mk.swap_blocks(d, host, [[0, 4]])


def test_python_shim_messages(gpu):
    k = [DeviceArray.from_numpy(np.zeros((4, 6), np.float32))]
    with pytest.raises(ValueError, match="size mismatch"):
        mk.copy_blocks(k, [], [[0, 1]])
    with pytest.raises(ValueError, match=r"shape \[num_pairs, 2\]"):
        mk.copy_blocks(k, k, [[0, 1, 2]])
