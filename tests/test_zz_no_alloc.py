"""The allocation-free split-K decode (kvc_paged_attention_v2_noalloc).

Some users of this library cannot hand it device memory: a host framework that
owns every byte of the GPU through its own pool, a serving loop that cannot
afford the device-wide stall of cudaMalloc/cudaFree, or a binding from another
language that has no device allocator to call.  For them the split-K decode
keeps its partial results in a fixed 16 MiB array compiled into the library
instead of the three workspace tensors kvc_paged_attention_v2 asks for.

This file is collected last on purpose: if it fails, every other test has
already run.  It works both alone in a fresh process and after the others.
"""

import ctypes

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close, fill_cache, upload_case
from sglang_mlx_b200 import _lib
from sglang_mlx_b200 import metal_kernels as mk
from sglang_mlx_b200.device_array import DeviceArray
from sglang_mlx_b200.dlpack import as_dltensor, make_dltensor

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # KVC_NOALLOC_SCRATCH_BYTES in include/kvcache.h


def noalloc(d, c, partition_size, out):
    """One call of the allocation-free entry point straight through the C ABI."""
    ptrs = [as_dltensor(x) for x in (out, d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"])]
    rc = _lib.lib.kvc_paged_attention_v2_noalloc(
        ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0], ptrs[5][0], c["num_kv_heads"], c["scale"],
        c["block_size"], c["max_seq_len"], None, partition_size, None)
    _lib.check(rc)
    return out


@pytest.mark.parametrize("dtype,bs,lens", [
    ("bfloat16", 32, [4096 - 7, 513, 1, 2048]),  # long-context split-K shape, 32-token blocks
    ("float16", 16, [700, 33, 1500]),
])
def test_noalloc_matches_the_workspace_entry_point(gpu, dtype, bs, lens):
    c = cases.paged_batch(4242 + bs, dtype, len(lens), 32, 8, 128, bs, lens)
    d = upload_case(c)
    fill_cache(d)
    psize = 512
    # the existing entry point, with caller-owned workspace
    want = mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"],
                                 c["num_kv_heads"], c["scale"], bs, c["max_seq_len"],
                                 partition_size=psize).to_numpy()
    # two calls in a row share the static scratch; both must match
    for _ in range(2):
        out = DeviceArray.empty(d["q"].shape, dtype)
        got = noalloc(d, c, psize, out).to_numpy()
        assert_close(got, want, ATOL_NS, RTOL_NS, "noalloc vs workspace split-K")
    assert gpu.get_status(clear=True) == 0


def test_noalloc_rejects_work_beyond_its_scratch(gpu):
    """64 seqs x 64 heads x 8 partitions x (128 + 2) floats is 17 MB > 16 MiB:
    refused before anything is launched."""
    fake = 0x10000
    keep = []

    def t(shape, dtype):
        acc, st = 1, []
        for s in reversed(shape):
            st.append(acc)
            acc *= s
        dl, k = make_dltensor(fake, shape, tuple(reversed(st)), dtype, 0)
        keep.append((dl, k))
        return ctypes.pointer(dl)

    need = 64 * 64 * 8 * (128 + 2) * 4
    assert need > SCRATCH_BYTES
    rc = _lib.lib.kvc_paged_attention_v2_noalloc(
        t((64, 64, 128), "bfloat16"), t((64, 64, 128), "bfloat16"), t((100, 8, 16, 16, 8), "bfloat16"),
        t((100, 8, 128, 16), "bfloat16"), t((64, 256), "int32"), t((64,), "int32"), 8, 0.1, 16, 4096, None, 512,
        None)
    assert rc == _lib.KVC_EINVAL
    assert "static scratch" in _lib.last_error()
