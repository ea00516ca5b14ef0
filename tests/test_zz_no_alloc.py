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
import math
import os
import subprocess
import sys

import numpy as np
import pytest

import cases
from helpers import ATOL_NS, RTOL_NS, assert_close, fill_cache, oracle_fill, upload_case
from oracle import kv_oracle
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


def need_bytes(num_seqs, num_heads, max_seq_len, partition_size, head_size):
    return num_seqs * num_heads * (-(-max_seq_len // partition_size)) * (head_size + 2) * 4


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
    kc, vc = oracle_fill(c, dtype)
    ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], c["num_kv_heads"],
                                       c["scale"], bs, c["max_seq_len"])
    # two calls in a row share the static scratch; both must match
    for _ in range(2):
        out = DeviceArray.empty(d["q"].shape, dtype)
        got = noalloc(d, c, psize, out).to_numpy()
        assert_close(got, want, ATOL_NS, RTOL_NS, "noalloc vs workspace split-K")
        assert_close(got, ref, ATOL_NS, RTOL_NS, "noalloc vs CPU oracle")
    assert gpu.get_status(clear=True) == 0


def test_noalloc_after_a_call_that_filled_the_scratch(gpu):
    """The array keeps whatever the previous call left in it.  A call that uses
    nearly all of it (63 sequences x 8 heads x 64 partitions x 130 floats, the
    largest batch of this shape that fits, 4 KiB short of 16 MiB) is followed by
    smaller calls with other head counts, lengths (one of them 0) and partition
    counts: each must match the workspace entry point and the CPU oracle, so no
    partial of the earlier call is read."""
    torch = pytest.importorskip("torch")
    B, Hq, D, bs, psize = 63, 8, 128, 16, 512
    max_seq_len = 64 * psize
    assert need_bytes(B, Hq, max_seq_len, psize, D) <= SCRATCH_BYTES < need_bytes(B, Hq, max_seq_len + 1, psize, D)
    rng = np.random.default_rng(11)
    lens = rng.integers(max_seq_len - 600, max_seq_len + 1, size=B).astype(np.int32)
    nblk = max_seq_len // bs
    tables = np.ascontiguousarray(rng.permutation(B * nblk).reshape(B, nblk).astype(np.int32))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    big = {"k_cache": torch.randn((B * nblk, 1, D // 8, bs, 8), generator=g, device=dev, dtype=torch.bfloat16),
           "v_cache": torch.randn((B * nblk, 1, D, bs), generator=g, device=dev, dtype=torch.bfloat16),
           "q": torch.randn((B, Hq, D), generator=g, device=dev, dtype=torch.bfloat16),
           "block_tables": DeviceArray.from_numpy(tables), "context_lens": DeviceArray.from_numpy(lens)}
    cb = {"num_kv_heads": 1, "scale": 1.0 / math.sqrt(D), "block_size": bs, "max_seq_len": max_seq_len}
    got = noalloc(big, cb, psize, DeviceArray.empty((B, Hq, D), "bfloat16")).to_numpy()
    want = mk.paged_attention_v2(big["q"], big["k_cache"], big["v_cache"], big["block_tables"], big["context_lens"],
                                 1, cb["scale"], bs, max_seq_len, partition_size=psize).to_numpy()
    assert_close(got, want, ATOL_NS, RTOL_NS, "scratch-filling call")
    del big
    for dtype, Hq2, Hkv2, D2, bs2, lens2, p2 in (("float16", 4, 2, 64, 16, [0, 1, 700, 33, 1500], 256),
                                                  ("bfloat16", 16, 2, 128, 32, [5, 2000, 64], 512)):
        c = cases.paged_batch(4300 + Hq2, dtype, len(lens2), Hq2, Hkv2, D2, bs2, lens2)
        d = upload_case(c)
        fill_cache(d)
        kc, vc = oracle_fill(c, dtype)
        ref = kv_oracle.paged_attention_v1(c["q"], kc, vc, c["block_tables"], c["context_lens"], Hkv2, c["scale"],
                                           bs2, c["max_seq_len"])
        want = mk.paged_attention_v2(d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"], Hkv2,
                                     c["scale"], bs2, c["max_seq_len"], partition_size=p2).to_numpy()
        for _ in range(2):
            got = noalloc(d, c, p2, DeviceArray.empty(d["q"].shape, dtype)).to_numpy()
            assert_close(got, want, ATOL_NS, RTOL_NS, "after a larger call: vs workspace split-K")
            assert_close(got, ref, ATOL_NS, RTOL_NS, "after a larger call: vs CPU oracle")
        if 0 in lens2:
            assert not got[lens2.index(0)].any()
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
    # one partition more than the largest batch that fits (see the test above) is refused too
    assert need_bytes(63, 8, 65 * 512, 512, 128) > SCRATCH_BYTES
    rc = _lib.lib.kvc_paged_attention_v2_noalloc(
        t((63, 8, 128), "bfloat16"), t((63, 8, 128), "bfloat16"), t((100, 1, 16, 16, 8), "bfloat16"),
        t((100, 1, 128, 16), "bfloat16"), t((63, 65 * 32), "int32"), t((63,), "int32"), 1, 0.1, 16, 65 * 512, None,
        512, None)
    assert rc == _lib.KVC_EINVAL
    assert "static scratch" in _lib.last_error()


FIRST_CALL_IN_CAPTURE = r"""
import ctypes, sys
sys.path[:0] = {paths!r}
import numpy as np
import cases
from helpers import upload_case, fill_cache
from sglang_mlx_b200 import _lib
from sglang_mlx_b200.device_array import DeviceArray, Stream
from sglang_mlx_b200.dlpack import as_dltensor
c = cases.paged_batch(5, "bfloat16", 2, 8, 2, 64, 16, [100, 300])
d = upload_case(c)
fill_cache(d)
_lib.synchronize()
out = DeviceArray.empty((2, 8, 64), "bfloat16")
st = Stream()
ptrs = [as_dltensor(x) for x in (out, d["q"], d["k_cache"], d["v_cache"], d["block_tables"], d["context_lens"])]
def call():
    return _lib.lib.kvc_paged_attention_v2_noalloc(ptrs[0][0], ptrs[1][0], ptrs[2][0], ptrs[3][0], ptrs[4][0],
        ptrs[5][0], 2, c["scale"], 16, c["max_seq_len"], None, 256, ctypes.c_void_p(st.handle))
_lib.check(_lib.lib.kvc_stream_begin_capture(ctypes.c_void_p(st.handle)))
rc = call()
msg = _lib.last_error()
h = ctypes.c_void_p()
_lib.check(_lib.lib.kvc_stream_end_capture(ctypes.c_void_p(st.handle), ctypes.byref(h)))
_lib.lib.kvc_graph_destroy(h)
assert rc == _lib.KVC_EINVAL and "outside stream capture" in msg, (rc, msg)
_lib.check(call())   # eagerly it runs
st.synchronize()
print("ok")
"""


def test_noalloc_first_call_inside_a_capture_is_refused(gpu):
    """The first call on a device looks the scratch address up, which must not
    happen inside a stream capture: in a fresh process such a call returns
    KVC_EINVAL with a message, launches nothing, and the capture still ends
    cleanly; the same call made eagerly then runs."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    paths = [here, os.path.join(here, "golden"), root, os.path.join(root, "sglang-mlx_b200")]
    r = subprocess.run([sys.executable, "-c", FIRST_CALL_IN_CAPTURE.format(paths=paths)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
