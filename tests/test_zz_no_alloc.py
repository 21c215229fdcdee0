"""The allocation-free paged-attention entry (ti_op_paged_attention_noalloc).

It exists for callers that cannot allocate device memory where they run the op:
plugins whose host application owns the device-memory budget, or processes whose
memory another framework's allocator has reserved.  Its scratch is a fixed
library-owned device array instead of the memory pool.  This test calls it
through the C ABI, twice in a row on different inputs (the shared scratch keeps
the previous call's contents), and compares each result, and the K/V rows it
appends, with the pool-backed ti_op_paged_attention on the same inputs, within
the same tolerance as the other attention parity tests.  The file is collected
last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import DevBuf, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2  # as test_gpu_ops.py's attention tests


def _state(seed, B, nq, nkv, hd, max_len):
    rng = np.random.default_rng(seed)
    pt_stride = (max_len + 15) // 16
    n_pages = B * pt_stride + 5
    table = rng.permutation(n_pages)[: B * pt_stride].reshape(B, pt_stride).astype(np.int32)
    pos = rng.integers(0, max_len - 1, size=B).astype(np.int32)
    kpool = oracle.f32_to_bf16(rng.standard_normal((n_pages, nkv, 16, hd)).astype(np.float32))
    vpool = oracle.f32_to_bf16(rng.standard_normal((n_pages, nkv, 16, hd)).astype(np.float32))
    qkv = oracle.f32_to_bf16(rng.standard_normal((B, (nq + 2 * nkv) * hd)).astype(np.float32))
    return dict(qkv=qkv, table=table, pos=pos, seq=np.arange(B, dtype=np.int32), kpool=kpool, vpool=vpool,
                B=B, nq=nq, nkv=nkv, hd=hd, pt_stride=pt_stride, n_pages=n_pages, max_len=max_len)


def _call(fn, c, theta=500000.0):
    bufs = {k: DevBuf.from_array(c[k]) for k in ("qkv", "table", "kpool", "vpool", "pos", "seq")}
    out = DevBuf(c["B"] * c["nq"] * c["hd"] * 2)
    ti.check(getattr(ti.lib(), fn)(bufs["qkv"].ptr, c["B"], c["nq"], c["nkv"], c["hd"], bufs["pos"].ptr,
                                   bufs["seq"].ptr, bufs["table"].ptr, c["pt_stride"], bufs["kpool"].ptr,
                                   bufs["vpool"].ptr, c["n_pages"], c["max_len"], theta, None, -1, out.ptr, None))
    return (out.to_array((c["B"], c["nq"] * c["hd"]), np.uint16),
            bufs["kpool"].to_array(c["kpool"].shape, np.uint16), bufs["vpool"].to_array(c["vpool"].shape, np.uint16))


def test_noalloc_matches_pool_backed_entry_two_calls():
    f32 = oracle.bf16_to_f32
    # two calls in a row with different shapes: the second must not see the first's scratch
    for seed, shape in ((21, (4, 32, 8, 128, 700)), (22, (3, 28, 4, 128, 300))):
        c = _state(seed, *shape)
        ref_out, ref_k, ref_v = _call("ti_op_paged_attention", c)
        out, k, v = _call("ti_op_paged_attention_noalloc", c)
        assert rel_err(f32(out), f32(ref_out)) <= TOL
        assert rel_err(f32(k), f32(ref_k)) <= TOL and rel_err(f32(v), f32(ref_v)) <= TOL


def test_noalloc_rejects_sizes_beyond_its_scratch():
    c = _state(23, 2, 32, 8, 128, 64)
    bufs = {k: DevBuf.from_array(c[k]) for k in ("qkv", "table", "kpool", "vpool", "pos", "seq")}
    out = DevBuf(2 * 32 * 128 * 2)
    # a batch this large needs more than the fixed scratch: refused before any launch
    st = ti.lib().ti_op_paged_attention_noalloc(bufs["qkv"].ptr, 4096, 32, 8, 128, bufs["pos"].ptr, bufs["seq"].ptr,
                                                bufs["table"].ptr, 1 << 12, bufs["kpool"].ptr, bufs["vpool"].ptr,
                                                c["n_pages"], 1 << 16, 500000.0, None, -1, out.ptr, None)
    assert st == ti.TI_ERR_INVALID
    assert "scratch" in ti.lib().ti_last_error().decode()
