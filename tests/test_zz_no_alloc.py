"""The allocation-free paged-attention entry (ti_op_paged_attention_noalloc).

Some callers of this library cannot allocate device memory at the point where
they run attention: a plugin inside a host application that owns the whole
device-memory budget and forbids allocation during its execute call, or a
process whose memory another framework's caching allocator has reserved up
front.  For them the entry takes its scratch from a fixed array that the
library owns instead of the stream-ordered memory pool.

This test calls it through the C ABI twice in a row on different inputs (the
shared scratch keeps the previous call's contents) and checks each result, and
the K/V rows it appends to the pages, against the CPU oracle's RoPE + attention
(restating ops.cu:210-312 and ops.cu:444-544) and against the pool-backed
ti_op_paged_attention on the same inputs, within the tolerance of the other
attention parity tests.  The file is collected last so that a run stopping at
the first failure has run every other test.
"""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import DevBuf, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2  # the attention tolerance of tests/test_gpu_ops.py
f32 = oracle.bf16_to_f32


def _case(seed, B, nq, nkv, hd, max_len, theta=500000.0):
    """random paged K/V state (shuffled page ids, `pos[b]` cached tokens) and the
    oracle's output and rotated K row for one decode-attention call"""
    rng = np.random.default_rng(seed)
    pt_stride = (max_len + 15) // 16
    n_pages = B * pt_stride + 5
    table = rng.permutation(n_pages)[: B * pt_stride].reshape(B, pt_stride).astype(np.int32)
    pos = rng.integers(1, max_len - 1, size=B).astype(np.int32)
    kpool = oracle.f32_to_bf16(rng.standard_normal((n_pages, nkv, 16, hd)).astype(np.float32))
    vpool = oracle.f32_to_bf16(rng.standard_normal((n_pages, nkv, 16, hd)).astype(np.float32))
    qkv = oracle.f32_to_bf16(rng.standard_normal((B, (nq + 2 * nkv) * hd)).astype(np.float32))
    fr = np.empty(hd // 2, np.float32)
    oracle.lib().orc_rope_freqs(hd, theta, None, oracle.ptr(fr))
    ref, knew = [], []
    for b in range(B):
        p = int(pos[b])
        pages = table[b, : (p + 15) // 16]
        kc = kpool[pages].transpose(0, 2, 1, 3).reshape(-1, nkv, hd)[:p]
        vc = vpool[pages].transpose(0, 2, 1, 3).reshape(-1, nkv, hd)[:p]
        q = np.ascontiguousarray(qkv[b, : nq * hd].reshape(1, nq, hd))
        k = np.ascontiguousarray(qkv[b, nq * hd:(nq + nkv) * hd].reshape(1, nkv, hd))
        v = np.ascontiguousarray(qkv[b, (nq + nkv) * hd:].reshape(1, nkv, hd))
        qr, kr = np.empty_like(q), np.empty_like(k)
        oracle.lib().orc_rope(oracle.ptr(q), oracle.ptr(qr), 1, nq, hd, p, oracle.ptr(fr))
        oracle.lib().orc_rope(oracle.ptr(k), oracle.ptr(kr), 1, nkv, hd, p, oracle.ptr(fr))
        K = np.ascontiguousarray(np.concatenate([kc, kr]))
        V = np.ascontiguousarray(np.concatenate([vc, v]))
        o = np.empty((1, nq, hd), np.uint16)
        oracle.lib().orc_attention(oracle.ptr(qr), oracle.ptr(K), oracle.ptr(V), oracle.ptr(o), 1, nq, p + 1, nkv,
                                   hd, 0, -1)
        ref.append(o.reshape(-1))
        knew.append(kr.reshape(nkv, hd))
    return dict(qkv=qkv, table=table, pos=pos, seq=np.arange(B, dtype=np.int32), kpool=kpool, vpool=vpool,
                ref=np.stack(ref), knew=knew, B=B, nq=nq, nkv=nkv, hd=hd, pt_stride=pt_stride, n_pages=n_pages,
                max_len=max_len, theta=theta)


def _call(fn, c):
    bufs = {k: DevBuf.from_array(c[k]) for k in ("qkv", "table", "kpool", "vpool", "pos", "seq")}
    out = DevBuf(c["B"] * c["nq"] * c["hd"] * 2)
    ti.check(getattr(ti.lib(), fn)(bufs["qkv"].ptr, c["B"], c["nq"], c["nkv"], c["hd"], bufs["pos"].ptr,
                                   bufs["seq"].ptr, bufs["table"].ptr, c["pt_stride"], bufs["kpool"].ptr,
                                   bufs["vpool"].ptr, c["n_pages"], c["max_len"], c["theta"], None, -1, out.ptr,
                                   None))
    return (out.to_array((c["B"], c["nq"] * c["hd"]), np.uint16),
            bufs["kpool"].to_array(c["kpool"].shape, np.uint16), bufs["vpool"].to_array(c["vpool"].shape, np.uint16))


def test_noalloc_matches_oracle_and_pool_backed_entry_two_calls():
    # two calls in a row, different shapes and RoPE bases: the second must not
    # see the first's counters, partials or frequency table
    for seed, shape, theta in ((21, (4, 32, 8, 128, 700), 500000.0), (22, (3, 28, 4, 128, 300), 1e6)):
        c = _case(seed, *shape, theta=theta)
        out, k, v = _call("ti_op_paged_attention_noalloc", c)
        assert rel_err(f32(out), f32(c["ref"])) <= TOL
        nq, nkv, hd = c["nq"], c["nkv"], c["hd"]
        for b in range(c["B"]):
            p = int(c["pos"][b])
            page = c["table"][b, p // 16]
            assert rel_err(f32(k[page, :, p % 16]), f32(c["knew"][b])) <= TOL
            np.testing.assert_array_equal(v[page, :, p % 16], c["qkv"][b, (nq + nkv) * hd:].reshape(nkv, hd))
        pool_out, pool_k, pool_v = _call("ti_op_paged_attention", c)
        assert rel_err(f32(out), f32(pool_out)) <= TOL
        np.testing.assert_array_equal(k, pool_k)
        np.testing.assert_array_equal(v, pool_v)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    c = _case(23, 2, 32, 8, 128, 64)
    bufs = {k: DevBuf.from_array(c[k]) for k in ("qkv", "table", "kpool", "vpool", "pos", "seq")}
    out = DevBuf(2 * 32 * 128 * 2)
    # a batch this large needs more than the fixed scratch: refused before any launch
    st = ti.lib().ti_op_paged_attention_noalloc(bufs["qkv"].ptr, 4096, 32, 8, 128, bufs["pos"].ptr, bufs["seq"].ptr,
                                                bufs["table"].ptr, 1 << 12, bufs["kpool"].ptr, bufs["vpool"].ptr,
                                                c["n_pages"], 1 << 16, 500000.0, None, -1, out.ptr, None)
    assert st == ti.TI_ERR_INVALID
    assert "scratch" in ti.lib().ti_last_error().decode()
