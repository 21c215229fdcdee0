"""Parity of every ti_op_* kernel (the tensor::backend::ops replacements) with
the oracle's restatement of the same reference op, on seeded inputs."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import DevBuf, rel_err

pytestmark = pytest.mark.gpu
L = None


def lib():
    return ti.lib()


def bf(shape, name, seed=0, std=1.0):
    return oracle.fill_bf16(name, shape, seed, std)


def f32(a):
    return oracle.bf16_to_f32(a)


@pytest.mark.parametrize("M,N,K", [(1, 1000, 256), (3, 4096, 4096), (8, 512, 1024), (37, 300, 200), (128, 256, 512)])
def test_matmul_t_bf16(M, N, K):
    a, b = bf((M, K), "a", M), bf((N, K), "b", N, 0.05)
    ref = np.empty((M, N), np.uint16)
    oracle.lib().orc_matmul_t_bf16(oracle.ptr(a), oracle.ptr(b), oracle.ptr(ref), M, N, K)
    da, db, dc = DevBuf.from_array(a), DevBuf.from_array(b), DevBuf(M * N * 2)
    ti.check(lib().ti_op_matmul_t(ti.DTYPE_BF16, da.ptr, db.ptr, dc.ptr, M, N, K, None))
    out = dc.to_array((M, N), np.uint16)
    assert rel_err(f32(out), f32(ref)) < 1e-2


def test_matmul_t_f32():
    M, N, K = 5, 70, 33
    a = oracle.fill_f32("a", (M, K), 1)
    b = oracle.fill_f32("b", (N, K), 2)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    da, db, dc = DevBuf.from_array(a), DevBuf.from_array(b), DevBuf(M * N * 4)
    ti.check(lib().ti_op_matmul_t(ti.DTYPE_F32, da.ptr, db.ptr, dc.ptr, M, N, K, None))
    assert rel_err(dc.to_array((M, N), np.float32), ref) < 1e-5


@pytest.mark.parametrize("offset", [0, 1])
def test_rms_norm(offset):
    rows, H = 3, 4096
    x, w = bf((rows, H), "x", 1), bf((H,), "w", 2, 0.1)
    ref = np.empty_like(x)
    oracle.lib().orc_rms_norm(oracle.ptr(x), oracle.ptr(w), oracle.ptr(ref), rows, H, 1e-5, offset)
    dx, dw, do = DevBuf.from_array(x), DevBuf.from_array(w), DevBuf(x.nbytes)
    ti.check(lib().ti_op_rms_norm(dx.ptr, dw.ptr, do.ptr, rows, H, 1e-5, offset, None))
    assert rel_err(f32(do.to_array(x.shape, np.uint16)), f32(ref)) < 1e-2


@pytest.mark.parametrize("scaling", [False, True])
def test_rope(scaling):
    seq, heads, hd, off = 5, 8, 128, 1000
    x = bf((seq, heads, hd), "x", 3)
    sc = ti.RopeScaling(1, 8.0, 1.0, 4.0, 8192) if scaling else None
    osc = oracle.RopeScaling(1, 8.0, 1.0, 4.0, 8192) if scaling else None
    fr = np.empty(hd // 2, np.float32)
    oracle.lib().orc_rope_freqs(hd, 500000.0, C.byref(osc) if osc else None, oracle.ptr(fr))
    ref = np.empty_like(x)
    oracle.lib().orc_rope(oracle.ptr(x), oracle.ptr(ref), seq, heads, hd, off, oracle.ptr(fr))
    dx, do = DevBuf.from_array(x), DevBuf(x.nbytes)
    ti.check(lib().ti_op_rope(dx.ptr, do.ptr, seq, heads, hd, off, 500000.0, C.byref(sc) if sc else None, None))
    assert rel_err(f32(do.to_array(x.shape, np.uint16)), f32(ref)) < 1e-2


@pytest.mark.parametrize("kind", [ti.EW_SILU, ti.EW_GELU, ti.EW_MUL, ti.EW_ADD, ti.EW_MUL_SCALAR])
def test_elementwise(kind):
    n = 10007
    a, b = bf((n,), "a", 4, 2.0), bf((n,), "b", 5, 2.0)
    ref = np.empty_like(a)
    O = oracle.lib()
    if kind == ti.EW_SILU:
        O.orc_silu(oracle.ptr(a), oracle.ptr(ref), n)
    elif kind == ti.EW_GELU:
        O.orc_gelu(oracle.ptr(a), oracle.ptr(ref), n)
    elif kind == ti.EW_MUL:
        O.orc_mul(oracle.ptr(a), oracle.ptr(b), oracle.ptr(ref), n)
    elif kind == ti.EW_ADD:
        O.orc_add(oracle.ptr(a), oracle.ptr(b), oracle.ptr(ref), n)
    else:
        O.orc_mul_scalar(oracle.ptr(a), 64.0, oracle.ptr(ref), n)
    da, db, do = DevBuf.from_array(a), DevBuf.from_array(b), DevBuf(a.nbytes)
    ti.check(lib().ti_op_elementwise(kind, da.ptr, db.ptr, 64.0, do.ptr, n, None))
    out = do.to_array(a.shape, np.uint16)
    # transcendental ops may differ by one bf16 ulp; arithmetic ones are exact
    if kind in (ti.EW_MUL, ti.EW_ADD, ti.EW_MUL_SCALAR):
        np.testing.assert_array_equal(out, ref)
    else:
        assert rel_err(f32(out), f32(ref)) < 1e-2


def test_add_bias():
    x, bias = bf((4, 1152), "x", 6), bf((1152,), "b", 7)
    ref = np.empty_like(x)
    oracle.lib().orc_add_bias(oracle.ptr(x), oracle.ptr(bias), oracle.ptr(ref), 4, 1152)
    dx, db, do = DevBuf.from_array(x), DevBuf.from_array(bias), DevBuf(x.nbytes)
    ti.check(lib().ti_op_add_bias(dx.ptr, db.ptr, do.ptr, 4, 1152, None))
    np.testing.assert_array_equal(do.to_array(x.shape, np.uint16), ref)


def test_softmax():
    x = oracle.fill_f32("x", (6, 3000), 8, 3.0)
    ref = x.copy()
    oracle.lib().orc_softmax_f32(oracle.ptr(ref), 6, 3000)
    dx, do = DevBuf.from_array(x), DevBuf(x.nbytes)
    ti.check(lib().ti_op_softmax(ti.DTYPE_F32, dx.ptr, do.ptr, 6, 3000, None))
    assert rel_err(do.to_array(x.shape, np.float32), ref) < 1e-5


@pytest.mark.parametrize("seq,kv_len,causal,window", [(1, 300, 0, -1), (7, 7, 1, -1), (9, 25, 1, -1), (12, 12, 1, 4)])
def test_attention(seq, kv_len, causal, window):
    nq, nkv, hd = 8, 2, 128
    q, k, v = bf((seq, nq, hd), "q", 9), bf((kv_len, nkv, hd), "k", 9), bf((kv_len, nkv, hd), "v", 9)
    ref = np.empty_like(q)
    oracle.lib().orc_attention(oracle.ptr(q), oracle.ptr(k), oracle.ptr(v), oracle.ptr(ref), seq, nq, kv_len, nkv, hd,
                               causal, window)
    dq, dk, dv, do = DevBuf.from_array(q), DevBuf.from_array(k), DevBuf.from_array(v), DevBuf(q.nbytes)
    ti.check(lib().ti_op_attention(dq.ptr, dk.ptr, dv.ptr, do.ptr, seq, nq, kv_len, nkv, hd, causal, window, None))
    assert rel_err(f32(do.to_array(q.shape, np.uint16)), f32(ref)) < 1e-2


def test_embedding_and_bad_id():
    w = bf((100, 64), "w", 10)
    ids = np.array([3, 99, 0, 3], np.int32)
    dw, do = DevBuf.from_array(w), DevBuf(4 * 64 * 2)
    ti.check(lib().ti_op_embedding(dw.ptr, 100, 64, ids.ctypes.data_as(C.c_void_p), 4, do.ptr, None))
    np.testing.assert_array_equal(do.to_array((4, 64), np.uint16), w[ids])
    bad = np.array([100], np.int32)
    assert lib().ti_op_embedding(dw.ptr, 100, 64, bad.ctypes.data_as(C.c_void_p), 1, do.ptr, None) == ti.TI_ERR_INVALID


def test_cast_and_transpose():
    x = oracle.fill_f32("x", (33, 65), 11)
    dx, db, dt = DevBuf.from_array(x), DevBuf(x.size * 2), DevBuf(x.nbytes)
    ti.check(lib().ti_op_cast(ti.DTYPE_F32, ti.DTYPE_BF16, dx.ptr, db.ptr, x.size, None))
    np.testing.assert_array_equal(db.to_array(x.shape, np.uint16), oracle.f32_to_bf16(x))
    ti.check(lib().ti_op_transpose2d(ti.DTYPE_F32, dx.ptr, dt.ptr, 33, 65, None))
    np.testing.assert_array_equal(dt.to_array((65, 33), np.float32), x.T)


def paged_case(seed=12, B=3, nq=8, nkv=2, hd=128, pos=(0, 17, 40), max_len=64, theta=10000.0, window=-1):
    """random paged K/V state (shuffled page ids) plus the oracle's expected output
    for one decode-attention call (with `window` > 0: over the last `window` tokens)"""
    rng = np.random.default_rng(seed)
    pt_stride = (max_len + 15) // 16
    n_pages = B * pt_stride + 3
    table = rng.permutation(n_pages)[: B * pt_stride].reshape(B, pt_stride).astype(np.int32)
    kpool = np.zeros((n_pages, nkv, 16, hd), np.uint16)
    vpool = np.zeros_like(kpool)
    cached = []
    for b in range(B):
        kc = oracle.f32_to_bf16(rng.standard_normal((pos[b], nkv, hd)).astype(np.float32))
        vc = oracle.f32_to_bf16(rng.standard_normal((pos[b], nkv, hd)).astype(np.float32))
        for j in range(pos[b]):
            kpool[table[b, j // 16], :, j % 16] = kc[j]
            vpool[table[b, j // 16], :, j % 16] = vc[j]
        cached.append((kc, vc))
    qkv = oracle.f32_to_bf16(rng.standard_normal((B, (nq + 2 * nkv) * hd)).astype(np.float32))
    fr = np.empty(hd // 2, np.float32)
    oracle.lib().orc_rope_freqs(hd, theta, None, oracle.ptr(fr))
    ref, knew = [], []
    for b in range(B):
        q = np.ascontiguousarray(qkv[b, : nq * hd].reshape(1, nq, hd))
        k = np.ascontiguousarray(qkv[b, nq * hd:(nq + nkv) * hd].reshape(1, nkv, hd))
        v = np.ascontiguousarray(qkv[b, (nq + nkv) * hd:].reshape(1, nkv, hd))
        qr, kr = np.empty_like(q), np.empty_like(k)
        oracle.lib().orc_rope(oracle.ptr(q), oracle.ptr(qr), 1, nq, hd, pos[b], oracle.ptr(fr))
        oracle.lib().orc_rope(oracle.ptr(k), oracle.ptr(kr), 1, nkv, hd, pos[b], oracle.ptr(fr))
        lo = max(0, pos[b] - window + 1) if window > 0 else 0
        K = np.ascontiguousarray(np.concatenate([cached[b][0], kr])[lo:])
        V = np.ascontiguousarray(np.concatenate([cached[b][1], v])[lo:])
        o = np.empty((1, nq, hd), np.uint16)
        oracle.lib().orc_attention(oracle.ptr(qr), oracle.ptr(K), oracle.ptr(V), oracle.ptr(o), 1, nq, pos[b] + 1 - lo,
                                   nkv, hd, 0, -1)
        ref.append(o.reshape(-1))
        knew.append(kr.reshape(nkv, hd))
    return dict(qkv=qkv, table=table, kpool=kpool, vpool=vpool, pos=np.array(pos, np.int32),
                seq=np.arange(B, dtype=np.int32), ref=np.stack(ref), knew=knew, B=B, nq=nq, nkv=nkv, hd=hd,
                pt_stride=pt_stride, n_pages=n_pages, max_len=max_len, theta=theta, window=window)


def run_paged(c, fn="ti_op_paged_attention"):
    bufs = {k: DevBuf.from_array(c[k]) for k in ("qkv", "table", "kpool", "vpool", "pos", "seq")}
    out = DevBuf(c["B"] * c["nq"] * c["hd"] * 2)
    ti.check(getattr(lib(), fn)(bufs["qkv"].ptr, c["B"], c["nq"], c["nkv"], c["hd"], bufs["pos"].ptr,
                                bufs["seq"].ptr, bufs["table"].ptr, c["pt_stride"], bufs["kpool"].ptr,
                                bufs["vpool"].ptr, c["n_pages"], c["max_len"], c["theta"], None, c["window"], out.ptr,
                                None))
    return (out.to_array((c["B"], c["nq"] * c["hd"]), np.uint16),
            bufs["kpool"].to_array(c["kpool"].shape, np.uint16), bufs["vpool"].to_array(c["vpool"].shape, np.uint16))


def check_paged(c, out, kp, vp):
    nq, nkv, hd = c["nq"], c["nkv"], c["hd"]
    assert rel_err(f32(out), f32(c["ref"])) < 1e-2
    for b in range(c["B"]):
        p = int(c["pos"][b])
        page = c["table"][b, p // 16]
        assert rel_err(f32(kp[page, :, p % 16]), f32(c["knew"][b])) < 1e-2
        np.testing.assert_array_equal(vp[page, :, p % 16],
                                      c["qkv"][b, (nq + nkv) * hd:].reshape(nkv, hd))


@pytest.mark.parametrize("hd,nq,nkv,spp", [(128, 16, 2, None), (128, 16, 2, 3), (64, 8, 2, 2), (256, 8, 1, 4),
                                           (128, 4, 4, 16), (128, 8, 2, 1000), (64, 4, 1, 1000), (256, 16, 1, 1000)])
def test_paged_attention_long(hd, nq, nkv, spp, monkeypatch):
    """long contexts: many ring stages per split (TI_ATTN_SPP), several splits merged
    or (TI_ATTN_SPP beyond the context) one split per (token, kv head)"""
    if spp:
        monkeypatch.setenv("TI_ATTN_SPP", str(spp))
    c = paged_case(seed=5, B=2, nq=nq, nkv=nkv, hd=hd, pos=(1500, 777), max_len=2048)
    check_paged(c, *run_paged(c))


@pytest.mark.parametrize("window", [100, 16, 1])
def test_paged_attention_window(window, monkeypatch):
    monkeypatch.setenv("TI_ATTN_SPP", "2")
    c = paged_case(seed=7, B=3, nq=8, nkv=2, hd=128, pos=(300, 50, 129), max_len=512, window=window)
    check_paged(c, *run_paged(c))


@pytest.mark.parametrize("hd,nq,nkv", [(128, 8, 2), (64, 4, 4), (128, 28, 4), (256, 8, 1), (128, 16, 1), (64, 8, 1),
                                       (256, 2, 1)])
def test_paged_attention_op(hd, nq, nkv):
    c = paged_case(hd=hd, nq=nq, nkv=nkv)
    out, kp, vp = run_paged(c)
    assert rel_err(f32(out), f32(c["ref"])) < 1e-2
    for b in range(c["B"]):
        p = int(c["pos"][b])
        page = c["table"][b, p // 16]
        assert rel_err(f32(kp[page, :, p % 16]), f32(c["knew"][b])) < 1e-2
        np.testing.assert_array_equal(vp[page, :, p % 16],
                                      c["qkv"][b, (nq + nkv) * hd:].reshape(nkv, hd))


def test_init_shutdown_and_ops_after_it():
    # every device is an sm_100 part; shutdown frees the cached RoPE tables and
    # the pools' unused blocks, and the ops rebuild what they need afterwards
    n = C.c_int(0)
    ti.check(lib().ti_init(C.byref(n)))
    assert n.value >= 1
    seq, heads, hd = 5, 4, 64
    x = bf((seq, heads, hd), "rope-sd", 3, 1.0)
    dx, do = DevBuf.from_array(x), DevBuf(x.nbytes)
    ti.check(lib().ti_op_rope(dx.ptr, do.ptr, seq, heads, hd, 7, 500000.0, None, None))
    before = do.to_array(x.shape, np.uint16)
    ti.check(lib().ti_shutdown())
    ti.check(lib().ti_op_rope(dx.ptr, do.ptr, seq, heads, hd, 7, 500000.0, None, None))
    np.testing.assert_array_equal(do.to_array(x.shape, np.uint16), before)


def test_bounded_waits_give_up_and_report():
    # a flag nothing writes and an mbarrier nothing completes, 20 ms each: both
    # waits end, set their error bits, and the context stays usable
    waited = (C.c_double * 2)()
    ti.check(lib().ti_selftest_waits(0, 20000, waited))
    for w in waited:
        assert 20000.0 <= w < 2e6, list(waited)
    x = bf((3, 4, 64), "after-wait", 5, 1.0)
    dx, do = DevBuf.from_array(x), DevBuf(x.nbytes)
    ti.check(lib().ti_op_rope(dx.ptr, do.ptr, 3, 4, 64, 0, 10000.0, None, None))
