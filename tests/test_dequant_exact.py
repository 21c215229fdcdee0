"""The tcgen05 GEMM's Q4_0 dequantisation in bf16x2 arithmetic, checked exhaustively on the CPU.

The dequantising warps of csrc/tc_gemm.cu never convert an element from fp32: per
32-element block the fp16 scale d is split into dh = bf16(d) and dl = d - dh, and per
pair of codes they form P = (128 + q_even, 128 + 8 q_odd) from the code bits, subtract
(136, 192) and evaluate fma(a, (dh, dh/8), a * (dl, dl/8)) in bf16x2.  That is the
oracle's fp32 weight d * (q - 8) (orc_q4_0_dequantize in oracle/oracle.cpp, the GGUF
Q4_0 formula) rounded once to bf16, the operand type of the bf16 MMA, only if every
intermediate is exact: dl and dl/8 representable in bf16, dh/8 = bf16(d/8), and a * dl
exact.  These tests check those facts for every finite fp16 scale and every code, and the
bit construction of P for sampled code words (every byte position), with numpy standing
in for the instructions' round-to-nearest-even.
"""
import numpy as np


def bf16_rne(x):
    """float32 array -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f64(b):
    return (np.asarray(b, np.uint32) << 16).astype(np.uint32).view(np.float32).astype(np.float64)


def all_finite_fp16():
    h = np.arange(1 << 16, dtype=np.uint16).view(np.float16)
    return h[np.isfinite(h)].astype(np.float64)


def test_scale_split_is_exact_for_every_fp16_scale():
    d = all_finite_fp16()
    dh = bf16_to_f64(bf16_rne(d.astype(np.float32)))
    # the high lane's dh/8 is bf16(d/8): scaling by a power of two commutes with rounding
    dh8 = bf16_to_f64(bf16_rne((d / 8).astype(np.float32)))
    assert np.array_equal(dh8, dh / 8)
    dl = d - dh  # exact in float64
    # dl and dl/8 are bf16 values (at most 3 significant bits)
    assert np.array_equal(bf16_to_f64(bf16_rne(dl.astype(np.float32))), dl)
    assert np.array_equal(bf16_to_f64(bf16_rne((dl / 8).astype(np.float32))), dl / 8)


def test_fused_form_equals_rounded_product_for_every_code():
    d = all_finite_fp16()
    dh = bf16_to_f64(bf16_rne(d.astype(np.float32)))
    dl = d - dh
    for q in range(16):
        a = float(q - 8)
        # a * dl is exact in bf16 (the bf16x2 multiply rounds nothing)
        c = a * dl
        assert np.array_equal(bf16_to_f64(bf16_rne(c.astype(np.float32))), c)
        # the high lane: (8a) * (dl/8) is the same value
        assert np.array_equal((8 * a) * (dl / 8), c)
        # fma rounds a*dh + c once; a*dh + c == a*d exactly, and a*d is exact in fp32
        exact = a * dh + c
        assert np.array_equal(exact, a * d)
        got = bf16_rne(exact.astype(np.float32))
        want = bf16_rne((np.float32(a) * d.astype(np.float32)))  # the oracle: fp32 product, one rounding
        # signed zeros aside (q = 8), the bit patterns agree
        nz = exact != 0
        assert np.array_equal(got[nz], want[nz])


def byte_perm(x, y, s):
    """CUDA __byte_perm: result byte i = byte (s >> 4i) & 7 of the 8-byte value y:x."""
    src = (np.uint64(y) << np.uint64(32)) | np.uint64(x)
    out = 0
    for i in range(4):
        sel = (s >> (4 * i)) & 7
        out |= ((int(src) >> (8 * sel)) & 0xFF) << (8 * i)
    return out


def test_pair_bits_for_every_code_byte():
    # P for pair e of a code word: byte e of w (low nibble = even element) and byte e of
    # w >> 1 (its bits 3..6 = the high nibble), masked and under the bf16 exponent of 128
    rng = np.random.default_rng(0)
    for _ in range(64):
        w = int(rng.integers(0, 1 << 32))
        for e in range(4):
            t = byte_perm(w, w >> 1, e | ((e + 4) << 8))
            P = (t & 0x0078000F) | 0x43004300
            lo, hi = P & 0xFFFF, P >> 16
            b = (w >> (8 * e)) & 0xFF
            assert bf16_to_f64(np.uint16(lo)) == 128 + (b & 15)
            assert bf16_to_f64(np.uint16(hi)) == 128 + 8 * (b >> 4)
            # minus (136, 192): (q_even - 8, 8 (q_odd - 8)), exact small integers
            assert bf16_to_f64(np.uint16(lo)) - 136 == (b & 15) - 8
            assert bf16_to_f64(np.uint16(hi)) - 192 == 8 * ((b >> 4) - 8)
    # the constant (136, 192)
    assert bf16_to_f64(np.uint16(0x4308)) == 136 and bf16_to_f64(np.uint16(0x4340)) == 192
