"""Arithmetic identities the GEMV decode relies on, checked on the CPU from the
constants in the kernel headers (no GPU needed).

* IQ4_XS: the byte-permute P + Q decode (qb_iq4.cuh `iq4_pq`) reproduces the
  16-entry int8 value table (`kIq4I8T0..T3`) for every code.  A permute
  selector nibble with bit 3 set yields the selected byte's sign replicated;
  P looks up with the code, Q with code ^ 8.
* Q6_K: a scale byte stored as sc + 128 becomes the float 2^23 + sc + 128 by
  placing it under the exponent byte 0x4B, and subtracting 2^23 + 128 gives sc
  exactly (qb_quant.cu `stage_q6k`).
* Activations: X = 65536 d0 + 256 d1 + d2 with balanced int8 digits for every
  |X| <= 2^22, |d0| <= 64 (qb_xprep.cuh).
* The IQ4_XS int32 sums, scaled by summation by parts, cannot overflow.
"""
import os
import re

import numpy as np

from conftest import ROOT

CSRC = os.path.join(ROOT, "qwen3.8-27b-in-c_b200", "csrc")


def _const(name, text):
    m = re.search(r"constexpr uint32_t %s = (0x[0-9A-Fa-f]+)u;" % name, text)
    assert m, name
    return int(m.group(1), 16)


def _prmt(a, b, sel):
    """PTX prmt.b32 default mode: byte j of the result is byte (sel nibble j & 7)
    of {b, a}, or that byte's sign replicated when the nibble's bit 3 is set."""
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for j in range(4):
        s = (sel >> (4 * j)) & 0xF
        v = src[s & 7]
        if s & 8:
            v = 0xFF if v & 0x80 else 0x00
        out |= v << (8 * j)
    return out


def _s8(x):
    return x - 256 if x >= 128 else x


def test_iq4_pq_decode_reproduces_the_table():
    text = open(os.path.join(CSRC, "qb_iq4.cuh")).read()
    t = [_const("kIq4I8T%d" % i, text) for i in range(4)]
    q2, q3 = _const("kIq4QT2", text), _const("kIq4QT3", text)
    table = [_s8((t[i // 4] >> (8 * (i % 4))) & 0xFF) for i in range(16)]
    rng = np.random.default_rng(0)
    words = [int(w) for w in rng.integers(0, 2 ** 32, 2000, dtype=np.uint64)] + [0, 0xFFFFFFFF, 0x76543210, 0xFEDCBA98]
    for w in words:
        x = w ^ 0x88888888
        p_lo, p_hi = _prmt(t[0], t[1], w & 0xFFFF), _prmt(t[0], t[1], w >> 16)
        q_lo, q_hi = _prmt(q2, q3, x & 0xFFFF), _prmt(q2, q3, x >> 16)
        for j in range(4):
            for p, q, shift in ((p_lo, q_lo, 0), (p_hi, q_hi, 16)):
                code = (w >> (shift + 4 * j)) & 0xF
                got = _s8((p >> (8 * j)) & 0xFF) + _s8((q >> (8 * j)) & 0xFF)
                assert got == table[code], (hex(w), j, shift, code, got, table[code])


def test_q6k_scale_byte_to_float_is_exact():
    for sc in range(-128, 128):
        u = (sc + 128) & 0xFF                     # stored byte
        bits = _prmt(u, 0x4B000000, 0x7650)       # byte 0 from the word, bytes 1..3 from the constant
        f = np.frombuffer(np.uint32(bits).tobytes(), np.float32)[0]
        assert np.float32(f) - np.float32(8388736.0) == np.float32(sc)


def test_balanced_digits_reconstruct_the_integer():
    rng = np.random.default_rng(1)
    xs = list(rng.integers(-(2 ** 22), 2 ** 22 + 1, 20000)) + [0, 1, -1, 2 ** 22, -(2 ** 22), 127, 128, -128, -129]
    for X in map(int, xs):
        d2 = _s8(X & 0xFF)
        X1 = (X - d2) >> 8
        d1 = _s8(X1 & 0xFF)
        d0 = (X1 - d1) >> 8
        assert 65536 * d0 + 256 * d1 + d2 == X
        assert -128 <= d1 <= 127 and -128 <= d2 <= 127 and abs(d0) <= 64


def test_iq4_int32_accumulators_cannot_overflow():
    """Worst case of the IQ4_XS int8 path's int32 sums (qb_quant.cu stage_iq4_i8):
    per 32-column sub-block and digit column C_j = sum of 32 products of a table
    value (or a P / Q term) and a digit (|d0| <= 64, |d1|, |d2| <= 128); the mma
    chain holds R_j = C_0 + .. + C_j (and, between the P and Q steps, R_{j-1}
    plus the P products); the scales apply by summation by parts,
    sum_j s_j C_j = sum_{j<7} (s_j - s_{j+1}) R_j + s_7 R_7, s_j = ls_j - 32 in
    [-32, 31].  Every partial value must fit in int32."""
    text = open(os.path.join(CSRC, "qb_iq4.cuh")).read()
    t = [_const("kIq4I8T%d" % i, text) for i in range(4)]
    q2, q3 = _const("kIq4QT2", text), _const("kIq4QT3", text)
    vals = [_s8((w >> (8 * i)) & 0xFF) for w in t for i in range(4)]
    pq = [_s8((w >> (8 * i)) & 0xFF) for w in t[:2] for i in range(4)] + [-1] + \
         [_s8((w >> (8 * i)) & 0xFF) for w in (q2, q3) for i in range(4)]
    wmax = max(max(abs(v) for v in vals), max(abs(v) for v in pq))
    dmax = 128
    c_max = 32 * wmax * dmax                 # one sub-block, one digit column
    r_max = [(j + 1) * c_max for j in range(8)]
    p_mid = [r_max[j - 1] + c_max if j else c_max for j in range(8)]   # after the P step of sub-block j
    delta_max, s_max = 63, 32
    acc_max = sum(delta_max * r_max[j] for j in range(7)) + s_max * r_max[7]
    assert max(r_max + p_mid) < 2 ** 31
    assert acc_max < 2 ** 31, acc_max
