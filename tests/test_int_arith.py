"""The integer identities of the CUDA-core q4 dot products, checked exactly in
numpy on the CPU (no GPU; a model of the kernels' byte arithmetic, not the
kernels themselves, whose outputs the GPU parity tests compare with the
restatement).

A q4 word holds 8 nibbles e_0..e_7, low nibble first in each byte. Its even
nibbles are the bytes of w & 0x0F0F0F0F, its odd nibbles times 16 the bytes of
w & 0xF0F0F0F0. The activation is a block fixed-point integer split into byte
planes: a signed high byte and unsigned lower bytes, each plane's word holding
the even elements' bytes and the odd elements' bytes apart.

- dot_group_x16 (qmoe_prefill.cu): 16-bit x, one 64-element group (8 words):
  hi = he + (ho >> 4), lo = le + (lo16 >> 4), sum = hi * 256 + lo, where ho and
  lo16 are the dp4a sums of the odd nibbles used in place (unsigned x signed
  for the high plane).
- dot_unit_h24 (qmoe_prefill.cu): 24-bit h, one 32-element unit (4 words):
  the same with a middle plane, sum = hi * 65536 + mid * 256 + low.
Both must equal sum_k e_k * v_k exactly."""
import numpy as np

RNG = np.random.default_rng(20261202)


def _bytes(words):
    """uint32 words -> [..., 4] bytes (little-endian)."""
    w = np.asarray(words, dtype=np.uint64)
    return np.stack([(w >> (8 * i)) & 0xFF for i in range(4)], axis=-1).astype(np.int64)


def _dp4a(a_bytes, b_bytes, signed_b):
    b = b_bytes.copy()
    if signed_b:
        b = np.where(b >= 128, b - 256, b)
    return (a_bytes * b).sum(axis=-1)


def _pack_q4(e):
    """[..., 8] nibbles -> uint32 word, low nibble first."""
    w = np.zeros(e.shape[:-1], dtype=np.uint64)
    for b in range(4):
        byte = (e[..., 2 * b] | (e[..., 2 * b + 1] << 4)).astype(np.uint64)
        w |= byte << np.uint64(8 * b)
    return w


def _planes(v, nb):
    """[..., 8] signed integers of 8*nb bits -> nb planes of (even, odd) words;
    plane 0 is the signed high byte, the others unsigned."""
    out = []
    for p in range(nb):
        sh = 8 * (nb - 1 - p)
        byte = (v >> sh) & 0xFF  # two's complement byte (numpy >> is arithmetic)
        ev = np.zeros(v.shape[:-1], dtype=np.uint64)
        od = np.zeros(v.shape[:-1], dtype=np.uint64)
        for j in range(4):
            ev |= byte[..., 2 * j].astype(np.uint64) << np.uint64(8 * j)
            od |= byte[..., 2 * j + 1].astype(np.uint64) << np.uint64(8 * j)
        out.append((ev, od))
    return out


def _kernel_sum(e, v, nb):
    """The kernels' sum for words of nibbles e [..., W, 8] and activations v
    [..., W, 8] (nb byte planes), accumulated over the W words."""
    w = _pack_q4(e)
    evb = _bytes(w & np.uint64(0x0F0F0F0F))
    ohb = _bytes(w & np.uint64(0xF0F0F0F0))
    acc = []
    for p, (pe, po) in enumerate(_planes(v, nb)):
        a_e = _dp4a(evb, _bytes(pe), signed_b=(p == 0)).sum(axis=-1)
        a_o = _dp4a(ohb, _bytes(po), signed_b=(p == 0)).sum(axis=-1)
        assert np.all(a_o % 16 == 0)
        acc.append(a_e + (a_o >> 4))  # the shift back, exact
    if nb == 2:
        return acc[0] * 256 + acc[1]
    return acc[0] * 65536 + acc[1] * 256 + acc[2]


def _check(nb, words, n=2000):
    # quant_word's range: |x| below 2^15 (16-bit x), |h| below 2^22 (24-bit h)
    bits = 16 if nb == 2 else 23
    lo_v, hi_v = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    e = RNG.integers(0, 16, size=(n, words, 8))
    v = RNG.integers(lo_v, hi_v + 1, size=(n, words, 8))
    # extremes: every nibble 15 against the largest and the smallest values
    e[0] = 15
    v[0] = hi_v
    e[1] = 15
    v[1] = lo_v
    e[2] = 0
    v[3] = 0
    got = _kernel_sum(e, v, nb)
    want = (e * v).sum(axis=(-1, -2))
    np.testing.assert_array_equal(got, want)
    # the kernels' per-plane 32-bit accumulators hold their sums: at most
    # words * 4 * 240 * 255 (odd nibbles in place) for an unsigned plane,
    # words * 4 * 240 * 128 in magnitude for the signed one
    assert words * 4 * 240 * 255 < 2**32 and words * 4 * 240 * 128 < 2**31
    if nb == 2:  # dot_group_x16 forms the whole sum in int32
        assert np.abs(want).max() < 2**31
    else:  # dot_unit_h24 forms mid * 256 + low in uint32
        assert (words * 4 * 15 * 255 * 2) * 257 < 2**32


def test_dot_group_x16_identity():
    """16-bit x, a 64-element group (8 words): exact, and the whole sum within
    int32 (at most 64 * 15 * 2^15)."""
    _check(2, 8)


def test_dot_unit_h24_identity():
    """24-bit h (|h| below 2^22), a 32-element unit (4 words): exact. The kernel
    forms hi * 65536 + (mid * 256 + low) in fp32 (one rounding)."""
    _check(3, 4)


def test_group_sum_fits_fp32_conversion_bound():
    """dot_group_x16's sum is converted to fp32 once: at most 64 * 15 * 2^15
    in magnitude (x is quantised to at most 2^15), under 2^25, so the
    conversion rounds at most once by one part in 2^24."""
    assert 64 * 15 * 2**15 < 2**25
