"""Index and arithmetic restatements of the kernels' shared-memory layouts and decode tricks (CPU).

The GPU parity suites check these paths end to end; this file restates their index math in
numpy so that a layout change that reorders a sum, or a bank-conflict regression, shows here:

* the superblock squares of csrc/qs_common.cuh (sb_put_sq32 / sb_sum256_partial32 for
  32-value groups, sb_put_sq16 / sb_sum256_partial16 for 16-value groups) read back, in
  torch's `.sum(-1)` order, exactly the elements of a row-major layout, and
  their writer and reader phases touch distinct banks;
* the word-wide level packing of csrc/qs_kquant.cu (Q2_K crumbs, Q4_K / Q5_K nibbles, Q5_K
  high bits) equals the byte-by-byte packing;
* the decode's byte-to-float (2^23 + byte minus 2^23 + bias) and 8-byte loads at any
  alignment (csrc/qs_dequant.cu byte_f, ld8) give the bytes' values.
"""

import numpy as np

RNG = np.random.default_rng(11)


# --- superblock squares ------------------------------------------------------------------
def partial_rowmajor(sq: np.ndarray, lane8: int) -> np.float32:
    """torch's order on row-major squares: acc_k = sum over i of sq[32 i + 8 k + lane8], then ((a0+a1)+a2)+a3."""
    acc = []
    for k in range(4):
        a = np.float32(0.0)
        for i in range(8):
            a = np.float32(a + sq[32 * i + 8 * k + lane8])
        acc.append(a)
    return np.float32(np.float32(np.float32(acc[0] + acc[1]) + acc[2]) + acc[3])


def put_sq32(x: np.ndarray) -> np.ndarray:
    """Row g (32 values), column c: chunk j = c & 7 at position (j + g) & 7, component c >> 3."""
    sq = np.full(256, np.nan, np.float32)
    for g in range(8):
        for j in range(8):
            for k in range(4):
                sq[32 * g + 4 * ((j + g) & 7) + k] = x[32 * g + j + 8 * k] ** 2
    return sq


def partial32(sq: np.ndarray, lane8: int) -> np.float32:
    a = [np.float32(0.0)] * 4
    for i in range(8):
        base = 32 * i + 4 * ((lane8 + i) & 7)
        a = [np.float32(a[k] + sq[base + k]) for k in range(4)]
    return np.float32(np.float32(np.float32(a[0] + a[1]) + a[2]) + a[3])


def put_sq16(x: np.ndarray) -> np.ndarray:
    """Row g (16 values), column c: pair p = c & 7 at position (p + g / 2) & 7, half c >> 3."""
    sq = np.full(256, np.nan, np.float32)
    for g in range(16):
        for p in range(8):
            for h in range(2):
                sq[16 * g + 2 * ((p + (g >> 1)) & 7) + h] = x[16 * g + p + 8 * h] ** 2
    return sq


def partial16(sq: np.ndarray, lane8: int) -> np.float32:
    a = [np.float32(0.0)] * 4
    for i in range(8):
        pos = 2 * ((lane8 + i) & 7)
        v = (sq[32 * i + pos], sq[32 * i + pos + 1])
        u = (sq[32 * i + 16 + pos], sq[32 * i + 16 + pos + 1])
        a = [np.float32(a[0] + v[0]), np.float32(a[1] + v[1]), np.float32(a[2] + u[0]), np.float32(a[3] + u[1])]
    return np.float32(np.float32(np.float32(a[0] + a[1]) + a[2]) + a[3])


def test_square_layouts_sum_like_the_row_major_order():
    for _ in range(50):
        x = (RNG.standard_normal(256) * RNG.choice([1e-3, 1.0, 1e3])).astype(np.float32)
        ref = (x * x).astype(np.float32)
        s32, s16 = put_sq32(x), put_sq16(x)
        assert not np.isnan(s32).any() and not np.isnan(s16).any()  # every slot written once
        for l in range(8):
            want = partial_rowmajor(ref, l)
            assert partial32(s32, l) == want
            assert partial16(s16, l) == want


def banks(word_addrs):
    return [a % 32 for a in word_addrs]


def test_square_layouts_are_bank_conflict_free():
    # 32-value groups: a quarter-warp of 16-byte accesses is the 8 groups of one superblock;
    # each access covers 4 banks starting at a multiple of 4
    for j in range(8):  # writer, chunk j of every row
        quads = [(32 * g + 4 * ((j + g) & 7)) // 4 % 8 for g in range(8)]
        assert len(set(quads)) == 8
    for i in range(8):  # reader, row i for every lane
        quads = [(32 * i + 4 * ((l + i) & 7)) // 4 % 8 for l in range(8)]
        assert len(set(quads)) == 8
    # 16-value groups: a half-warp of 8-byte accesses is the 16 groups of one superblock
    for p in range(8):
        pairs = [(16 * g + 2 * ((p + (g >> 1)) & 7)) // 2 % 16 for g in range(16)]
        assert len(set(pairs)) == 16
    for i in range(8):  # the 8 partial lanes of a superblock (the other half-warp lanes idle)
        for off in (0, 16):
            pairs = [(32 * i + off + 2 * ((l + i) & 7)) // 2 % 16 for l in range(8)]
            assert len(set(pairs)) == 8
    # the row-major store it replaced: one bank for all 32 lanes of a warp
    assert len(set(banks([256 * sb + 32 * g + 5 for sb in range(4) for g in range(8)]))) == 1


# --- word-wide level packing ---------------------------------------------------------------
def words(b: np.ndarray) -> np.ndarray:
    return b.view(np.uint32)


def test_word_packing_equals_byte_packing():
    lev2 = RNG.integers(0, 4, 256).astype(np.uint8)    # Q2_K levels
    lev4 = RNG.integers(0, 16, 256).astype(np.uint8)   # Q4_K levels
    lev5 = RNG.integers(0, 32, 256).astype(np.uint8)   # Q5_K levels
    # Q2_K: bytes 4g..4g+3 = levels l, l+32, l+64, l+96 of half h as 2-bit fields
    byte2 = np.array([lev2[128 * (i >> 5) + (i & 31)] | (lev2[128 * (i >> 5) + (i & 31) + 32] << 2)
                      | (lev2[128 * (i >> 5) + (i & 31) + 64] << 4) | (lev2[128 * (i >> 5) + (i & 31) + 96] << 6)
                      for i in range(64)], np.uint8)
    w2 = words(lev2)
    for g in range(16):
        h, l = g >> 3, (4 * g) & 31
        q = (128 * h + l) // 4
        assert w2[q] | (w2[q + 8] << 2) | (w2[q + 16] << 4) | (w2[q + 24] << 6) == words(byte2)[g]
    # Q4_K / Q5_K qs: byte 16g + i = low nibbles of levels 64j + l0 + i and 64j + 32 + l0 + i
    for lev in (lev4, lev5):
        for g in range(8):
            j, l0 = g >> 1, 16 * (g & 1)
            want = np.array([(lev[64 * j + l0 + i] & 0xF) | ((lev[64 * j + 32 + l0 + i] & 0xF) << 4) for i in range(16)],
                            np.uint8)
            a, b = words(lev[64 * j + l0:64 * j + l0 + 16].copy()), words(lev[64 * j + 32 + l0:64 * j + 48 + l0].copy())
            got = (a & 0x0F0F0F0F) | ((b & 0x0F0F0F0F) << 4)
            assert (got == words(want)).all()
    # Q5_K qh: bit s of byte l is bit 4 of level 32 s + l
    w5 = words(lev5)
    for g in range(8):
        v = np.uint32(0)
        for s in range(8):
            v |= ((w5[(32 * s + 4 * g) // 4] >> 4) & 0x01010101) << s
        want = np.array([sum(((lev5[32 * s + l] >> 4) & 1) << s for s in range(8)) for l in range(4 * g, 4 * g + 4)], np.uint8)
        assert v == words(want)[0]


# --- decode: byte_f and ld8 ----------------------------------------------------------------
def test_byte_to_float_is_exact():
    b = np.arange(256, dtype=np.uint32)
    for bias in (0, 4, 8, 32, 128):
        f = (0x4B000000 | b).view(np.float32)
        got = (f + np.float32(-(8388608.0 + bias))).astype(np.float32)
        assert (got == (b.astype(np.int64) - bias).astype(np.float32)).all()
    # Q8_0: int8 x + 128 is byte ^ 0x80
    x = np.arange(-128, 128, dtype=np.int64)
    assert ((((x & 0xFF) ^ 0x80)) == x + 128).all()


def ld8_shared(buf: bytes, off: int):
    """ld8 without BY: aligned 8-byte load, two aligned words, or three words and funnel shifts."""
    w = np.frombuffer(buf, np.uint32)
    if off % 8 == 0 or off % 4 == 0:
        return int(w[off // 4]), int(w[off // 4 + 1])
    base, sh = off // 4, (off % 4) * 8
    w0, w1, w2 = int(w[base]), int(w[base + 1]), int(w[base + 2])
    fs = lambda lo, hi: ((hi << 32 | lo) >> sh) & 0xFFFFFFFF  # __funnelshift_r(lo, hi, sh)
    return fs(w0, w1), fs(w1, w2)


def test_ld8_reads_the_eight_bytes_at_any_alignment():
    buf = RNG.integers(0, 256, 64, dtype=np.uint8).tobytes()
    for off in range(0, 40):
        lo, hi = ld8_shared(buf, off)
        assert lo == int.from_bytes(buf[off:off + 4], "little") and hi == int.from_bytes(buf[off + 4:off + 8], "little")
        # the words read never pass the one holding byte off + 7
        last_word = (off // 4 + (1 if off % 4 == 0 else 2)) if off % 8 else off // 4 + 1
        assert 4 * last_word <= off + 7 < 4 * last_word + 4
