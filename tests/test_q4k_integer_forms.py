"""The exactness argument of the one-token kernel's tensor-core Q4_K products (layouts.cuh: trx_prep_q4m_block,
trx_q4k_blk_mma), restated in numpy and checked against Trochilus's integer definition of a Q4_K block
(src/kernels/kernels.c:196-253: T = sum_j sc_j sum_{k in j} q_k X_k, M = sum_j m_j sum_{k in j} X_k, exact).

The kernel forms T from mma.sync m16n8k32 products (u8 quants x s8 digits, s32 sums) of one sub-block each:
- X is split into four balanced base-256 digits, D0 + 256 D1 + 65536 D2 + 2^24 D3, each in [-128, 127];
- a high-nibble sub-block enters as 16 q (the byte masked in place) and its scaled sum is shifted right by 4;
- the 6-bit scales and mins are unpacked four at a time from the 12 packed bytes.
Every step must be exact and every partial sum must fit its int32 register. CPU only: the GPU tests compare the
kernel's outputs with the oracle bit for bit."""
import numpy as np
import pytest

from trochilus_b200 import gguf_blocks as gb

XMAX = 2085998640  # the largest |X| the input preparation produces (its shift keeps max|x| 2^sh below this)


def balanced_digits(X):
    D = np.zeros((4,) + X.shape, dtype=np.int64)
    r = X.astype(np.int64)
    for p in range(4):
        d = ((r + 128) & 255) - 128 if p < 3 else r.copy()
        D[p] = d
        r = (r - d) >> 8
    return D


def packed_scales(blk):
    """the kernel's four-at-a-time unpacking of the 12 scale bytes (header words y, z, w)"""
    y, z, w = (int.from_bytes(blk[o:o + 4].tobytes(), "little") for o in (4, 8, 12))
    sc03, sc47 = y & 0x3F3F3F3F, (w & 0x0F0F0F0F) | ((y >> 2) & 0x30303030)
    m03, m47 = z & 0x3F3F3F3F, ((w >> 4) & 0x0F0F0F0F) | ((z >> 2) & 0x30303030)
    byte = lambda v, i: (v >> (8 * i)) & 255
    return ([byte(sc03, i) for i in range(4)] + [byte(sc47, i) for i in range(4)],
            [byte(m03, i) for i in range(4)] + [byte(m47, i) for i in range(4)])


def definition_scales(blk):
    """the GGUF / Trochilus unpacking, one value at a time"""
    s = blk[4:16].astype(int)
    sc = [s[j] & 63 if j < 4 else (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4) for j in range(8)]
    mm = [s[j + 4] & 63 if j < 4 else (s[j + 4] >> 4) | ((s[j] >> 6) << 4) for j in range(8)]
    return sc, mm


def quants(blk):
    q = np.zeros(256, dtype=np.int64)
    qs = blk[16:144].astype(np.int64)
    for j in range(4):
        q[64 * j:64 * j + 32] = qs[32 * j:32 * j + 32] & 15
        q[64 * j + 32:64 * j + 64] = qs[32 * j:32 * j + 32] >> 4
    return q


def tensor_core_T(blk, X):
    """T as the kernel forms it, with every int32 partial checked for range"""
    D = balanced_digits(X)
    assert D.min() >= -128 and D.max() <= 127
    sc, _ = packed_scales(blk)
    qs = blk[16:144].astype(np.int64)
    lo, hi = np.zeros(4, dtype=np.int64), np.zeros(4, dtype=np.int64)
    for j in range(4):
        ql = qs[32 * j:32 * j + 32] & 0x0F   # sub-block 2 j: the low nibbles
        qh = qs[32 * j:32 * j + 32] & 0xF0   # sub-block 2 j + 1: 16 q, masked in place
        for p in range(4):
            cl = int(np.dot(ql, D[p, 64 * j:64 * j + 32]))
            ch = int(np.dot(qh, D[p, 64 * j + 32:64 * j + 64]))
            assert abs(cl) < 2 ** 31 and abs(ch) < 2 ** 31 and ch % 16 == 0
            lo[p] += sc[2 * j] * cl
            hi[p] += sc[2 * j + 1] * ch
    assert np.all(np.abs(lo) < 2 ** 31) and np.all(np.abs(hi) < 2 ** 31)
    P = lo + (hi >> 4)
    assert np.all(np.abs(P) < 2 ** 31)
    return int(P[0] + 256 * P[1]) + 65536 * int(P[2] + 256 * P[3])


def test_balanced_digits_fit_s8_at_the_extremes():
    # (8421504 = 128 (1 + 256 + 65536): the most the three lower digits can take away from the top one)
    X = np.array([XMAX, -XMAX, XMAX - 1, -XMAX + 1, XMAX - 8421504, -XMAX + 8421504, 0, 1, -1, 127, 128, -128, -129,
                  8421504, -8421504, 2 ** 31 - 2 ** 24 - 8421505], dtype=np.int64)
    D = balanced_digits(X)
    assert D.min() >= -128 and D.max() <= 127
    assert np.array_equal(D[0] + 256 * D[1] + 65536 * D[2] + 16777216 * D[3], X)


@pytest.mark.parametrize("special", [False, True])
def test_tensor_core_sums_equal_the_definition(special):
    rng = np.random.default_rng(20261202 + special)
    for trial in range(300):
        blk = gb.random_blocks(gb.Q4_K, 1, 256, rng, special=special)[0]
        sc, mm = packed_scales(blk)
        assert (sc, mm) == definition_scales(blk)
        # inputs at the full range of the preparation, random and at the extremes
        X = rng.integers(-XMAX, XMAX + 1, size=256, dtype=np.int64)
        if trial % 3 == 0:
            X = rng.choice(np.array([XMAX, -XMAX, 0], dtype=np.int64), size=256)
        q = quants(blk)
        T_def = sum(sc[j] * int(np.dot(q[32 * j:32 * j + 32], X[32 * j:32 * j + 32])) for j in range(8))
        assert tensor_core_T(blk, X) == T_def
        assert abs(T_def) < 2 ** 49  # exact as a double, as the f64 finish needs
        # M from the sub-block sums, as the kernel's lanes add it in f64 (exact: below 2^53)
        S = [int(X[32 * j:32 * j + 32].sum()) for j in range(8)]
        M = sum(mm[j] * S[j] for j in range(8))
        assert abs(M) < 2 ** 53 and float(M) == M
