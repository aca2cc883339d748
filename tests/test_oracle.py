"""The CPU oracle (oracle/moe_oracle.c) pinned against Trochilus's own code (oracle/_ref) and against the
golden vectors that code produced (tests/golden). CPU only."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import CASES, build_case, digest, same_bits
from trochilus_b200 import gguf_blocks as gb

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _special_floats():
    u = np.array([0x00000000, 0x80000000, 0x00000001, 0x007fffff, 0x00800000, 0x3f800000, 0xbf800000, 0x7f7fffff,
                  0xff7fffff, 0x7f800000, 0xff800000, 0x7fc00000, 0x42b17218, 0x42b17217, 0x42b17219, 0xc2d00000,
                  0xc2cff1b5, 0xc2cff1b4, 0xc2ce8ed0], dtype=np.uint32)
    return u.view(np.float32)


def test_expf_pinned_to_reference_sampled(oracle, reflib):
    rng = np.random.default_rng(5)
    x = rng.integers(0, 2 ** 32, size=1 << 22, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([x, _special_floats(), np.linspace(-110, 90, 200001, dtype=np.float32)])
    assert same_bits(oracle.expf(x), reflib.expf(x))


def test_expf_exception_table(oracle):
    from trochilus_b200.csrc_consts import exceptions
    for xb, yb in exceptions():
        y = oracle.expf(np.array([xb], np.uint32).view(np.float32))
        assert y.view(np.uint32)[0] == yb


@pytest.mark.skipif(os.environ.get("TRX_EXHAUSTIVE") != "1", reason="all 2^32 floats: set TRX_EXHAUSTIVE=1")
def test_expf_exhaustive(oracle, reflib):
    for hi in range(1 << 8):
        u = (np.arange(1 << 24, dtype=np.uint64) + (hi << 24)).astype(np.uint32)
        x = u.view(np.float32)
        assert same_bits(oracle.expf(x), reflib.expf(x)), hex(hi)


@pytest.mark.parametrize("type_,n", [(gb.F32, 2048), (gb.BF16, 2048), (gb.Q8_0, 2048), (gb.Q8_0, 1024),
                                     (gb.Q4_K, 2048), (gb.Q4_K, 512), (gb.Q6_K, 1024), (gb.Q6_K, 256)])
@pytest.mark.parametrize("special", [False, True])
def test_dot_row_pinned_to_reference(oracle, reflib, type_, n, special):
    from tests.golden.cases import witness_inputs
    rng = np.random.default_rng(n + type_ + special)
    if type_ in (gb.F32, gb.BF16):
        rows = gb.quantize(type_, gb.round_to_bf16(rng.normal(0, 0.02, size=(8, n)).astype(np.float32)))
    else:
        rows = gb.random_blocks(type_, 8, n, rng, special=special)
    xs = witness_inputs(rng, 6, n) if special else rng.normal(size=(6, n)).astype(np.float32)
    for r in range(rows.shape[0]):
        for x in xs:
            a, b = oracle.dot_row(type_, rows[r], x), reflib.dot_row(type_, rows[r], x)
            assert same_bits(np.float32(a), np.float32(b)), (r, a, b)


def test_dot_row_not_blind(oracle):
    """one ulp of one block's d changes the result (the comparison can see a wrong bit)"""
    rng = np.random.default_rng(3)
    for t in (gb.Q8_0, gb.Q4_K, gb.Q6_K):
        row = gb.random_blocks(t, 1, 512, rng)[0]
        x = rng.normal(size=512).astype(np.float32)
        good = oracle.dot_row(t, row, x)
        off = {gb.Q8_0: 34, gb.Q4_K: 144, gb.Q6_K: 210 + 208}[t]
        bad = row.copy()
        bad[off] ^= 1
        assert not same_bits(np.float32(good), np.float32(oracle.dot_row(t, bad, x)))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_golden(oracle, case):
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    lay, bias, normed, x = build_case(case)
    assert digest(lay, bias, normed, x) == str(g["digest"]), "the synthetic generator changed: regenerate fixtures"
    if case["T"] > 16:
        pytest.skip("long case: covered on the GPU against the reference fixture")
    d, keep = make_desc(lay, case["H"], case["F"], case["k"], case["norm_topk"], case["router"], case["gate"],
                        case["down"], bias)
    r = oracle.moe_layer(d, normed, x)
    for key in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out", "x"):
        assert same_bits(r[key], g[key]), key


def test_oracle_matches_reference_live(oracle, reflib):
    """fresh seeds, every type pair, T from 1 to 9, routing with and without renormalisation"""
    rng = np.random.default_rng(77)
    pool = reflib.pool(0)
    for i, (gt, dt, rt) in enumerate([(gb.Q8_0, gb.Q8_0, gb.F32), (gb.Q4_K, gb.Q6_K, gb.BF16),
                                      (gb.Q4_K, gb.Q4_K, gb.F32), (gb.Q8_0, gb.Q4_K, gb.BF16)]):
        E, k, H, F = (64, 8, 2048, 1024) if i % 2 == 0 else (32, 6, 2048, 512)
        lay = gb.make_layer(500 + i, E, H, F, gt, dt, rt, mode="random", special=(i == 2))
        T = int(rng.integers(1, 10))
        normed = rng.normal(size=(T, H)).astype(np.float32)
        x = rng.normal(size=(T, H)).astype(np.float32)
        d, keep = make_desc(lay, H, F, k, i % 2, rt, gt, dt, None)
        a = oracle.moe_layer(d, normed, x)
        b = reflib.moe_layer(d, normed, x, pool=pool)
        for key in ("logits", "sel_id", "sel_w", "offsets", "place", "h1", "h3", "ffn_out", "x"):
            assert same_bits(a[key], b[key]), (i, key)
    reflib.pool_destroy(pool)


def test_grouped_layout_edges(oracle, reflib):
    """the reference's grouped-matmul layouts (tests/test_kernels.c:1785-1888): empty groups first, middle
    and last, one-row groups, odd row counts"""
    rng = np.random.default_rng(9)
    for t, rows, cols in ((gb.Q8_0, 48, 512), (gb.Q4_K, 32, 512), (gb.Q6_K, 16, 256), (gb.F32, 24, 64)):
        mats = [gb.random_blocks(t, rows, cols, rng) if t != gb.F32 else
                gb.quantize(gb.F32, rng.normal(size=(rows, cols)).astype(np.float32)) for _ in range(6)]
        offsets = np.array([0, 0, 1, 1, 4, 9, 9])
        x = rng.normal(size=(9, cols)).astype(np.float32)
        assert same_bits(oracle.matmul_grouped(t, rows, cols, mats, offsets, x),
                         reflib.matmul_grouped(t, rows, cols, mats, offsets, x))


def test_softmax_swiglu_pinned(oracle, reflib):
    rng = np.random.default_rng(4)
    for n in (1, 7, 16, 64, 100, 1000):
        x = (rng.normal(size=n) * 5).astype(np.float32)
        assert same_bits(oracle.softmax(x), reflib.softmax(x))
    x = (rng.normal(size=5000) * 8).astype(np.float32)
    y = rng.normal(size=5000).astype(np.float32)
    x[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 100.0]
    assert same_bits(oracle.swiglu(x, y), reflib.swiglu(x, y))


@pytest.mark.parametrize("tier", ["scalar", "avx2", "avx512"])
def test_rmsnorm_pinned(oracle, reflib, tier):
    """ffn_norm (src/kernels/kernels.c:1351-1360): the restatement against the reference's every tier, on rows of
    several widths and scales, and rows holding zeros, subnormals, huge values, infinities and NaNs"""
    try:
        reflib.set_tier(tier)
    except RuntimeError:
        pytest.skip(f"tier {tier} not on this CPU")
    try:
        rng = np.random.default_rng(9)
        for n in (16, 64, 100, 2048):
            for scale in (1e-20, 1e-3, 1.0, 40.0, 1e18):
                x = (rng.normal(size=(3, n)) * scale).astype(np.float32)
                w = rng.normal(size=n).astype(np.float32)
                for eps in (1e-5, 1e-6, 0.0):
                    assert same_bits(oracle.rmsnorm(x, w, eps), reflib.rmsnorm(x, w, eps)), (n, scale, eps)
        x = rng.normal(size=(6, 2048)).astype(np.float32)
        w = rng.normal(size=2048).astype(np.float32)
        x[0] = 0.0
        x[1, :64] = np.resize(_special_floats(), 64)
        x[2, 5] = np.inf
        x[3, 7] = np.nan
        x[4] *= 1e-41  # subnormal squares
        assert same_bits(oracle.rmsnorm(x, w, 1e-5), reflib.rmsnorm(x, w, 1e-5))
    finally:
        reflib.set_tier(None)


@pytest.mark.parametrize("t", [gb.Q8_0, gb.Q4_K, gb.Q6_K])
def test_encoders_decode_close(reflib, t):
    """this project's encoders give blocks the reference decodes back to the inputs (within the format's step)"""
    rng = np.random.default_rng(t)
    w = rng.normal(0, 0.02, size=(4, 512)).astype(np.float32)
    q = gb.quantize(t, w)
    for r in range(4):
        back = reflib.dequant_row(t, q[r], 512)
        tol = {gb.Q8_0: 0.02 * 4 / 127, gb.Q4_K: 0.02 * 8 / 15 * 1.2, gb.Q6_K: 0.02 * 4 / 31}[t]
        assert np.max(np.abs(back - w[r])) < tol


class _PmScratch(C.Structure):
    """Trochilus's tr_pm_scratch (src/kernels/kernels.h:250-262)"""
    _fields_ = [("xil", C.c_void_p), ("max_x", C.c_int64), ("xq", C.c_void_p), ("xq_bytes", C.c_int64),
                ("work", C.c_void_p), ("max_cols", C.c_int64), ("n_workers", C.c_int), ("plan", C.c_void_p),
                ("max_groups", C.c_int64), ("max_tokens", C.c_int64)]


def _aligned(nbytes, align=64):
    buf = np.zeros(nbytes + align, dtype=np.uint8)
    off = (-buf.ctypes.data) % align
    return buf[off:off + nbytes]


@pytest.mark.parametrize("rows,cols", [(64, 512), (1024, 2048), (2048, 1024)])
def test_reference_prepared_road_equals_float_road(oracle, reflib, rows, cols):
    """The premise of the library's prepared road: the reference's Q4_K road on rows prepared once
    (tr_q4x_prepare + tr_matmul_q4x_prepared(_n), src/kernels/kernels.c:1157-1228), a group's row read through a map,
    gives the float road's outputs (the oracle's grouped matmul on the gathered floats) bit for bit, so a library
    whose prepared rows are the floats themselves returns the same y."""
    L = reflib.lib
    L.tr_pm_scratch_init.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
    L.tr_pm_scratch_free.argtypes = [C.c_void_p]
    L.tr_q4x_bytes.restype = C.c_size_t
    L.tr_q4x_bytes.argtypes = [C.c_int64]
    L.tr_q4x_prepare.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
    L.tr_matmul_q4x_prepared.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p]
    L.tr_matmul_q4x_prepared_n.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p]

    class Mat(C.Structure):
        _fields_ = [("type", C.c_int32), ("rows", C.c_int64), ("cols", C.c_int64), ("data", C.c_void_p)]

    rng = np.random.default_rng(rows + cols)
    G, T, k = 6, 5, 4
    R = T * k
    sel = np.stack([rng.choice(G, size=k, replace=False) for _ in range(T)]).ravel()
    order = np.argsort(sel, kind="stable")  # the counting sort's rows: by group, then by (token, slot)
    offsets = np.concatenate([[0], np.cumsum(np.bincount(sel, minlength=G))]).astype(np.int64)
    xmap = (order // k).astype(np.int64)
    x = rng.normal(size=(T, cols)).astype(np.float32)
    x[1, :7] = [0.0, -0.0, 1e-40, -3e38, 3e38, 1.0, -1.0]
    mats = [[np.ascontiguousarray(gb.random_blocks(gb.Q4_K, rows, cols, rng)) for _ in range(G)] for _ in range(2)]
    want = [oracle.matmul_grouped(gb.Q4_K, rows, cols, m, offsets, x[xmap]) for m in mats]
    pool = reflib.pool(4)
    s = _PmScratch()
    assert L.tr_pm_scratch_init(C.byref(s), 4, G, R, cols, R * cols) == 0
    try:
        xq = _aligned(T * int(L.tr_q4x_bytes(cols)))
        L.tr_q4x_prepare(pool, x.ctypes.data, T, cols, xq.ctypes.data)
        ws = [(Mat * G)(*[Mat(gb.Q4_K, rows, cols, mm.ctypes.data) for mm in m]) for m in mats]
        y = np.full((R, rows), np.nan, dtype=np.float32)
        assert L.tr_matmul_q4x_prepared(pool, C.cast(ws[0], C.c_void_p), offsets.ctypes.data, G, xq.ctypes.data,
                                        xmap.ctypes.data, y.ctypes.data, C.byref(s)) == 1
        assert same_bits(y, want[0])
        ys = [np.full((R, rows), np.nan, dtype=np.float32) for _ in range(2)]
        wp = (C.c_void_p * 2)(*[C.cast(w, C.c_void_p) for w in ws])
        yp = (C.c_void_p * 2)(*[v.ctypes.data for v in ys])
        assert L.tr_matmul_q4x_prepared_n(pool, wp, 2, offsets.ctypes.data, G, xq.ctypes.data, xmap.ctypes.data, yp,
                                          C.byref(s)) == 1
        assert same_bits(ys[0], want[0]) and same_bits(ys[1], want[1])
    finally:
        L.tr_pm_scratch_free(C.byref(s))
        reflib.lib.ref_pool_destroy(pool)


@pytest.mark.parametrize("m,what", [(1, "lanes joined in sequence"), (2, "mix in decreasing slot order"),
                                    (3, "ties to the higher id"), (4, "Q4_K blocks summed in float"),
                                    (5, "SwiGLU by a reciprocal"), (6, "RMSNorm associated the other way")])
def test_planted_mistakes_are_seen(oracle, reflib, m, what):
    """Each mistake planted in the restatement (one step of the definition changed) makes its result differ from
    the reference's in the bits the GPU tests compare, so those comparisons are not blind (the restatement without
    it matches the reference in the tests above; Trochilus's mutation tests, tools/mutate_gpu.sh:2-10)."""
    rng = np.random.default_rng(60 + m)
    pool = reflib.pool(0)

    def layer(lay, E, k, H, F, rt, gt, dt, T):
        d, keep = make_desc(lay, H, F, k, 0, rt, gt, dt, None)
        normed = rng.normal(size=(T, H)).astype(np.float32)
        x = rng.normal(size=(T, H)).astype(np.float32)
        return oracle.moe_layer(d, normed, x), reflib.moe_layer(d, normed, x, pool=pool)

    try:
        oracle.set_mutation(m)
        if m in (1, 2, 4):
            gt = gb.Q4_K if m == 4 else gb.Q8_0
            lay = gb.make_layer(70 + m, 16, 512, 256, gt, gt, gb.F32, mode="random")
            a, b = layer(lay, 16, 4, 512, 256, gb.F32, gt, gt, 3)
            key = "logits" if m == 1 else "x"
            seen = not same_bits(a[key], b[key])
        elif m == 3:  # a zero router: every probability ties
            lay = gb.make_layer(73, 16, 512, 256, gb.Q8_0, gb.Q8_0, gb.F32, mode="random")
            lay["router"] = np.zeros_like(lay["router"])
            a, b = layer(lay, 16, 4, 512, 256, gb.F32, gb.Q8_0, gb.Q8_0, 2)
            assert (b["sel_id"] == np.arange(4)).all()  # the reference: ties to the lower id
            seen = not same_bits(a["sel_id"], b["sel_id"])
        elif m == 5:
            x = (rng.normal(size=4096) * 4).astype(np.float32)
            y = rng.normal(size=4096).astype(np.float32)
            seen = not same_bits(oracle.swiglu(x, y), reflib.swiglu(x, y))
        else:
            x = (rng.normal(size=(4, 2048)) * 3).astype(np.float32)
            w = (1.0 + 0.1 * rng.normal(size=2048)).astype(np.float32)
            seen = not same_bits(oracle.rmsnorm(x, w, 1e-5), reflib.rmsnorm(x, w, 1e-5))
        assert seen, what
    finally:
        oracle.set_mutation(0)
        reflib.pool_destroy(pool)


@pytest.mark.parametrize("tier", ["scalar", "avx2", "avx512"])
def test_attention_head_pinned(oracle, reflib, tier):
    """one decode token's attention (tr_attention_head, src/kernels/kernels.c:1521-1528; the GPU attention's
    contract, src/backend/gpu_attn.h:1-9): the restatement against the reference's every tier, head by head at its
    offset in the cache rows, for contexts from one position to past 2048, with huge scores, a NaN and an
    infinity"""
    try:
        reflib.set_tier(tier)
    except RuntimeError:
        pytest.skip(f"tier {tier} not on this CPU")
    L = reflib.lib
    L.tr_attention_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                    C.c_float, C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(11)
    n_head, hd = 4, 128
    scale = np.float32(1.0 / np.sqrt(hd))
    try:
        for n_pos in (1, 2, 7, 100, 2049):
            q = rng.normal(size=(n_head, hd)).astype(np.float32)
            keys = rng.normal(size=(n_pos, n_head, hd)).astype(np.float32)
            values = rng.normal(size=(n_pos, n_head, hd)).astype(np.float32)
            q[1] *= 40.0  # scores far apart: probabilities underflow to 0
            if n_pos > 5:
                values[3, 2, 9] = np.nan
                keys[4, 3, 0] = np.inf
            want = np.zeros((n_head, hd), dtype=np.float32)
            scores = np.zeros(n_pos, dtype=np.float32)
            for h in range(n_head):
                L.tr_attention_head(q[h].ctypes.data, keys.ctypes.data, values.ctypes.data, n_head * hd, h * hd, n_pos,
                                    hd, scale, scores.ctypes.data, want[h].ctypes.data)
            assert same_bits(oracle.attention(q, keys, values, scale), want), n_pos
    finally:
        reflib.set_tier(None)


@pytest.mark.parametrize("t", [gb.Q8_0, gb.Q4_K, gb.Q6_K])
def test_block_formats_match_gguf_py(reflib, t):
    """the GGUF block formats as the reference decodes them equal gguf-py's dequantisation bit for bit (Trochilus's
    tools/check_dequant.py check), on random blocks with special scales (zero, subnormal, negative, large): the
    weights every parity test feeds the GPU are read as the file format defines them"""
    import gguf
    from gguf import quants
    rng = np.random.default_rng(40 + t)
    for special in (False, True):
        blk = gb.random_blocks(t, 6, 1024, rng, special=special)
        ref = np.stack([reflib.dequant_row(t, blk[i], 1024) for i in range(6)])
        want = quants.dequantize(blk, gguf.GGMLQuantizationType(t)).astype(np.float32)
        assert same_bits(ref, want), (t, special)
