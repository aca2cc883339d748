"""The kernel-level C ABI (tr_matmul, tr_matmul_grouped(_s), tr_softmax, tr_swiglu) on host arrays,
bit for bit against the CPU oracle, on the reference's grouped layouts (tests/test_kernels.c:1785-1888)."""
import numpy as np
import pytest

from tests.golden.cases import same_bits, witness_inputs
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu

LAYOUTS = [np.array([0, 0, 1, 1, 4, 9, 9]), np.array([0, 5]), np.array([0, 1, 2, 3, 4, 5, 6]),
           np.array([0, 0, 0, 3])]


@pytest.mark.parametrize("t,rows,cols", [(gb.Q8_0, 48, 512), (gb.Q8_0, 1024, 2048), (gb.Q4_K, 40, 512),
                                         (gb.Q4_K, 2048, 1024), (gb.Q4_K, 24, 2560), (gb.Q6_K, 30, 256),
                                         (gb.Q6_K, 2048, 1024), (gb.F32, 64, 2048), (gb.BF16, 17, 96),
                                         (gb.F16, 33, 48)])
def test_matmul_grouped(cuda, oracle, t, rows, cols):
    from trochilus_b200 import moe
    rng = np.random.default_rng(rows * 7 + cols + t)
    for li, offsets in enumerate(LAYOUTS):
        G = len(offsets) - 1
        if t in (gb.F32, gb.BF16, gb.F16):
            w = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
            if t == gb.BF16:
                mk = lambda: gb.quantize(gb.BF16, gb.round_to_bf16(rng.normal(0, .02, size=(rows, cols)).astype(np.float32)))
            elif t == gb.F16:
                mk = lambda: rng.normal(0, .02, size=(rows, cols)).astype(np.float16).view(np.uint8).reshape(rows, -1)
            else:
                mk = lambda: gb.quantize(gb.F32, rng.normal(0, .02, size=(rows, cols)).astype(np.float32))
        else:
            mk = lambda: gb.random_blocks(t, rows, cols, rng, special=(li == 0))
        mats = [np.ascontiguousarray(mk()) for _ in range(G)]
        n = int(offsets[-1])
        x = witness_inputs(rng, n, cols) if li == 0 and n >= 6 else rng.normal(size=(n, cols)).astype(np.float32)
        want = oracle.matmul_grouped(t, rows, cols, mats, offsets, x)
        moe.kernel_cache_clear()  # the cache keys weights by host address, which numpy reuses
        got = moe.matmul_grouped(t, rows, cols, mats, offsets, x, use_s=(li % 2 == 1))
        assert same_bits(got, want), (li, np.argwhere(~((got == want) | (np.isnan(got) & np.isnan(want))))[:5])


def test_matmul_router_shape(cuda, oracle):
    from trochilus_b200 import moe
    rng = np.random.default_rng(2)
    w = gb.quantize(gb.F32, rng.normal(0, 0.02, size=(64, 2048)).astype(np.float32))
    x = rng.normal(size=(5, 2048)).astype(np.float32)
    moe.kernel_cache_clear()
    assert same_bits(moe.matmul(gb.F32, 64, 2048, w, x), oracle.matmul_grouped(gb.F32, 64, 2048, [w], [0, 5], x))


def test_softmax_and_swiglu(cuda, oracle):
    from trochilus_b200 import moe
    rng = np.random.default_rng(3)
    for n in (1, 5, 64, 333, 5000):
        x = (rng.normal(size=n) * 6).astype(np.float32)
        assert same_bits(moe.softmax(x), oracle.softmax(x)), n
    x = (rng.normal(size=100000) * 9).astype(np.float32)
    x[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 88.7]
    y = rng.normal(size=100000).astype(np.float32)
    assert same_bits(moe.swiglu(x, y), oracle.swiglu(x, y))


def test_expf_through_softmax_exceptions(cuda, oracle):
    """every argument of the exception table reaches the device exp (a two-element softmax with 0 puts x - 0)"""
    from trochilus_b200 import moe
    from trochilus_b200.csrc_consts import exceptions
    for xb, _ in exceptions():
        v = np.array([xb], np.uint32).view(np.float32)[0]
        z = np.array([v, np.float32(0) if v < 0 else v], np.float32)
        assert same_bits(moe.softmax(z), oracle.softmax(z))
