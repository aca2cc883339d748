"""Q4_K's prepared road at the kernel level (tr_q4x_prepare, tr_matmul_q4x_prepared(_n), tr_swiglu_prepare,
tr_matmul_s; src/kernels/kernels.h:279-300, 350) on host arrays, bit for bit against the CPU oracle, in the calls
Trochilus's expert_stages makes (src/models/olmoe.c:1642-1680): gate and up from the tokens' rows prepared once and
read through the counting sort's map, SwiGLU preparing the down's rows, the down from those."""
import numpy as np
import pytest

from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu


def _routing(rng, T, k, G):
    """the (token, slot) rows grouped by expert, stably (olmoe.c:1850-1861): offsets and each row's token"""
    sel = np.stack([rng.choice(G, size=k, replace=False) for _ in range(T)]).ravel()
    order = np.argsort(sel, kind="stable")
    offsets = np.concatenate([[0], np.cumsum(np.bincount(sel, minlength=G))]).astype(np.int64)
    return offsets, (order // k).astype(np.int64)


@pytest.mark.parametrize("H,F,T,G", [(512, 256, 3, 5), (2048, 1024, 4, 12), (2048, 1024, 1, 64)])
def test_expert_stages_on_the_prepared_road(cuda, oracle, H, F, T, G):
    from trochilus_b200 import moe
    rng = np.random.default_rng(H + T + G)
    k = min(8, G)
    offsets, xmap = _routing(rng, T, k, G)
    x = rng.normal(size=(T, H)).astype(np.float32)
    gate = [np.ascontiguousarray(gb.random_blocks(gb.Q4_K, F, H, rng, special=(g == 0))) for g in range(G)]
    up = [np.ascontiguousarray(gb.random_blocks(gb.Q4_K, F, H, rng)) for g in range(G)]
    down = [np.ascontiguousarray(gb.random_blocks(gb.Q4_K, H, F, rng)) for g in range(G)]
    xg = x[xmap]
    want_g = oracle.matmul_grouped(gb.Q4_K, F, H, gate, offsets, xg)
    want_u = oracle.matmul_grouped(gb.Q4_K, F, H, up, offsets, xg)
    want_h = oracle.swiglu(want_g, want_u)
    want_d = oracle.matmul_grouped(gb.Q4_K, H, F, down, offsets, want_h)

    moe.kernel_cache_clear()
    assert moe.q4x_road(gb.Q4_K, F, H) == 1 and moe.q4x_road(gb.Q4_K, H, F) == 1
    xq = moe.q4x_prepare(x)
    before = moe.q4x_fused_calls()
    rc, (h1, h2) = moe.matmul_q4x_prepared(F, H, [gate, up], offsets, xq, xmap)  # gate and up in one call
    assert rc == 1 and moe.q4x_fused_calls() == before + 1
    assert same_bits(h1, want_g) and same_bits(h2, want_u)
    rc, (h1b,) = moe.matmul_q4x_prepared(F, H, [gate], offsets, xq, xmap)  # the one-weight call
    assert rc == 1 and same_bits(h1b, want_g)
    h, hq = moe.swiglu_prepare(h1, h2)
    assert same_bits(h, want_h)
    rc, (y,) = moe.matmul_q4x_prepared(H, F, [down], offsets, hq)  # the down reads slot p for row p
    assert rc == 1 and same_bits(y, want_d)


def test_matmul_s_and_prepared_rows_without_map(cuda, oracle):
    from trochilus_b200 import moe
    rng = np.random.default_rng(9)
    w = np.ascontiguousarray(gb.random_blocks(gb.Q4_K, 48, 768, rng, special=True))
    x = rng.normal(size=(6, 768)).astype(np.float32)
    want = oracle.matmul_grouped(gb.Q4_K, 48, 768, [w], [0, 6], x)
    moe.kernel_cache_clear()
    assert same_bits(moe.matmul_s(gb.Q4_K, 48, 768, w, x), want)
    rc, (y,) = moe.matmul_q4x_prepared(48, 768, [[w]], [0, 6], moe.q4x_prepare(x))
    assert rc == 1 and same_bits(y, want)
    q8 = np.ascontiguousarray(gb.random_blocks(gb.Q8_0, 40, 512, rng))
    x8 = rng.normal(size=(3, 512)).astype(np.float32)
    assert same_bits(moe.matmul_s(gb.Q8_0, 40, 512, q8, x8), oracle.matmul_grouped(gb.Q8_0, 40, 512, [q8], [0, 3], x8))
