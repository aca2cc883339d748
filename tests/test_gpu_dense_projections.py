"""The dense projections of an OLMoE layer through the kernel level, as a relinked engine calls them
(src/models/olmoe.c:1722-1737, 1822, 1989): q, k and v (2048 x 2048, Q4_K) in one tr_matmul_q4x_prepared_n call on
the tokens' rows prepared once, o (2048 x 2048, Q4_K) by tr_matmul_s, and the output head (50304 x 2048, Q6_K) by
tr_matmul_s; each bit for bit the oracle's dot rows."""
import numpy as np
import pytest

from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
H = 2048


def test_qkv_o_and_head(cuda, oracle):
    from trochilus_b200 import moe
    rng = np.random.default_rng(12)
    T = 3
    x = rng.normal(size=(T, H)).astype(np.float32)
    moe.kernel_cache_clear()
    qkv = [np.ascontiguousarray(gb.random_blocks(gb.Q4_K, H, H, rng)) for _ in range(3)]
    rc, ys = moe.matmul_q4x_prepared(H, H, [[w] for w in qkv], [0, T], moe.q4x_prepare(x))
    assert rc == 1
    for w, y in zip(qkv, ys):
        assert same_bits(y, oracle.matmul_grouped(gb.Q4_K, H, H, [w], [0, T], x))
    wo = np.ascontiguousarray(gb.random_blocks(gb.Q4_K, H, H, rng))
    assert same_bits(moe.matmul_s(gb.Q4_K, H, H, wo, x), oracle.matmul_grouped(gb.Q4_K, H, H, [wo], [0, T], x))
    n_vocab = 50304
    head = np.ascontiguousarray(gb.random_blocks(gb.Q6_K, n_vocab, H, rng))
    got = moe.matmul_s(gb.Q6_K, n_vocab, H, head, x[:1])
    assert same_bits(got, oracle.matmul_grouped(gb.Q6_K, n_vocab, H, [head], [0, 1], x[:1]))
    moe.kernel_cache_clear()
