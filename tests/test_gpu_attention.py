"""Decode attention on the GPU (tr_gpu_open, tr_gpu_attn_create / _write / _decode / _warm: Trochilus's
src/backend/gpu_attn.h on the B200) bit for bit against the CPU oracle's tr_attention_head (itself pinned to every
tier of the reference in test_oracle.py), as the reference's tests/test_gpu_attn.c checks its own backend: a
prompt written into the cache, then decode tokens at contexts that cross the value kernel's 64-position stages,
several layers and heads, a NaN and an infinity in the cache."""
import numpy as np
import pytest

from tests.golden.cases import same_bits

pytestmark = pytest.mark.gpu


def test_decode_attention_matches_oracle(cuda, oracle):
    from trochilus_b200.moe import GpuAttn
    n_layers, n_head, hd, n_ctx = 2, 16, 128, 2100
    rng = np.random.default_rng(5)
    a = GpuAttn(n_layers, n_head, n_ctx)
    assert a.name()
    scale = np.float32(1.0 / np.sqrt(hd))
    for layer in range(n_layers):
        P = 1000 + 37 * layer  # the prompt's positions
        keys = rng.normal(size=(n_ctx, n_head, hd)).astype(np.float32)
        values = rng.normal(size=(n_ctx, n_head, hd)).astype(np.float32)
        keys[5, 3, 7] = np.inf
        values[9, 2, 100] = np.nan
        a.write(layer, 0, keys[:P], values[:P])
        written = P  # positions 0 .. written - 1 hold keys / values
        for pos in (P, P + 1, P + 63, P + 64, P + 1099 - 37 * layer):
            if pos > written:  # the positions between: written as a prompt's would be
                a.write(layer, written, keys[written:pos], values[written:pos])
            q = (rng.normal(size=(n_head, hd)) * (1 + layer)).astype(np.float32)
            got = a.decode(layer, pos, q, keys[pos], values[pos], scale)  # stores k and v at pos first
            written = pos + 1
            want = oracle.attention(q, keys[:pos + 1], values[:pos + 1], scale)
            assert same_bits(got, want), (layer, pos)
    a.warm(1_000_000)
    got = a.decode(0, 0, np.ones((n_head, hd), np.float32), keys[0], values[0], scale)  # one position: its value
    assert same_bits(got, oracle.attention(np.ones((n_head, hd), np.float32), keys[:1], values[:1], scale))
    a.close()


def test_decode_attention_small_contexts(cuda, oracle):
    """the first positions of a cache (1..70) and a single head"""
    from trochilus_b200.moe import GpuAttn
    rng = np.random.default_rng(6)
    a = GpuAttn(1, 1, 80)
    keys = rng.normal(size=(80, 1, 128)).astype(np.float32)
    values = rng.normal(size=(80, 1, 128)).astype(np.float32)
    for pos in range(70):
        q = rng.normal(size=(1, 128)).astype(np.float32)
        got = a.decode(0, pos, q, keys[pos], values[pos], 0.125)
        assert same_bits(got, oracle.attention(q, keys[:pos + 1], values[:pos + 1], np.float32(0.125))), pos
    a.close()
