"""The tie rule of the routing on the GPU roads: a zero router makes every probability equal (Trochilus's synthetic
model knob for ties, tests/synth_olmoe.h:22-80), and the k rounds of argmax must take ids 0..k-1."""
import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 5, 70])
def test_zero_router_ties(cuda, oracle, T):
    """a zero router (Trochilus's synthetic-model knob for ties, tests/synth_olmoe.h:22-80): every probability is
    1/E, so the k rounds of argmax take ids 0..k-1 (strict >, ties to the lower id, olmoe.c:1455-1502) on the fused
    kernel (T <= 64) and on the multi-kernel road; bit for bit the oracle's, which tests/test_oracle.py shows would
    see ties broken the other way"""
    from trochilus_b200.moe import GpuMoe
    E, k, H, F = 16, 4, 512, 256
    lay = gb.make_layer(880 + T, E, H, F, gb.Q8_0, gb.Q6_K, gb.F32, mode="random")
    lay["router"] = np.zeros_like(lay["router"])
    d, keep = make_desc(lay, H, F, k, 0, gb.F32, gb.Q8_0, gb.Q6_K)
    m = GpuMoe(1, E, k, H, F, gb.F32, gb.Q8_0, gb.Q6_K, max_tokens=T)
    m.set_layer(0, lay)
    rng = np.random.default_rng(T)
    normed = rng.normal(size=(T, H)).astype(np.float32)
    x = rng.normal(size=(T, H)).astype(np.float32)
    want = oracle.moe_layer(d, normed, x)
    assert (want["sel_id"] == np.arange(k)).all()
    xo = x.copy()
    sid, sw = m.layer(0, normed, xo)
    assert same_bits(sid, want["sel_id"]) and same_bits(sw, want["sel_w"]) and same_bits(xo, want["x"])
    m.check()
    m.close()
