"""The north star's other configurations at their full sizes, where the CPU oracle would take too long, through a
size-independent property: a pass's routing and outputs equal, bit for bit, those of the same tokens run in passes
of 64 (the fused kernel's road, which the other tests hold to the oracle). Each token's arithmetic is its own, so
the split changes nothing (Trochilus's own test_prefill.c holds its engine to the same invariance).
  the router microbenchmark's T in {512, 4096, 16384}, Zipf-biased routing, experts all Q4_K and all Q8_0
              (the exact road for every pass: the tensor-core road is test_gpu_prefill.py's);
  256 rows a step (64 sequences x 4 verify rows), Q4_K_M."""
import numpy as np
import pytest

from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
E, K, H, F = 64, 8, 2048, 1024


@pytest.mark.parametrize("gt,dt,T,zipf", [(gb.Q4_K, gb.Q4_K, 512, True), (gb.Q4_K, gb.Q4_K, 4096, True),
                                          (gb.Q4_K, gb.Q4_K, 16384, True), (gb.Q8_0, gb.Q8_0, 512, True),
                                          (gb.Q8_0, gb.Q8_0, 4096, True), (gb.Q8_0, gb.Q8_0, 16384, True),
                                          (gb.Q4_K, gb.Q6_K, 256, False)])
def test_long_pass_equals_passes_of_64(cuda, gt, dt, T, zipf):
    from trochilus_b200.moe import GpuMoe
    seed = 300 + T + gt
    lay = gb.make_layer(seed, E, H, F, gt, dt, gb.F32, mode="normal")
    bias = gb.zipf_bias(seed, E) if zipf else None
    m = GpuMoe(1, E, K, H, F, gb.F32, gt, dt, max_tokens=T)
    m.set_layer(0, lay, bias)
    m.set_prefill(0)  # the exact road for every pass
    rng = np.random.default_rng(seed)
    normed = rng.normal(size=(T, H)).astype(np.float32)
    x = rng.normal(size=(T, H)).astype(np.float32)
    x_long = x.copy()
    sid, sw = m.layer(0, normed, x_long)
    x_short = x.copy()
    sid_s = np.zeros_like(sid)
    sw_s = np.zeros_like(sw)
    for i in range(0, T, 64):
        sid_s[i:i + 64], sw_s[i:i + 64] = m.layer(0, normed[i:i + 64], x_short[i:i + 64])
    assert same_bits(sid, sid_s) and same_bits(sw, sw_s)
    assert same_bits(x_long, x_short)
    if zipf:  # the bias skews the selection: the most chosen expert well above the uniform share k / E
        freq = np.bincount(sid.ravel(), minlength=E) / T
        assert freq.max() > 2 * K / E
    m.check()
    m.close()
