"""The tensor-core road for long passes (prefill.cuh: 3xTF32 tcgen05 GEMMs) against the exact definition: the routing
(logits, top-k ids and weights, the dispatch permutation) bit for bit, the layer output within the north-star bound
of 1e-5 relative error.

The bound held is normwise per token: max_d |got - want| <= 1e-5 * max_d |want| over the token's output row. The
element-wise figure max_d |got - want| / |want| is printed beside it, over the elements whose magnitude is at least
1 % of their row's largest (an element of a sum with cancellation, near zero, has no meaningful relative error of its
own: there the normwise bound is the one that says something)."""
import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
REL = 1e-5


def _run(torch, m, normed, x, E, k):
    T, H = normed.shape
    dn = torch.from_numpy(normed).cuda()
    dx = torch.from_numpy(x.copy()).cuda()
    o = {"logits": torch.full((T, E), float("nan"), device="cuda"),
         "sel_id": torch.full((T * k,), -1, dtype=torch.int64, device="cuda"),
         "sel_w": torch.full((T * k,), float("nan"), device="cuda"),
         "offsets": torch.full((E + 1,), -1, dtype=torch.int64, device="cuda"),
         "place": torch.full((T * k,), -1, dtype=torch.int64, device="cuda"),
         "ffn_out": torch.full((T, H), float("nan"), device="cuda")}
    m.layer_dev(0, dn.data_ptr(), T, dx.data_ptr(), {kk: v.data_ptr() for kk, v in o.items()},
                stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    m.check()
    r = {kk: v.cpu().numpy() for kk, v in o.items()}
    r["x"] = dx.cpu().numpy()
    r["sel_id"] = r["sel_id"].reshape(T, k)
    r["sel_w"] = r["sel_w"].reshape(T, k)
    r["place"] = r["place"].reshape(T, k)
    return r


def _rel_err(got, want):
    """per token row: max |got - want| / max |want|"""
    num = np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)), axis=1)
    den = np.maximum(np.max(np.abs(want.astype(np.float64)), axis=1), 1e-30)
    return num / den


def _elem_err(got, want, floor=1e-2):
    """element-wise max |got - want| / |want| over the elements with |want| >= floor * their row's max |want|"""
    g, w = got.astype(np.float64), want.astype(np.float64)
    big = np.abs(w) >= floor * np.max(np.abs(w), axis=1, keepdims=True)
    big &= np.abs(w) > 0
    return float(np.max(np.abs(g - w)[big] / np.abs(w)[big])) if big.any() else 0.0


def _check(got, want, tag):
    for key in ("logits", "sel_id", "sel_w", "offsets", "place"):
        assert same_bits(got[key], want[key]), (tag, key)
    for key in ("ffn_out", "x"):
        assert np.all(np.isfinite(got[key])), (tag, key)
        err = _rel_err(got[key], want[key])
        print(f"{tag} {key}: max normwise relative error {err.max():.3e} (bound {REL:.0e}); "
              f"element-wise {_elem_err(got[key], want[key]):.3e} (elements >= 1% of the row's max)")
        assert err.max() <= REL, (tag, key, float(err.max()), int(err.argmax()))


@pytest.mark.parametrize("dt", [gb.Q8_0, gb.Q6_K])
def test_prefill_small_shape_against_oracle(cuda, oracle, dt):
    """a small shape against the oracle, Q8_0 gate/up with a Q8_0 or a Q6_K down (the Q6L converter)"""
    from trochilus_b200.moe import GpuMoe
    E, k, H, F, T = 16, 4, 512, 256, 300
    lay = gb.make_layer(4242, E, H, F, gb.Q8_0, dt, gb.F32, mode="random")
    bias = gb.zipf_bias(5, E)
    d, keep = make_desc(lay, H, F, k, 0, gb.F32, gb.Q8_0, dt, bias)
    m = GpuMoe(1, E, k, H, F, gb.F32, gb.Q8_0, dt, max_tokens=T)
    m.set_layer(0, lay, bias)
    assert m.launches(T) == 7  # the tensor-core road is the default for long passes
    rng = np.random.default_rng(7)
    normed = rng.normal(size=(T, H)).astype(np.float32)
    x = rng.normal(size=(T, H)).astype(np.float32)
    want = oracle.moe_layer(d, normed, x)
    _check(_run(cuda, m, normed, x, E, k), want, "tensor road")
    _check(_run(cuda, m, normed, x, E, k), want, "tensor road, second call")
    m.set_prefill(0)  # the exact road on the same context: bit for bit
    got = _run(cuda, m, normed, x, E, k)
    for key in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out", "x"):
        assert same_bits(got[key], want[key]), key
    m.close()


@pytest.mark.parametrize("gt,dt,T", [(gb.Q8_0, gb.Q8_0, 256), (gb.Q8_0, gb.Q8_0, 1000), (gb.Q8_0, gb.Q8_0, 2048),
                                     (gb.Q4_K, gb.Q6_K, 256), (gb.Q4_K, gb.Q6_K, 512), (gb.Q4_K, gb.Q4_K, 512)])
def test_prefill_olmoe_shape_against_exact_road(cuda, gt, dt, T):
    """OLMoE shape with Zipf-skewed routing (experts from one row to several 128-row tiles); the reference result is
    the exact road on the GPU, itself bit for bit the oracle's (test_gpu_layer). T = 2048 Q8_0 is the benched
    prefill call (configs[2]'s layer: Q8_0 gate/up and down, BF16 router); Q4_K / Q6_K is configs[1]'s Q4_K_M
    prompt pass, Q4_K / Q4_K configs[3]'s all-Q4_K pass."""
    from trochilus_b200.moe import GpuMoe
    E, k, H, F = 64, 8, 2048, 1024
    lay = gb.make_layer(77 + T + gt + dt, E, H, F, gt, dt, gb.BF16, mode="random")
    bias = gb.zipf_bias(9, E)
    m = GpuMoe(1, E, k, H, F, gb.BF16, gt, dt, max_tokens=T)
    m.set_layer(0, lay, bias)
    rng = np.random.default_rng(T)
    normed = rng.normal(size=(T, H)).astype(np.float32)
    x = rng.normal(size=(T, H)).astype(np.float32)
    m.set_prefill(0)
    want = _run(cuda, m, normed, x, E, k)
    m.set_prefill(T)
    got = _run(cuda, m, normed, x, E, k)
    _check(got, want, f"T={T}")
    counts = np.diff(want["offsets"])
    assert counts.max() > 128 and counts[counts > 0].min() < 128  # partial and multi-tile segments both covered
    m.close()


def test_set_prefill_on_a_q4_k_m_context(cuda):
    """Q4_K_M contexts have the tensor-core road too: the threshold moves it, a negative one is refused"""
    from trochilus_b200.moe import GpuMoe
    m = GpuMoe(1, 64, 8, 2048, 1024, gb.BF16, gb.Q4_K, gb.Q6_K, max_tokens=512)
    m.set_prefill(0)
    assert m.launches(512) != 7
    m.set_prefill(256)
    assert m.launches(512) == 7 and m.launches(255) != 7
    with pytest.raises(RuntimeError):
        m.set_prefill(-1)
    m.close()
