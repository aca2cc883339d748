"""ffn_norm moved into the hook (tr_gpu_moe_set_ffn_norm, tr_gpu_moe_ffn, tr_gpu_moe_ffn_dev): the residual
stream normalised on the GPU (Trochilus's tr_rmsnorm per token, src/kernels/kernels.c:1351-1360, as norm_body
applies it for the MoE block, src/models/olmoe.c:1834-1840), then the MoE layer. Bit for bit the oracle's
rmsnorm (itself pinned to the reference in test_oracle.py) followed by its layer: the normalised rows, the routing
and the residual, on every road (the fused kernel, the multi-kernel road, pinned x in place, device pointers)."""
import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
E, K, H, F = 64, 8, 2048, 1024


def _setup(gt, dt, rt, seed, max_tokens=80):
    from trochilus_b200.moe import GpuMoe
    rng = np.random.default_rng(seed)
    lay = gb.make_layer(int(rng.integers(1 << 30)), E, H, F, gt, dt, rt, mode="random")
    wn = (1.0 + 0.1 * rng.normal(size=H)).astype(np.float32)
    m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=max_tokens)
    m.set_layer(0, lay)
    m.set_ffn_norm(0, wn, 1e-5)
    d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt)
    return m, d, keep, wn, rng


@pytest.mark.parametrize("gt,dt,rt", [(gb.Q4_K, gb.Q6_K, gb.BF16), (gb.Q8_0, gb.Q8_0, gb.F32)])
def test_ffn_host_matches_oracle(cuda, oracle, gt, dt, rt):
    m, d, keep, wn, rng = _setup(gt, dt, rt, 31 + gt)
    for T in (1, 3, 16, 70):
        x = (rng.normal(size=(T, H)) * 3).astype(np.float32)
        normed = oracle.rmsnorm(x, wn, 1e-5)
        want = oracle.moe_layer(d, normed, x)
        got = x.copy()
        nrm, sid, sw = m.ffn(0, got, want_normed=True, want_sel=True)
        assert same_bits(nrm, normed), T
        assert same_bits(sid, want["sel_id"]) and same_bits(sw, want["sel_w"]), T
        assert same_bits(got, want["x"]), T
    m.check()
    m.close()


def test_ffn_pinned_and_device(cuda, oracle):
    torch = cuda
    m, d, keep, wn, rng = _setup(gb.Q4_K, gb.Q6_K, gb.BF16, 5)
    for T in (1, 4, 16, 24):
        x = rng.normal(size=(T, H)).astype(np.float32)
        want = oracle.moe_layer(d, oracle.rmsnorm(x, wn, 1e-5), x)
        hx = torch.from_numpy(x.copy()).pin_memory()  # short calls: read and written in place
        m.ffn_ptrs(0, T, hx.data_ptr(), host=True)
        assert same_bits(hx.numpy(), want["x"]), T
        dx = torch.from_numpy(x.copy()).cuda()
        dn = torch.full((T, H), float("nan"), device="cuda")
        m.ffn_ptrs(0, T, dx.data_ptr(), host=False, normed_ptr=dn.data_ptr(),
                   stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert same_bits(dx.cpu().numpy(), want["x"]), T
        assert same_bits(dn.cpu().numpy(), oracle.rmsnorm(x, wn, 1e-5)), T
    m.check()
    m.close()


def test_ffn_without_norm_weight_is_an_error(cuda):
    from trochilus_b200.moe import GpuMoe
    m = GpuMoe(2, E, K, H, F, gb.F32, gb.Q8_0, gb.Q8_0, max_tokens=1)
    m.set_layer(1, gb.make_layer(3, E, H, F, gb.Q8_0, gb.Q8_0, gb.F32, mode="random"))
    with pytest.raises(RuntimeError, match="ffn_norm"):
        m.ffn(1, np.zeros((1, H), np.float32))
    m.close()
