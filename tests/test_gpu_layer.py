"""The MoE layer on the GPU through the C ABI (tr_gpu_moe_*), compared bit for bit with Trochilus's own
outputs (golden vectors) and with the CPU oracle (fresh seeds): logits, top-k ids and weights, the
dispatch permutation, the layer output and the residual."""
import os

import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import CASES, build_case, digest, same_bits
from trochilus_b200 import gguf_blocks as gb

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
pytestmark = pytest.mark.gpu


def _ctx(c, n_layers=1, max_tokens=None):
    from trochilus_b200.moe import GpuMoe
    return GpuMoe(n_layers, c["E"], c["k"], c["H"], c["F"], c["router"], c["gate"], c["down"],
                  max_tokens or c["T"], norm_topk=c["norm_topk"])


def _dev_outputs(torch, m, layer, normed, x, E, k):
    T, H = normed.shape
    dn = torch.from_numpy(normed).cuda()
    dx = torch.from_numpy(x.copy()).cuda()
    o = {"logits": torch.full((T, E), float("nan"), device="cuda"),
         "sel_id": torch.full((T * k,), -1, dtype=torch.int64, device="cuda"),
         "sel_w": torch.full((T * k,), float("nan"), device="cuda"),
         "offsets": torch.full((E + 1,), -1, dtype=torch.int64, device="cuda"),
         "place": torch.full((T * k,), -1, dtype=torch.int64, device="cuda"),
         "ffn_out": torch.full((T, H), float("nan"), device="cuda")}
    m.layer_dev(layer, dn.data_ptr(), T, dx.data_ptr(), {kk: v.data_ptr() for kk, v in o.items()},
                stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    res = {kk: v.cpu().numpy() for kk, v in o.items()}
    res["x"] = dx.cpu().numpy()
    res["sel_id"] = res["sel_id"].reshape(T, k)
    res["sel_w"] = res["sel_w"].reshape(T, k)
    res["place"] = res["place"].reshape(T, k)
    return res


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_layer_matches_reference_golden(cuda, case):
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    lay, bias, normed, x = build_case(case)
    assert digest(lay, bias, normed, x) == str(g["digest"]), "the synthetic generator changed"
    m = _ctx(case)
    m.set_layer(0, lay, bias)
    for rep in range(2):  # a second call: counters and scratch left clean by the first
        xo = x.copy()
        sid, sw = m.layer(0, normed, xo)
        assert same_bits(sid, g["sel_id"]), rep
        assert same_bits(sw, g["sel_w"]), rep
        assert same_bits(xo, g["x"]), rep
    r = _dev_outputs(cuda, m, 0, normed, x, case["E"], case["k"])
    for key in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out", "x"):
        assert same_bits(r[key], g[key]), key
    m.close()


@pytest.mark.parametrize("gt,dt,rt", [(gb.Q8_0, gb.Q8_0, gb.F32), (gb.Q4_K, gb.Q6_K, gb.BF16),
                                      (gb.Q4_K, gb.Q4_K, gb.BF16), (gb.Q8_0, gb.Q4_K, gb.F32),
                                      (gb.Q4_K, gb.Q8_0, gb.F32), (gb.Q8_0, gb.Q6_K, gb.BF16)])
def test_layer_matches_oracle_fresh_seeds(cuda, oracle, gt, dt, rt):
    rng = np.random.default_rng(gt * 100 + dt)
    lay = gb.make_layer(int(rng.integers(1 << 30)), 64, 2048, 1024, gt, dt, rt, mode="random")
    bias = gb.zipf_bias(3, 64)
    d, keep = make_desc(lay, 2048, 1024, 8, 0, rt, gt, dt, bias)
    m = _ctx(dict(E=64, k=8, H=2048, F=1024, router=rt, gate=gt, down=dt, norm_topk=0, T=16))
    m.set_layer(0, lay, bias)
    for T in (1, 2, 7, 16):
        normed = rng.normal(size=(T, 2048)).astype(np.float32)
        x = rng.normal(size=(T, 2048)).astype(np.float32)
        want = oracle.moe_layer(d, normed, x)
        got = _dev_outputs(cuda, m, 0, normed, x, 64, 8)
        for key in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out", "x"):
            assert same_bits(got[key], want[key]), (T, key)
    m.close()


@pytest.mark.parametrize("gt,dt,rt,T", [(gb.Q4_K, gb.Q6_K, gb.BF16, 2), (gb.Q4_K, gb.Q6_K, gb.BF16, 8),
                                        (gb.Q4_K, gb.Q6_K, gb.BF16, 32), (gb.Q8_0, gb.Q8_0, gb.F32, 1),
                                        (gb.Q8_0, gb.Q8_0, gb.BF16, 8), (gb.Q8_0, gb.Q8_0, gb.F32, 64),
                                        (gb.Q4_K, gb.Q4_K, gb.BF16, 1), (gb.Q4_K, gb.Q4_K, gb.F32, 12)])
def test_short_calls_one_launch_a_token(cuda, oracle, gt, dt, rt, T):
    """Q4_K_M, all-Q4_K and Q8_0 calls of 1..64 tokens (all-Q4_K: below the tensor road's 32) without the dispatch
    permutation run the one-token kernel once a token:
    every output bit for bit the oracle's on the device road, the host road with copies and (up to 16 tokens) the
    zero-copy host road"""
    torch = cuda
    from trochilus_b200.moe import GpuMoe
    lay = gb.make_layer(31 + T + gt, 64, 2048, 1024, gt, dt, rt, mode="random")
    bias = gb.zipf_bias(4, 64)
    d, keep = make_desc(lay, 2048, 1024, 8, 0, rt, gt, dt, bias)
    m = GpuMoe(1, 64, 8, 2048, 1024, rt, gt, dt, max_tokens=T)
    m.set_layer(0, lay, bias)
    assert m.launches(T) == T and m.kernel_name(T) == "trx_k_dec1"
    rng = np.random.default_rng(T)
    normed = rng.normal(size=(T, 2048)).astype(np.float32)
    x = rng.normal(size=(T, 2048)).astype(np.float32)
    want = oracle.moe_layer(d, normed, x)
    for rep in range(2):
        dn = torch.from_numpy(normed).cuda()
        dx = torch.from_numpy(x.copy()).cuda()
        o = {"logits": torch.full((T, 64), float("nan"), device="cuda"),
             "sel_id": torch.full((T * 8,), -1, dtype=torch.int64, device="cuda"),
             "sel_w": torch.full((T * 8,), float("nan"), device="cuda"),
             "ffn_out": torch.full((T, 2048), float("nan"), device="cuda")}
        m.layer_dev(0, dn.data_ptr(), T, dx.data_ptr(), {kk: v.data_ptr() for kk, v in o.items()},
                    stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        m.check()
        got = {kk: v.cpu().numpy() for kk, v in o.items()}
        assert same_bits(got["logits"], want["logits"]), rep
        assert same_bits(got["sel_id"].reshape(T, 8), want["sel_id"]), rep
        assert same_bits(got["sel_w"].reshape(T, 8), want["sel_w"]), rep
        assert same_bits(got["ffn_out"], want["ffn_out"]), rep
        assert same_bits(dx.cpu().numpy(), want["x"]), rep
    xo = x.copy()
    sid, sw = m.layer(0, normed, xo)
    assert same_bits(xo, want["x"]) and same_bits(sid, want["sel_id"]) and same_bits(sw, want["sel_w"])
    hn = torch.from_numpy(normed.copy()).pin_memory()
    hx = torch.from_numpy(x.copy()).pin_memory()
    m.layer_ptrs(0, hn.data_ptr(), T, hx.data_ptr(), host=True)
    assert same_bits(hx.numpy(), want["x"])
    m.close()


def test_many_layers_one_context(cuda, oracle):
    """layers set independently, called in any order, each its own weights"""
    c = dict(E=64, k=8, H=2048, F=1024, router=gb.BF16, gate=gb.Q4_K, down=gb.Q6_K, norm_topk=0, T=3)
    m = _ctx(c, n_layers=3)
    lays = [gb.make_layer(900 + i, 64, 2048, 1024, gb.Q4_K, gb.Q6_K, gb.BF16, mode="random") for i in range(3)]
    for i in (2, 0, 1):
        m.set_layer(i, lays[i])
    rng = np.random.default_rng(1)
    for L in (1, 2, 0, 1):
        normed = rng.normal(size=(3, 2048)).astype(np.float32)
        x = rng.normal(size=(3, 2048)).astype(np.float32)
        d, keep = make_desc(lays[L], 2048, 1024, 8, 0, gb.BF16, gb.Q4_K, gb.Q6_K)
        want = oracle.moe_layer(d, normed, x)
        xo = x.copy()
        sid, sw = m.layer(L, normed, xo)
        assert same_bits(xo, want["x"]) and same_bits(sid, want["sel_id"]), L
    with pytest.raises(RuntimeError):
        m.layer(0, np.zeros((4, 2048), np.float32), np.zeros((4, 2048), np.float32))  # past max_tokens
    m.close()


def test_misaligned_rows_are_refused(cuda):
    """input rows that do not start on a 16-byte boundary (the kernels read them 16 bytes at a time) are refused with
    an error before any launch, and the context keeps working"""
    torch = cuda
    c = dict(E=64, k=8, H=2048, F=1024, router=gb.BF16, gate=gb.Q4_K, down=gb.Q6_K, norm_topk=0, T=2)
    m = _ctx(c)
    m.set_layer(0, gb.make_layer(5, 64, 2048, 1024, gb.Q4_K, gb.Q6_K, gb.BF16, mode="random"))
    dn = torch.zeros((2 * 2048 + 4,), device="cuda")
    dx = torch.zeros((2048,), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(RuntimeError, match="16-byte boundary"):
        m.layer_dev(0, dn.data_ptr() + 4, 1, dx.data_ptr(), None, stream=st)
    m.layer_dev(0, dn.data_ptr(), 1, dx.data_ptr(), None, stream=st)  # aligned: runs
    torch.cuda.synchronize()
    m.check()
    m.close()


def test_unset_layer_is_an_error(cuda):
    c = dict(E=64, k=8, H=2048, F=1024, router=gb.F32, gate=gb.Q8_0, down=gb.Q8_0, norm_topk=0, T=1)
    m = _ctx(c, n_layers=2)
    with pytest.raises(RuntimeError, match="not set"):
        m.layer(1, np.zeros((1, 2048), np.float32), np.zeros((1, 2048), np.float32))
    m.close()


def test_zone_profile_counts_calls(cuda):
    """the zone timer sees every call and gives positive times without changing results"""
    c = dict(E=64, k=8, H=2048, F=1024, router=gb.BF16, gate=gb.Q4_K, down=gb.Q4_K, norm_topk=0, T=2)
    m = _ctx(c)
    m.set_layer(0, gb.make_layer(31, 64, 2048, 1024, gb.Q4_K, gb.Q4_K, gb.BF16, mode="random"))
    rng = np.random.default_rng(0)
    normed = rng.normal(size=(2, 2048)).astype(np.float32)
    x = rng.normal(size=(2, 2048)).astype(np.float32)
    x0 = x.copy()
    m.layer(0, normed, x0)
    m.profile(True)
    for _ in range(5):
        x1 = x.copy()
        m.layer(0, normed, x1)
        assert same_bits(x1, x0)
    z = m.profile_read()
    assert all(z[k][1] == 5 and z[k][0] > 0 for k in ("router", "gate_up", "act_prep", "down")), z
    m.profile(False)
    m.close()


@pytest.mark.parametrize("T", [1, 7, 70])
def test_parts_path_matches_oracle(cuda, oracle, T):
    """tr_gpu_moe_layer_part 0..3 (the multi-kernel road, also the one of passes longer than the fused kernel
    takes) against the oracle, and against the single-call road"""
    gt, dt, rt = gb.Q8_0, gb.Q6_K, gb.F32
    lay = gb.make_layer(600 + T, 16, 512, 256, gt, dt, rt, mode="random")
    d, keep = make_desc(lay, 512, 256, 4, 0, rt, gt, dt)
    from trochilus_b200.moe import GpuMoe
    m = GpuMoe(1, 16, 4, 512, 256, rt, gt, dt, max_tokens=T)
    m.set_layer(0, lay)
    rng = np.random.default_rng(T)
    normed = rng.normal(size=(T, 512)).astype(np.float32)
    x = rng.normal(size=(T, 512)).astype(np.float32)
    want = oracle.moe_layer(d, normed, x)
    dn = cuda.from_numpy(normed).cuda()
    dx = cuda.from_numpy(x.copy()).cuda()
    st = cuda.cuda.current_stream().cuda_stream
    for part in range(4):
        m.layer_part(0, part, dn.data_ptr(), T, dx.data_ptr(), stream=st)
    cuda.cuda.synchronize()
    assert same_bits(dx.cpu().numpy(), want["x"])
    xo = x.copy()
    sid, sw = m.layer(0, normed, xo)
    assert same_bits(xo, want["x"]) and same_bits(sid, want["sel_id"]) and same_bits(sw, want["sel_w"])
    m.check()
    m.close()


def test_q4k_long_pass_multikernel(cuda, oracle):
    """a pass longer than the fused kernel serves (T > 64) on the OLMoE shape, Q4_K experts"""
    T = 72
    lay = gb.make_layer(777, 64, 2048, 1024, gb.Q4_K, gb.Q4_K, gb.BF16, mode="random")
    d, keep = make_desc(lay, 2048, 1024, 8, 0, gb.BF16, gb.Q4_K, gb.Q4_K)
    from trochilus_b200.moe import GpuMoe
    m = GpuMoe(1, 64, 8, 2048, 1024, gb.BF16, gb.Q4_K, gb.Q4_K, max_tokens=T)
    m.set_layer(0, lay)
    m.set_prefill(0)  # the exact road (a Q4_K down takes the tensor road from 32 tokens by default)
    rng = np.random.default_rng(5)
    normed = rng.normal(size=(T, 2048)).astype(np.float32)
    x = rng.normal(size=(T, 2048)).astype(np.float32)
    want = oracle.moe_layer(d, normed, x)
    xo = x.copy()
    sid, sw = m.layer(0, normed, xo)
    assert same_bits(sid, want["sel_id"]) and same_bits(sw, want["sel_w"])
    assert same_bits(xo, want["x"])
    m.close()


@pytest.mark.parametrize("gt,dt,rt", [(gb.Q4_K, gb.Q6_K, gb.BF16), (gb.Q8_0, gb.Q8_0, gb.F32)])
def test_host_call_on_pinned_x(cuda, oracle, gt, dt, rt):
    """tr_gpu_moe_layer with x in pinned host memory: short calls take the zero-copy road (x read and written in
    place through its mapping, completion posted to a pinned word), longer ones the copy road; both bit for bit the
    oracle's, call after call on the same buffers, normed pinned or pageable"""
    torch = cuda
    rng = np.random.default_rng(77 + gt)
    lay = gb.make_layer(int(rng.integers(1 << 30)), 64, 2048, 1024, gt, dt, rt, mode="random")
    d, keep = make_desc(lay, 2048, 1024, 8, 0, rt, gt, dt)
    m = _ctx(dict(E=64, k=8, H=2048, F=1024, router=rt, gate=gt, down=dt, norm_topk=0, T=24))
    m.set_layer(0, lay)
    for T in (1, 3, 16, 24, 1):
        normed = rng.normal(size=(T, 2048)).astype(np.float32)
        x = rng.normal(size=(T, 2048)).astype(np.float32)
        want = oracle.moe_layer(d, normed, x)
        hn = torch.from_numpy(normed).pin_memory()
        hx = torch.from_numpy(x.copy()).pin_memory()
        for rep in range(2):  # the second call adds the layer to the first call's output
            m.layer_ptrs(0, hn.data_ptr(), T, hx.data_ptr(), host=True)
            if rep == 0:
                assert same_bits(hx.numpy(), want["x"]), (T, rep)
        want2 = oracle.moe_layer(d, normed, want["x"])
        assert same_bits(hx.numpy(), want2["x"]), T
        # normed in pageable memory (copied by the copy engine), x still pinned
        hx.copy_(torch.from_numpy(x))
        m.layer_ptrs(0, normed.ctypes.data, T, hx.data_ptr(), host=True)
        assert same_bits(hx.numpy(), want["x"]), (T, "pageable normed")
    m.check()
    m.close()



def test_kernel_binary_is_sm100(cuda):
    """the runtime's own report for the fused decode kernel: native sm_100 code (binaryVersion 100), no JIT"""
    from trochilus_b200 import moe
    assert moe.lib().trmoe_kernel_arch() == 100, moe.last_error()
