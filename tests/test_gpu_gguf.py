"""The model loader on the GPU (tr_gpu_moe_config_from_gguf, tr_gpu_moe_load_gguf): a context made from an OLMoE GGUF
file and loaded from it (every layer's router, expert slices and ffn_norm, src/models/olmoe.c:541-641, 895-906),
then each layer's call bit for bit the oracle's on the arrays the file was written from."""
import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.gguf_fixture import write_olmoe_moe
from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu


def test_small_model_every_layer(cuda, oracle, tmp_path):
    """two layers of a small shape (experts of each layer at their slices of the stacked tensors)"""
    from trochilus_b200.moe import GpuMoe
    E, K, H, F = 16, 4, 512, 256
    lays = [gb.make_layer(900 + L, E, H, F, gb.Q8_0, gb.Q6_K, gb.F32, mode="random") for L in range(2)]
    norms = [(1.0 + 0.1 * np.random.default_rng(L).normal(size=H)).astype(np.float32) for L in range(2)]
    p = write_olmoe_moe(tmp_path / "small.gguf", lays, norms, n_used=K)
    m = GpuMoe.from_gguf(str(p), max_tokens=5)
    assert (m.cfg.n_layers, m.cfg.n_expert, m.cfg.n_used, m.cfg.router_type) == (2, E, K, gb.F32)
    rng = np.random.default_rng(3)
    for L in range(2):
        d, keep = make_desc(lays[L], H, F, K, 0, gb.F32, gb.Q8_0, gb.Q6_K)
        for T in (1, 5):
            normed = rng.normal(size=(T, H)).astype(np.float32)
            x = rng.normal(size=(T, H)).astype(np.float32)
            want = oracle.moe_layer(d, normed, x)
            got = x.copy()
            sid, sw = m.layer(L, normed, got)
            assert same_bits(got, want["x"]) and same_bits(sid, want["sel_id"]), (L, T)
    m.check()
    m.close()


def test_olmoe_layer_with_ffn_norm(cuda, oracle, tmp_path):
    """the OLMoE shape (Q4_K_M experts), an F32 router of bfloat16 values (narrowed to BF16 on load) and the layer's
    ffn_norm with the file's epsilon: tr_gpu_moe_ffn against the oracle's rmsnorm and layer"""
    from trochilus_b200.moe import GpuMoe
    E, K, H, F = 64, 8, 2048, 1024
    lay = gb.make_layer(77, E, H, F, gb.Q4_K, gb.Q6_K, gb.BF16, mode="random")  # the router's values are bf16
    r = gb.round_to_bf16(np.random.default_rng(5).normal(0, 0.02, size=(E, H)).astype(np.float32))
    lay["router"] = gb.quantize(gb.BF16, r)
    as_f32 = dict(lay, router=gb.quantize(gb.F32, r))  # the file holds it as F32
    wn = (1.0 + 0.1 * np.random.default_rng(6).normal(size=H)).astype(np.float32)
    p = write_olmoe_moe(tmp_path / "olmoe.gguf", [as_f32], [wn], eps=1e-5, n_used=K, gate_type=gb.Q4_K,
                        down_type=gb.Q6_K)
    m = GpuMoe.from_gguf(str(p), max_tokens=3)
    assert m.cfg.router_type == gb.BF16
    d, keep = make_desc(lay, H, F, K, 0, gb.BF16, gb.Q4_K, gb.Q6_K)
    rng = np.random.default_rng(8)
    for T in (1, 3):
        x = (rng.normal(size=(T, H)) * 2).astype(np.float32)
        want = oracle.moe_layer(d, oracle.rmsnorm(x, wn, np.float32(1e-5)), x)
        got = x.copy()
        m.ffn(0, got)
        assert same_bits(got, want["x"]), T
    m.check()
    m.close()
