"""The full-model greedy-token check: Trochilus's own engine (oracle/_ref/trochilus, compiled from the reference's
sources, unmodified) against the same objects relinked onto libtrmoe.so's kernel level (oracle/_ref/trochilus_trmoe:
-Wl,--wrap for every kernel-level name the library replaces, oracle/trmoe_wrap.c). Both run with TR_GPU=0, so the
reference's own GPU attention stays off and the only difference is where the matmuls, softmax and SwiGLU run.

As the reference's own GPU gate does (tools/gpu_exact.sh: the whole engine with and without its GPU, outputs
compared by SHA-256, and a `gpu:` line proving the GPU ran), each case asserts
  - the greedy tokens of `generate --tokens <seeded prompt> -n <N>` are identical,
  - the logits of `logits --tokens <prompt> --out <file>` are identical byte for byte (SHA-256),
  - the wrapped run printed `gpu: libtrmoe.so on <device>, <n> kernel-level calls` with n > 0.
The models are written here by tests/gguf_fixture.py (seeded, OLMoE-1B-7B architecture) and deleted afterwards."""
import hashlib
import os
import re
import subprocess

import numpy as np
import pytest

from tests.gguf_fixture import write_olmoe_model
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PLAIN = os.path.join(ROOT, "oracle", "_ref", "trochilus")
WRAPPED = os.path.join(ROOT, "oracle", "_ref", "trochilus_trmoe")


def _engines():
    if not (os.path.exists(PLAIN) and os.path.exists(WRAPPED)):
        pytest.skip("oracle/_ref holds no engine build (make -C oracle REF=<reference tree> engine builds it)")


def _run(binary, args, timeout):
    env = {**os.environ, "TR_GPU": "0", "TR_SERVER": "0", "TRMOE_LIB": os.path.join(ROOT, "trochilus_b200", "libtrmoe.so")}
    r = subprocess.run([binary, *args], capture_output=True, text=True, env=env, timeout=timeout)
    assert r.returncode == 0, (binary, r.returncode, r.stderr[-2000:])
    return r


def _tokens(stdout):
    m = re.search(r"^tokens:(.*)$", stdout, flags=re.M)
    assert m, stdout[-500:]
    return [int(v) for v in m.group(1).split(",") if v.strip()]


def _gpu_line(stderr):
    m = re.search(r"^gpu: libtrmoe\.so on (.+), (\d+) kernel-level calls$", stderr, flags=re.M)
    assert m, stderr[-1000:]
    return m.group(1), int(m.group(2))


def _check(tmp_path, model, prompt, n_gen, timeout):
    ids = ",".join(str(int(v)) for v in prompt)
    gen = ["generate", "-m", str(model), "--tokens", ids, "-n", str(n_gen)]
    want = _run(PLAIN, gen, timeout)
    got = _run(WRAPPED, gen, timeout)
    device, calls = _gpu_line(got.stderr)
    t_want, t_got = _tokens(want.stdout), _tokens(got.stdout)
    print(f"{model.name}: {len(t_want)} greedy tokens, wrapped run on {device} with {calls} kernel-level calls")
    assert len(t_want) == n_gen and t_got == t_want
    assert "B200" in device and calls > 0
    assert len(set(t_want)) > 1  # the tokens move: the check is not of a constant output
    digests = []
    for binary, name in ((PLAIN, "plain"), (WRAPPED, "wrapped")):
        out = tmp_path / f"logits_{name}.bin"
        _run(binary, ["logits", "-m", str(model), "--tokens", ids, "--out", str(out)], timeout)
        data = out.read_bytes()
        assert len(data) >= 4 * len(prompt) * 50304
        digests.append(hashlib.sha256(data).hexdigest())
        out.unlink()
    print(f"{model.name}: logits sha256 {digests[0]} (plain) {digests[1]} (wrapped)")
    assert digests[0] == digests[1]


def test_configs0_two_layer_q8_0_tokens_identical(cuda, tmp_path):
    """2 layers, Q8_0 weights N(0, 0.02), norms 1, a 128-token seeded uniform prompt, 32 greedy steps"""
    _engines()
    model = write_olmoe_model(tmp_path / "olmoe_cfg0_q8_0.gguf", 2, seed=20260)
    prompt = np.random.default_rng(128).integers(0, 50304, size=128)
    try:
        _check(tmp_path, model, prompt, 32, timeout=900)
    finally:
        model.unlink()


def test_configs1_sixteen_layer_q4_k_m_tokens_identical(cuda, tmp_path):
    """the 16-layer architecture, Q4_K experts and attention, Q6_K down and output head (the experts
    random-init quant blocks, the dense matrices N(0, 0.02) quantized), a 512-token seeded uniform prompt, 256 greedy
    steps"""
    _engines()
    model = write_olmoe_model(tmp_path / "olmoe_cfg1_q4km.gguf", 16, seed=20261, attn_type=gb.Q4_K,
                              gate_type=gb.Q4_K, down_type=gb.Q6_K, embd_type=gb.Q4_K, head_type=gb.Q6_K,
                              mode="random")
    prompt = np.random.default_rng(512).integers(0, 50304, size=512)
    try:
        _check(tmp_path, model, prompt, 256, timeout=1800)
    finally:
        model.unlink()
