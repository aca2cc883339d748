"""libtrmoe.so from C on the GPU: tests/c/abi_test.c's GPU part, one MoE layer of three tokens through
tr_gpu_moe_layer, bit for bit the C oracle's orc_moe_layer (ids, weights and x)."""
import subprocess

import pytest

from tests.test_c_abi import build_abi_test

pytestmark = pytest.mark.gpu


def test_c_abi_layer_on_gpu(cuda, tmp_path):
    exe = build_abi_test(tmp_path)
    out = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip() == "gpu ok", (out.returncode, out.stdout, out.stderr)
