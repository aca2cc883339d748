"""The C ABI without a GPU: libtrmoe.so loads and exports every function include/trmoe.h declares, and the
pure host logic (sizes, argument checks) answers without touching a device."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while")))


def test_library_builds_and_exports_every_declared_symbol():
    from trochilus_b200 import build, moe
    build.build()
    lib = moe.lib()
    declared = declared_functions()
    assert len(declared) >= 14
    out = subprocess.check_output(["nm", "-D", "--defined-only", moe.LIB_PATH], text=True)
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in declared if n not in exported]
    assert not missing, missing
    assert set(moe.EXPORTS) == set(declared)
    for n in declared:
        getattr(lib, n)


def test_library_is_sm100a():
    from trochilus_b200 import moe
    out = subprocess.check_output(["/usr/local/cuda/bin/cuobjdump", "--list-elf", moe.LIB_PATH], text=True)
    assert "sm_100a" in out


def test_bytes_and_config_checks_without_gpu():
    from trochilus_b200 import moe
    n = moe.GpuMoe.bytes_needed(n_layers=16, n_expert=64, n_used=8, n_embd=2048, n_ff=1024, router_type=moe.BF16,
                                gate_type=moe.Q4_K, down_type=moe.Q6_K, max_tokens=1)
    per_layer = 64 * (2 * 1024 * 1152 + 2048 * 840) + 64 * 2048 * 2
    assert per_layer * 16 <= n < per_layer * 16 + 64 << 20
    with pytest.raises(RuntimeError, match="not supported"):
        moe.GpuMoe(1, 64, 8, 2048, 1024, moe.Q8_0, moe.Q4_K, moe.Q6_K, 1)
    with pytest.raises(RuntimeError, match="unsupported counts"):
        moe.GpuMoe(1, 65, 8, 2048, 1024, moe.F32, moe.Q4_K, moe.Q6_K, 1)
    with pytest.raises(RuntimeError, match="n_embd 2048"):
        moe.GpuMoe(1, 64, 8, 1024, 1024, moe.F32, moe.Q4_K, moe.Q6_K, 1)
