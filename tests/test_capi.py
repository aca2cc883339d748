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


def test_library_is_built_for_sm100a_only():
    """the build names sm_100a alone (no PTX for a JIT to fall back on); on a device the runtime's own report of the
    fused kernel's binary version is checked (test_gpu_layer.py::test_kernel_binary_is_sm100); without one the query
    is an error with a message, not a crash"""
    from trochilus_b200 import build, moe
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert moe.lib().trmoe_kernel_arch() == -1 and moe.last_error()


def test_failed_void_calls_poison_their_outputs():
    """the reference's kernel API is void, so a failure cannot be returned: every output float is set to NaN (a
    refused type here, and with no device here every call fails at its first CUDA call) and TRMOE_ABORT_ON_ERROR=1
    ends the process instead"""
    import numpy as np
    from trochilus_b200 import moe
    L = moe.lib()
    w = np.zeros((16, 34 * 16), dtype=np.uint8)
    x = np.ones((3, 512), dtype=np.float32)
    for typ in (99, moe.Q8_0):  # a type the library does not take; a good call that finds no device
        y = np.zeros((3, 16), dtype=np.float32)
        L.tr_matmul(None, C.byref(moe.TrMat(typ, 16, 512, w.ctypes.data)), x.ctypes.data, 3, y.ctypes.data)
        assert np.isnan(y).all(), typ
        assert moe.last_error()
    v = np.ones(64, dtype=np.float32)
    L.tr_softmax(v.ctypes.data, 64)
    assert np.isnan(v).all()
    v = np.ones(64, dtype=np.float32)
    L.tr_swiglu(None, v.ctypes.data, np.ones(64, dtype=np.float32).ctypes.data, 64)
    assert np.isnan(v).all()
    code = ("import ctypes as C, numpy as np\nfrom trochilus_b200 import moe\n"
            "v = np.ones(8, dtype=np.float32)\nmoe.lib().tr_softmax(v.ctypes.data, 8)\nprint('survived')\n")
    r = subprocess.run([__import__("sys").executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       env={**os.environ, "TRMOE_ABORT_ON_ERROR": "1"})
    assert r.returncode != 0 and "survived" not in r.stdout and "aborting" in r.stderr


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


def test_prepared_road_host_logic_without_gpu():
    """Q4_K's prepared road (tr_q4x_road, tr_q4x_bytes, tr_q4x_prepare, and the refusals of
    tr_matmul_q4x_prepared(_n)) answers on the host: which weights it takes, the slot size (the reference's
    tr_q4x_bytes, src/kernels/kernels.c:489-492), where a prepared row's floats go, and a refused call leaves y
    untouched and returns 0 (an empty call returns 1)."""
    import numpy as np
    from trochilus_b200 import moe
    L = moe.lib()
    assert [moe.q4x_bytes(n) for n in (256, 512, 1024, 2048)] == [1152, 2304, 4544, 9024]
    assert moe.q4x_road(moe.Q4_K, 1024, 2048) == 1 and moe.q4x_road(moe.Q4_K, 2048, 1024) == 1
    assert moe.q4x_road(moe.Q8_0, 1024, 2048) == 0 and moe.q4x_road(moe.Q6_K, 2048, 1024) == 0
    assert moe.q4x_road(moe.Q4_K, 1000, 2048) == 0 and moe.q4x_road(moe.Q4_K, 1024, 2000) == 0
    x = np.random.default_rng(0).normal(size=(3, 512)).astype(np.float32)
    xq = moe.q4x_prepare(x)
    sl = moe.q4x_bytes(512)
    assert xq.size == 3 * sl
    for r in range(3):
        assert np.array_equal(xq[r * sl:r * sl + 2048].view(np.float32), x[r])
        assert not xq[r * sl + 2048:(r + 1) * sl].any()  # the rest of a slot is not written
    off = np.array([0, 2, 3], dtype=np.int64)
    w = np.zeros((16, 34 * 16), dtype=np.uint8)
    q8 = (moe.TrMat * 2)(moe.TrMat(moe.Q8_0, 16, 512, w.ctypes.data), moe.TrMat(moe.Q8_0, 16, 512, w.ctypes.data))
    y = np.full((3, 16), np.nan, dtype=np.float32)
    assert L.tr_matmul_q4x_prepared(None, q8, off.ctypes.data, 2, xq.ctypes.data, None, y.ctypes.data, None) == 0
    assert np.isnan(y).all()
    empty = np.array([0, 0, 0], dtype=np.int64)
    assert L.tr_matmul_q4x_prepared(None, q8, empty.ctypes.data, 2, xq.ctypes.data, None, y.ctypes.data, None) == 1
    w4 = np.zeros((16, 144 * 2), dtype=np.uint8)
    a = (moe.TrMat * 2)(*[moe.TrMat(moe.Q4_K, 16, 512, w4.ctypes.data)] * 2)
    b = (moe.TrMat * 2)(*[moe.TrMat(moe.Q4_K, 32, 512, w4.ctypes.data)] * 2)
    wp = (C.c_void_p * 4)(C.cast(a, C.c_void_p), C.cast(b, C.c_void_p), C.cast(a, C.c_void_p), C.cast(a, C.c_void_p))
    yp = (C.c_void_p * 4)(*[y.ctypes.data] * 4)
    before = moe.q4x_fused_calls()
    for n_w in (0, 2, 4):  # out of range, shapes that differ, out of range
        assert L.tr_matmul_q4x_prepared_n(None, wp, n_w, off.ctypes.data, 2, xq.ctypes.data, None, yp, None) == 0
    assert np.isnan(y).all() and moe.q4x_fused_calls() == before


def test_attention_host_logic_without_gpu():
    """the GPU attention backend's host side (src/backend/gpu_attn.h's conventions): no device is an error with a
    message, a shape the kernels do not take is refused before any device call, a missing session is an error,
    and the bytes a session takes"""
    import ctypes as C
    from trochilus_b200 import moe
    L = moe.lib()
    err = C.create_string_buffer(256)
    assert not L.tr_gpu_open(err, 256) and b"device" in err.value  # this container has no GPU
    assert not L.tr_gpu_attn_create(None, 2, 4, 64, 16, err, 256) and b"head_dim 64 not supported" in err.value
    assert not L.tr_gpu_attn_create(None, 2, 4, 128, 0, err, 256) and b"bad shape" in err.value
    assert not L.tr_gpu_attn_create(None, 2, 4, 128, 16, err, 256) and b"no device" in err.value
    assert L.tr_gpu_attn_decode(None, 0, 0, None, None, None, 1.0, None) == -1 and "bad arguments" in moe.last_error()
    assert L.tr_gpu_attn_write(None, 0, 0, 1, None, None) == -1
    cache = 2 * 16 * 16 * 4096 * 128 * 4
    assert cache < L.tr_gpu_attn_bytes(16, 16, 128, 4096) < cache + (8 << 20)
    assert L.tr_gpu_attn_bytes(0, 16, 128, 4096) == 0
    L.tr_gpu_close(None)
    L.tr_gpu_attn_free(None)
