"""tr_matmul_q4k_noalloc through the C ABI: the Q4_K product on caller-owned device memory with the library's fixed
scratch array, bit for bit the result of the existing entry point tr_matmul on the same weights and inputs, on two
calls in a row (the second with other inputs and fewer tokens, so a stale scratch would show), the size limit
rejected with an error, and no device memory taken by further calls. Collected last; passes alone in a fresh process
or after the other tests."""
import ctypes as C

import numpy as np
import pytest

from tests.golden.cases import same_bits
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, w_dev, rows, cols, x_dev, n_tok, y_dev):
    return lib.tr_matmul_q4k_noalloc(C.c_void_p(w_dev.data_ptr()), rows, cols, C.c_void_p(x_dev.data_ptr()), n_tok,
                                     C.c_void_p(y_dev.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_tr_matmul_on_two_calls(cuda):
    torch = cuda
    from trochilus_b200 import moe
    lib = moe.lib()
    rows, cols = 1024, 2048
    rng = np.random.default_rng(20261201)
    w = np.ascontiguousarray(gb.random_blocks(gb.Q4_K, rows, cols, rng))
    w_dev = torch.from_numpy(w).to("cuda")
    for n_tok in (9, 4):
        x = rng.normal(size=(n_tok, cols)).astype(np.float32)
        moe.kernel_cache_clear()
        want = moe.matmul(gb.Q4_K, rows, cols, w, x)  # the existing entry point, host arrays
        x_dev = torch.from_numpy(x).to("cuda")
        y_dev = torch.full((n_tok, rows), float("nan"), device="cuda")
        rc = _noalloc(lib, torch, w_dev, rows, cols, x_dev, n_tok, y_dev)
        assert rc == 0, moe.last_error()
        torch.cuda.synchronize()
        got = y_dev.cpu().numpy()
        assert same_bits(got, want), np.argwhere(~((got == want) | (np.isnan(got) & np.isnan(want))))[:5]


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    torch = cuda
    from trochilus_b200 import moe
    lib = moe.lib()
    rows, cols, n_tok = 8, 2048, 479  # 478 tokens of 2048 columns fit the 4 MiB scratch
    w_dev = torch.zeros((rows, cols // 256 * 144), dtype=torch.uint8, device="cuda")
    x_dev = torch.zeros((n_tok, cols), device="cuda")
    y_dev = torch.zeros((n_tok, rows), device="cuda")
    assert _noalloc(lib, torch, w_dev, rows, cols, x_dev, n_tok, y_dev) == -1
    assert "more than its 4194304" in moe.last_error()
    assert _noalloc(lib, torch, w_dev, rows, cols, x_dev, 478, y_dev) == 0, moe.last_error()
    torch.cuda.synchronize()


def test_noalloc_allocates_nothing(cuda):
    """the entry point's promise: after a first call on the device (which may load the library's device code), more
    calls change neither the device's free memory (cudaMemGetInfo) nor what torch's allocator holds"""
    torch = cuda
    from trochilus_b200 import moe
    lib = moe.lib()
    rows, cols, n_tok = 1024, 2048, 16
    rng = np.random.default_rng(7)
    w_dev = torch.from_numpy(np.ascontiguousarray(gb.random_blocks(gb.Q4_K, rows, cols, rng))).to("cuda")
    xs = [torch.from_numpy(rng.normal(size=(n_tok, cols)).astype(np.float32)).to("cuda") for _ in range(3)]
    y_dev = torch.zeros((n_tok, rows), device="cuda")
    assert _noalloc(lib, torch, w_dev, rows, cols, xs[0], n_tok, y_dev) == 0, moe.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    held0 = torch.cuda.memory_reserved()
    for x_dev in xs[1:] + xs[:1]:
        assert _noalloc(lib, torch, w_dev, rows, cols, x_dev, n_tok, y_dev) == 0, moe.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_reserved() == held0
