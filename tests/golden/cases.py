"""The golden cases: each a seeded MoE-layer configuration whose inputs and weights are regenerated
from the seed by trochilus_b200.gguf_blocks (deterministic numpy PCG64) and whose outputs were produced
by Trochilus's own code (oracle/_ref) by gen_golden.py. Shared by the generator and the tests."""
from __future__ import annotations

import hashlib

import numpy as np

from trochilus_b200 import gguf_blocks as gb

CASES = [
    # name, seed, E, k, H, F, router, gate, down, T, weight mode, special, zipf bias, norm_topk, input kind
    dict(name="q8_0_t1", seed=11, E=64, k=8, H=2048, F=1024, router=gb.F32, gate=gb.Q8_0, down=gb.Q8_0, T=1,
         mode="random", special=False, zipf=False, norm_topk=0, inputs="normal"),
    dict(name="q4km_bf16_t4", seed=12, E=64, k=8, H=2048, F=1024, router=gb.BF16, gate=gb.Q4_K, down=gb.Q6_K, T=4,
         mode="random", special=False, zipf=False, norm_topk=0, inputs="normal"),
    dict(name="q4k_zipf_special_t8", seed=13, E=64, k=8, H=2048, F=1024, router=gb.F32, gate=gb.Q4_K, down=gb.Q4_K,
         T=8, mode="random", special=True, zipf=True, norm_topk=0, inputs="normal"),
    dict(name="small_q8_normal_t5", seed=14, E=16, k=4, H=512, F=256, router=gb.F32, gate=gb.Q8_0, down=gb.Q6_K, T=5,
         mode="normal", special=False, zipf=False, norm_topk=0, inputs="normal"),
    dict(name="q8q6_normtopk_t2", seed=15, E=64, k=8, H=2048, F=1024, router=gb.F32, gate=gb.Q8_0, down=gb.Q6_K, T=2,
         mode="random", special=False, zipf=False, norm_topk=1, inputs="normal"),
    dict(name="q4k_witness_inputs_t6", seed=16, E=64, k=8, H=2048, F=1024, router=gb.F32, gate=gb.Q4_K,
         down=gb.Q4_K, T=6, mode="random", special=False, zipf=False, norm_topk=0, inputs="witness"),
    dict(name="q8_0_t64", seed=17, E=64, k=8, H=2048, F=1024, router=gb.BF16, gate=gb.Q8_0, down=gb.Q8_0, T=64,
         mode="random", special=False, zipf=True, norm_topk=0, inputs="normal"),
]


def witness_inputs(rng, T, H):
    """The reference's witness rows (Trochilus tests/test_kernels.c:367-377): a zero row, subnormals, one
    huge value, a block whose largest |x| is just under a power of two, a NaN, an infinity."""
    x = rng.normal(size=(T, H)).astype(np.float32)
    x[0] = 0.0
    if T > 1:
        x[1] = np.ldexp(rng.uniform(-1, 1, size=H), -140).astype(np.float32)
    if T > 2:
        x[2, 5] = 1.0e30
    if T > 3:
        x[3] = (0.79 * rng.uniform(-1, 1, size=H)).astype(np.float32)
        x[3, 17] = -7.99
    if T > 4:
        x[4, min(300, H - 1)] = np.nan
    if T > 5:
        x[5, min(1000, H - 1)] = np.inf
    return x


def build_case(c):
    """(layer dict, bias or None, normed, x) of a case."""
    lay = gb.make_layer(c["seed"], c["E"], c["H"], c["F"], c["gate"], c["down"], c["router"], mode=c["mode"],
                        special=c["special"])
    bias = gb.zipf_bias(c["seed"] + 1000, c["E"]) if c["zipf"] else None
    rng = np.random.Generator(np.random.PCG64(c["seed"] + 2000))
    if c["inputs"] == "witness":
        normed = witness_inputs(rng, c["T"], c["H"])
    else:
        normed = rng.normal(size=(c["T"], c["H"])).astype(np.float32)
    x = rng.normal(size=(c["T"], c["H"])).astype(np.float32)
    return lay, bias, normed, x


def digest(lay, bias, normed, x) -> str:
    h = hashlib.sha256()
    h.update(lay["router"].tobytes())
    for n in ("gate", "up", "down"):
        for m in lay[n]:
            h.update(m.tobytes())
    if bias is not None:
        h.update(bias.tobytes())
    h.update(normed.tobytes())
    h.update(x.tobytes())
    return h.hexdigest()


def same_bits(a, b) -> bool:
    """Bit equality, a NaN equal to any NaN (the reference allows the payload to differ)."""
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype.kind == "f":
        nan = np.isnan(a) & np.isnan(b)
        ua = a.view(np.uint32 if a.dtype == np.float32 else np.uint64)
        ub = b.view(np.uint32 if b.dtype == np.float32 else np.uint64)
        return bool(np.all((ua == ub) | nan))
    return bool(np.array_equal(a, b))
