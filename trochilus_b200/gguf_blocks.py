"""GGUF block encoders and seeded synthetic OLMoE MoE-layer weights.

The benchmark configurations name random-init OLMoE weights, N(0, 0.02), quantized to Q8_0, Q4_K
or Q6_K (GGUF block layouts as in Trochilus src/kernels/kernels_internal.h:12-217 and ggml). These
encoders are this project's own: any valid encoder will do, because every parity check runs the
reference and this library on the same bytes. Two generators:

  quantize_*   N(0, sigma) floats encoded the usual way (per-block absmax / min-scale fits);
  random_*     uniformly random quants with bounded f16 scales (fast, and every code appears),
               optionally with special scale values (0, subnormal, negative, large) mixed in.

Deterministic given the seed (numpy PCG64).
"""
from __future__ import annotations

import numpy as np

F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def row_bytes(type_: int, n: int) -> int:
    if type_ == F32:
        return 4 * n
    if type_ in (F16, BF16):
        return 2 * n
    be, bb = BLOCK[type_]
    assert n % be == 0
    return n // be * bb


# ---------------------------------------------------------------- encoders from floats

def _f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """rows x cols float32 -> rows x row_bytes uint8 (Q8_0)."""
    rows, cols = w.shape
    b = w.reshape(rows, cols // 32, 32).astype(np.float32)
    amax = np.abs(b).max(axis=2)
    d = _f16(amax / 127.0)
    df = d.astype(np.float32)
    inv = np.where(df > 0, 1.0 / np.where(df > 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.rint(b * inv[..., None]), -127, 127).astype(np.int8)
    out = np.empty((rows, cols // 32, 34), dtype=np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(rows, cols // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def _pack_q4k_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """sc, m: (..., 8) ints 0..63 -> (..., 12) bytes in ggml's packing."""
    s = np.zeros(sc.shape[:-1] + (12,), dtype=np.uint8)
    for j in range(4):
        s[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        s[..., j + 4] = (m[..., j] & 63) | ((m[..., j + 4] >> 4) << 6)
        s[..., j + 8] = (sc[..., j + 4] & 15) | ((m[..., j + 4] & 15) << 4)
    return s


def _pack_q4k_quants(q: np.ndarray) -> np.ndarray:
    """q: (..., 256) ints 0..15 -> (..., 128) bytes: byte 32c + i = q[64c + i] | q[64c + 32 + i] << 4."""
    q = q.reshape(q.shape[:-1] + (4, 2, 32)).astype(np.uint8)
    return (q[..., 0, :] | (q[..., 1, :] << 4)).reshape(q.shape[:-3] + (128,))


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    rows, cols = w.shape
    nb = cols // 256
    x = w.reshape(rows, nb, 8, 32).astype(np.float32)
    mn = np.minimum(x.min(axis=3), 0.0)
    mx = x.max(axis=3)
    scale = (mx - mn) / 15.0
    minv = -mn
    d = _f16(scale.max(axis=2) / 63.0)
    dmin = _f16(minv.max(axis=2) / 63.0)
    df, dmf = d.astype(np.float32), dmin.astype(np.float32)
    sc = np.clip(np.rint(np.where(df[..., None] > 0, scale / np.where(df[..., None] > 0, df[..., None], 1), 0)), 0, 63)
    m = np.clip(np.rint(np.where(dmf[..., None] > 0, minv / np.where(dmf[..., None] > 0, dmf[..., None], 1), 0)), 0, 63)
    sc, m = sc.astype(np.int64), m.astype(np.int64)
    step = df[..., None] * sc
    off = dmf[..., None] * m
    q = np.where(step[..., None] > 0, np.rint((x + off[..., None]) / np.where(step[..., None] > 0, step[..., None], 1)), 0)
    q = np.clip(q, 0, 15).astype(np.int64).reshape(rows, nb, 256)
    out = np.empty((rows, nb, 144), dtype=np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:4] = dmin.view(np.uint8).reshape(rows, nb, 2)
    out[..., 4:16] = _pack_q4k_scales(sc, m)
    out[..., 16:] = _pack_q4k_quants(q)
    return out.reshape(rows, -1)


def _pack_q6k(q: np.ndarray):
    """q: (..., 256) ints 0..63 -> ql (..., 128), qh (..., 64) in ggml's layout: element i = 128h + 32c + l
    takes nibble (c >> 1) of ql[64h + 32(c & 1) + l] and bits 2c of qh[32h + l]."""
    q = q.reshape(q.shape[:-1] + (2, 4, 32)).astype(np.uint8)  # h, c, l
    lo, hi = q & 15, q >> 4
    ql = np.empty(q.shape[:-3] + (2, 2, 32), dtype=np.uint8)
    ql[..., 0, :] = lo[..., 0, :] | (lo[..., 2, :] << 4)
    ql[..., 1, :] = lo[..., 1, :] | (lo[..., 3, :] << 4)
    qh = hi[..., 0, :] | (hi[..., 1, :] << 2) | (hi[..., 2, :] << 4) | (hi[..., 3, :] << 6)
    return ql.reshape(q.shape[:-3] + (128,)), qh.reshape(q.shape[:-3] + (64,))


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    rows, cols = w.shape
    nb = cols // 256
    x = w.reshape(rows, nb, 16, 16).astype(np.float32)
    amax = np.abs(x).max(axis=3)
    scale = amax / 31.0
    d = _f16(scale.max(axis=2) / 127.0)
    df = d.astype(np.float32)
    sc = np.clip(np.rint(np.where(df[..., None] > 0, scale / np.where(df[..., None] > 0, df[..., None], 1), 0)), -128,
                 127).astype(np.int64)
    step = df[..., None] * sc
    q = np.where(step[..., None] != 0, np.rint(x / np.where(step[..., None] != 0, step[..., None], 1)), 0)
    q = (np.clip(q, -32, 31) + 32).astype(np.int64).reshape(rows, nb, 256)
    ql, qh = _pack_q6k(q)
    out = np.empty((rows, nb, 210), dtype=np.uint8)
    out[..., 0:128] = ql
    out[..., 128:192] = qh
    out[..., 192:208] = sc.astype(np.int8).view(np.uint8)
    out[..., 208:210] = d.view(np.uint8).reshape(rows, nb, 2)
    return out.reshape(rows, -1)


def quantize(type_: int, w: np.ndarray) -> np.ndarray:
    if type_ == Q8_0:
        return quantize_q8_0(w)
    if type_ == Q4_K:
        return quantize_q4_k(w)
    if type_ == Q6_K:
        return quantize_q6_k(w)
    if type_ == F32:
        return np.ascontiguousarray(w, dtype=np.float32).view(np.uint8).reshape(w.shape[0], -1)
    if type_ == BF16:
        return to_bf16_exact(w).view(np.uint8).reshape(w.shape[0], -1)
    raise ValueError(type_)


def round_to_bf16(w: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (ties to even), still float32 (low halves zero)."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.view(np.float32)


def to_bf16_exact(w: np.ndarray) -> np.ndarray:
    """float32 whose low halves are zero -> uint16 bfloat16 (Trochilus tr_f32_to_bf16_exact)."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    assert not np.any(u & 0xFFFF), "values do not fit bfloat16 exactly"
    return (u >> 16).astype(np.uint16)


# ---------------------------------------------------------------- random blocks

def _rand_f16(rng, shape, lo, hi):
    return _f16(rng.uniform(lo, hi, size=shape))


def random_blocks(type_: int, rows: int, cols: int, rng: np.random.Generator, special: bool = False) -> np.ndarray:
    """rows x row_bytes uint8 of uniformly random quants with bounded scales. special: some scales are
    0, subnormal, negative or large."""
    rb = row_bytes(type_, cols)
    out = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
    be, bb = BLOCK[type_]
    nb = cols // be
    blk = out.reshape(rows, nb, bb)

    def put(off, vals):
        blk[..., off:off + 2] = vals.view(np.uint8).reshape(rows, nb, 2)

    if type_ == Q8_0:
        d = _rand_f16(rng, (rows, nb), 1e-4, 4e-4)
    elif type_ == Q4_K:
        d = _rand_f16(rng, (rows, nb), 2e-5, 1e-4)
        dm = _rand_f16(rng, (rows, nb), 1e-4, 5e-4)
    else:
        d = _rand_f16(rng, (rows, nb), 2e-5, 8e-5)
    if special:
        pick = rng.integers(0, 16, size=(rows, nb))
        sp = np.array([0.0, 6e-8, -3e-4, 65504.0, -0.0, 1e-7], dtype=np.float16)
        d = np.where(pick < len(sp), sp[np.minimum(pick, len(sp) - 1)], d).astype(np.float16)
        if type_ == Q4_K:
            pick2 = rng.integers(0, 16, size=(rows, nb))
            dm = np.where(pick2 < len(sp), sp[np.minimum(pick2, len(sp) - 1)], dm).astype(np.float16)
    if type_ == Q8_0:
        put(0, d)
    elif type_ == Q4_K:
        put(0, d)
        put(2, dm)
    else:
        put(208, d)
    return out


# ---------------------------------------------------------------- a synthetic MoE layer

def make_layer(seed: int, n_expert: int, n_embd: int, n_ff: int, gate_type: int, down_type: int,
               router_type: int = F32, mode: str = "random", sigma: float = 0.02, special: bool = False):
    """A seeded MoE layer: dict with 'router' (n_expert x row_bytes uint8), 'gate', 'up', 'down' (lists of
    per-expert uint8 matrices in GGUF layout). mode 'random': random blocks; 'normal': N(0, sigma) quantized."""
    rng = np.random.Generator(np.random.PCG64(seed))
    r = rng.normal(0.0, sigma, size=(n_expert, n_embd)).astype(np.float32)
    if router_type == BF16:
        r = round_to_bf16(r)
    router = quantize(router_type, r)
    lay = {"router": router, "gate": [], "up": [], "down": []}
    for e in range(n_expert):
        for name, t, rows, cols in (("gate", gate_type, n_ff, n_embd), ("up", gate_type, n_ff, n_embd),
                                    ("down", down_type, n_embd, n_ff)):
            if mode == "random":
                m = random_blocks(t, rows, cols, rng, special)
            else:
                m = quantize(t, rng.normal(0.0, sigma, size=(rows, cols)).astype(np.float32))
            lay[name].append(np.ascontiguousarray(m))
    return lay


def zipf_bias(seed: int, n_expert: int, s: float = 1.0) -> np.ndarray:
    """Per-expert router bias for Zipf(s) popularity: expert of rank r gets log(r^-s), centred; ranks by a
    seeded permutation."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ranks = rng.permutation(n_expert) + 1
    b = -s * np.log(ranks.astype(np.float64))
    return (b - b.mean()).astype(np.float32)
