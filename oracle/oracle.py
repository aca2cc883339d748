"""TEST INFRASTRUCTURE ONLY: ctypes loaders of the CPU checkers.

  Oracle()   oracle/liboracle.so, the plain-C restatement of Trochilus's MoE arithmetic (moe_oracle.c)
  RefLib()   oracle/_ref/libtrref_moe.so, Trochilus's own kernel sources compiled where they lie plus
             ref_harness.c (built in the development container; the GPU box receives the prebuilt file)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtrref_moe.so")

F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30


def build(ref_tree: str | None = None):
    """make -C oracle: the restatement always; with ref_tree (the reference's source tree, when it exists) also the
    reference's kernels with the harness and its whole engine, plain and relinked onto libtrmoe.so."""
    args = ["make", "-s", "-C", HERE, "all"]
    if ref_tree and os.path.exists(os.path.join(ref_tree, "src", "kernels", "kernels.c")):
        args.append(f"REF={ref_tree}")
    subprocess.check_call(args)


class Desc(C.Structure):
    _fields_ = [("n_expert", C.c_int64), ("n_used", C.c_int64), ("n_embd", C.c_int64), ("n_ff", C.c_int64),
                ("norm_topk", C.c_int32), ("router_type", C.c_int32), ("gate_type", C.c_int32),
                ("up_type", C.c_int32), ("down_type", C.c_int32), ("router", C.c_void_p),
                ("router_bias", C.c_void_p), ("gate", C.POINTER(C.c_void_p)), ("up", C.POINTER(C.c_void_p)),
                ("down", C.POINTER(C.c_void_p))]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def make_desc(layer: dict, n_embd: int, n_ff: int, n_used: int, norm_topk: int, router_type: int, gate_type: int,
              down_type: int, bias=None):
    """A Desc over numpy arrays; returns (desc, keep) where keep holds what the pointers point into."""
    E = len(layer["gate"])
    arrs = {name: (C.c_void_p * E)(*[m.ctypes.data for m in layer[name]]) for name in ("gate", "up", "down")}
    d = Desc()
    d.n_expert, d.n_used, d.n_embd, d.n_ff = E, n_used, n_embd, n_ff
    d.norm_topk = norm_topk
    d.router_type, d.gate_type, d.up_type, d.down_type = router_type, gate_type, gate_type, down_type
    d.router = layer["router"].ctypes.data
    d.router_bias = None if bias is None else bias.ctypes.data
    d.gate = C.cast(arrs["gate"], C.POINTER(C.c_void_p))
    d.up = C.cast(arrs["up"], C.POINTER(C.c_void_p))
    d.down = C.cast(arrs["down"], C.POINTER(C.c_void_p))
    return d, (arrs, layer, bias)


class _Common:
    prefix = ""

    def _bind(self, lib):
        f = lambda n: getattr(lib, self.prefix + n)
        self.lib = lib
        self._expf = f("expf")
        self._expf.restype = C.c_float
        self._expf.argtypes = [C.c_float]
        self._expf_many = f("expf_many")
        self._expf_many.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        self._softmax = f("softmax")
        self._softmax.argtypes = [C.c_void_p, C.c_int64]
        self._dot_row = f("dot_row")
        self._dot_row.restype = C.c_float
        self._dot_row.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        self._rmsnorm = f("rmsnorm")
        self._rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_float]

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """ffn_norm: each row of x (T x n, or one row) normalised by its RMS and scaled by w
        (src/kernels/kernels.c:1351-1360 per token, as norm_body applies it, src/models/olmoe.c:1360-1366)"""
        y = np.array(x, dtype=np.float32, copy=True)
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows = y.reshape(-1, y.shape[-1])
        for r in rows:  # a view of y's memory: normalised in place
            self._rmsnorm(r.ctypes.data, _ptr(w), r.size, eps)
        return y

    def expf(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self._expf_many(_ptr(x), _ptr(y), x.size)
        return y

    def softmax(self, x: np.ndarray) -> np.ndarray:
        y = np.array(x, dtype=np.float32, copy=True)
        self._softmax(_ptr(y), y.size)
        return y

    def dot_row(self, type_: int, row: np.ndarray, x: np.ndarray) -> np.float32:
        x = np.ascontiguousarray(x, dtype=np.float32)
        row = np.ascontiguousarray(row)
        return np.float32(self._dot_row(type_, _ptr(row), _ptr(x), x.size))


class Oracle(_Common):
    prefix = "orc_"

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        self._bind(C.CDLL(ORACLE_SO))
        L = self.lib
        L.orc_matmul_grouped.argtypes = [C.c_int, C.c_int64, C.c_int64, C.POINTER(C.c_void_p), C.c_void_p, C.c_int64,
                                         C.c_void_p, C.c_void_p]
        L.orc_swiglu.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.orc_route.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_counting_sort.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]
        L.orc_moe_layer.argtypes = [C.POINTER(Desc), C.c_void_p, C.c_int64, C.c_void_p] + [C.c_void_p] * 8
        L.orc_row_bytes.restype = C.c_size_t
        L.orc_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.orc_set_mutation.argtypes = [C.c_int]
        L.orc_attention_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                         C.c_int64, C.c_float, C.c_void_p, C.c_void_p]

    def attention(self, q, keys, values, scale):
        """one decode token's attention, head by head: q [n_head][hd], keys / values [n_pos][n_head][hd] (the
        engine's cache rows); returns out [n_head][hd] (tr_attention_head per head at its offset)"""
        q = np.ascontiguousarray(q, dtype=np.float32)
        keys = np.ascontiguousarray(keys, dtype=np.float32)
        values = np.ascontiguousarray(values, dtype=np.float32)
        n_pos, n_head, hd = keys.shape
        out = np.zeros((n_head, hd), dtype=np.float32)
        scores = np.zeros(max(n_pos, 1), dtype=np.float32)
        for h in range(n_head):
            self.lib.orc_attention_head(q[h].ctypes.data, _ptr(keys), _ptr(values), n_head * hd, h * hd, n_pos, hd,
                                        scale, _ptr(scores), out[h].ctypes.data)
        return out

    def set_mutation(self, m: int):
        """plants mistake m in the restatement (moe_oracle.c lists them; 0: none). Tests only, to show that a
        comparison sees a wrong step; every caller sets it back to 0."""
        self.lib.orc_set_mutation(m)

    def matmul_grouped(self, type_, rows, cols, mats, offsets, x):
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        x = np.ascontiguousarray(x, dtype=np.float32)
        ptrs = (C.c_void_p * len(mats))(*[m.ctypes.data for m in mats])
        y = np.zeros((int(offsets[-1]), rows), dtype=np.float32)
        self.lib.orc_matmul_grouped(type_, rows, cols, ptrs, _ptr(offsets), len(mats), _ptr(x), _ptr(y))
        return y

    def swiglu(self, x, y):
        x = np.array(x, dtype=np.float32, copy=True)
        y = np.ascontiguousarray(y, dtype=np.float32)
        self.lib.orc_swiglu(_ptr(x), _ptr(y), x.size)
        return x

    def route(self, logits, k, norm_topk=0):
        p = np.array(logits, dtype=np.float32, copy=True)
        T, E = p.shape
        ids = np.zeros((T, k), dtype=np.int64)
        ws = np.zeros((T, k), dtype=np.float32)
        self.lib.orc_route(_ptr(p), T, E, k, norm_topk, _ptr(ids), _ptr(ws))
        return ids, ws

    def counting_sort(self, sel_id, E):
        s = np.ascontiguousarray(sel_id, dtype=np.int64).ravel()
        off = np.zeros(E + 1, dtype=np.int64)
        place = np.zeros(s.size, dtype=np.int64)
        self.lib.orc_counting_sort(_ptr(s), s.size, E, _ptr(off), _ptr(place))
        return off, place

    def moe_layer(self, desc, normed, x):
        return _run_layer(lambda *a: self.lib.orc_moe_layer(C.byref(desc), *a), desc, normed, x)


def _run_layer(call, desc, normed, x):
    normed = np.ascontiguousarray(normed, dtype=np.float32)
    T, H = normed.shape
    E, k, F = desc.n_expert, desc.n_used, desc.n_ff
    out = {
        "x": np.array(x, dtype=np.float32, copy=True),
        "logits": np.zeros((T, E), np.float32),
        "sel_id": np.zeros((T, k), np.int64),
        "sel_w": np.zeros((T, k), np.float32),
        "offsets": np.zeros(E + 1, np.int64),
        "place": np.zeros((T, k), np.int64),
        "h1": np.zeros((T * k, F), np.float32),
        "h3": np.zeros((T * k, H), np.float32),
        "ffn_out": np.zeros((T, H), np.float32),
    }
    rc = call(_ptr(normed), T, _ptr(out["x"]), _ptr(out["logits"]), _ptr(out["sel_id"]), _ptr(out["sel_w"]),
              _ptr(out["offsets"]), _ptr(out["place"]), _ptr(out["h1"]), _ptr(out["h3"]), _ptr(out["ffn_out"]))
    out["rc"] = rc
    return out


class RefLib(_Common):
    """Trochilus's own code (oracle/_ref). tier: None = the best this CPU has, or 'scalar' / 'avx2' / 'avx512'."""
    prefix = "ref_"

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self, tier: str | None = None):
        if not os.path.exists(REF_SO):
            build()
        self._bind(C.CDLL(REF_SO))
        L = self.lib
        L.ref_pool_create.restype = C.c_void_p
        L.ref_pool_create.argtypes = [C.c_int]
        L.ref_pool_destroy.argtypes = [C.c_void_p]
        L.ref_pool_size.argtypes = [C.c_void_p]
        L.ref_set_tier.argtypes = [C.c_char_p]
        L.ref_tier.restype = C.c_char_p
        L.ref_state_create.restype = C.c_void_p
        L.ref_state_create.argtypes = [C.c_void_p, C.POINTER(Desc), C.c_int64]
        L.ref_state_free.argtypes = [C.c_void_p]
        L.ref_moe_layer.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(Desc), C.c_void_p, C.c_int64,
                                    C.c_void_p] + [C.c_void_p] * 8
        L.ref_matmul_grouped.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.POINTER(C.c_void_p), C.c_void_p,
                                         C.c_int64, C.c_void_p, C.c_void_p]
        L.ref_swiglu.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ref_dequant_row.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        if tier is not None and L.ref_set_tier(tier.encode()) != 0:
            raise RuntimeError(f"tier {tier} not available on this CPU")

    def tier(self) -> str:
        return self.lib.ref_tier().decode()

    def set_tier(self, tier: str | None):
        if self.lib.ref_set_tier((tier or "").encode()) != 0:
            raise RuntimeError(f"tier {tier} not available")

    def pool(self, n_threads: int = 0):
        return self.lib.ref_pool_create(n_threads)

    def pool_size(self, pool) -> int:
        return self.lib.ref_pool_size(pool)

    def pool_destroy(self, pool):
        self.lib.ref_pool_destroy(pool)

    def state(self, pool, desc, max_tokens):
        return self.lib.ref_state_create(pool, C.byref(desc), max_tokens)

    def state_free(self, st):
        self.lib.ref_state_free(st)

    def moe_layer(self, desc, normed, x, pool=None, state=None):
        own = state is None
        if own:
            state = self.state(pool, desc, normed.shape[0])
        try:
            return _run_layer(lambda *a: self.lib.ref_moe_layer(pool, state, C.byref(desc), *a), desc, normed, x)
        finally:
            if own:
                self.state_free(state)

    def matmul_grouped(self, type_, rows, cols, mats, offsets, x, pool=None):
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        x = np.ascontiguousarray(x, dtype=np.float32)
        ptrs = (C.c_void_p * len(mats))(*[m.ctypes.data for m in mats])
        y = np.zeros((int(offsets[-1]), rows), dtype=np.float32)
        self.lib.ref_matmul_grouped(pool, type_, rows, cols, ptrs, _ptr(offsets), len(mats), _ptr(x), _ptr(y))
        return y

    def swiglu(self, x, y):
        x = np.array(x, dtype=np.float32, copy=True)
        y = np.ascontiguousarray(y, dtype=np.float32)
        self.lib.ref_swiglu(_ptr(x), _ptr(y), x.size)
        return x

    def dequant_row(self, type_, row, n):
        out = np.zeros(n, np.float32)
        row = np.ascontiguousarray(row)
        self.lib.ref_dequant_row(type_, _ptr(row), _ptr(out), n)
        return out
