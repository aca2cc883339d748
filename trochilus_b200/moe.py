"""Python mirror of libtrmoe.so's C ABI (include/trmoe.h), through ctypes.

The C library is the product; this module only binds it, the way a Python host of Trochilus's
kernels would. It raises when the library is missing: there is no fallback of any kind.

  GpuMoe          the layer hook (tr_gpu_moe_*): Trochilus's forward_layer MoE block
                  (src/models/olmoe.c:1845-1933) on the GPU, weights resident in HBM
  matmul_grouped  tr_matmul_grouped (src/kernels/kernels.h:244-245) on host arrays
  matmul, softmax, swiglu   tr_matmul, tr_softmax, tr_swiglu
  q4x_road, q4x_prepare, matmul_q4x_prepared, swiglu_prepare   Q4_K's prepared road (kernels.h:280-300, 350)
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtrmoe.so")

F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30

# every function include/trmoe.h declares
EXPORTS = ["tr_gpu_moe_create", "tr_gpu_moe_free", "tr_gpu_moe_bytes", "tr_gpu_moe_set_layer", "tr_gpu_moe_layer",
           "tr_gpu_moe_layer_dev", "tr_gpu_moe_launches", "tr_gpu_moe_kernel_name", "tr_gpu_moe_profile",
           "tr_gpu_moe_profile_read", "tr_gpu_moe_check", "tr_gpu_moe_layer_part", "tr_gpu_moe_trace",
           "tr_gpu_moe_trace_read", "trmoe_last_error", "tr_matmul", "tr_matmul_grouped",
           "tr_matmul_grouped_s", "tr_softmax", "tr_swiglu", "trmoe_kernel_cache_clear", "tr_matmul_q4k_noalloc",
           "tr_gpu_moe_set_prefill", "tr_gpu_moe_ep_pack", "tr_gpu_moe_experts_dev", "tr_gpu_moe_ep_combine",
           "tr_gpu_moe_set_ffn_norm", "tr_gpu_moe_ffn", "tr_gpu_moe_ffn_dev", "tr_gpu_moe_ep_peer_region",
           "tr_gpu_moe_ep_peer_open", "tr_gpu_moe_ep_dispatch", "tr_gpu_moe_ep_experts", "tr_gpu_moe_ep_peer_combine",
           "tr_matmul_s", "tr_q4x_bytes", "tr_q4x_road", "tr_q4x_prepare", "tr_matmul_q4x_prepared",
           "tr_matmul_q4x_prepared_n", "tr_q4x_fused_calls", "tr_swiglu_prepare", "tr_gpu_moe_config_from_gguf",
           "tr_gpu_moe_load_gguf", "tr_gpu_open", "tr_gpu_close", "tr_gpu_name", "tr_gpu_attn_create",
           "tr_gpu_attn_free", "tr_gpu_attn_bytes", "tr_gpu_attn_write", "tr_gpu_attn_decode", "tr_gpu_attn_warm",
           "trmoe_kernel_arch"]


class Config(C.Structure):
    _fields_ = [("n_layers", C.c_int64), ("n_expert", C.c_int64), ("n_used", C.c_int64), ("n_embd", C.c_int64),
                ("n_ff", C.c_int64), ("norm_topk", C.c_int32), ("router_type", C.c_int32),
                ("gate_type", C.c_int32), ("down_type", C.c_int32), ("max_tokens", C.c_int64)]


class Outputs(C.Structure):
    _fields_ = [("logits", C.c_void_p), ("sel_id", C.c_void_p), ("sel_w", C.c_void_p), ("offsets", C.c_void_p),
                ("place", C.c_void_p), ("ffn_out", C.c_void_p)]


class TrMat(C.Structure):
    _fields_ = [("type", C.c_int32), ("rows", C.c_int64), ("cols", C.c_int64), ("data", C.c_void_p)]


_lib = None


def lib():
    """The loaded libtrmoe.so (built in-tree by trochilus_b200.build); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m trochilus_b200.build`")
    L = C.CDLL(LIB_PATH)
    L.tr_gpu_moe_create.restype = C.c_void_p
    L.tr_gpu_moe_create.argtypes = [C.POINTER(Config), C.c_int, C.c_char_p, C.c_size_t]
    L.tr_gpu_moe_free.argtypes = [C.c_void_p]
    L.tr_gpu_moe_bytes.restype = C.c_uint64
    L.tr_gpu_moe_bytes.argtypes = [C.POINTER(Config)]
    L.tr_gpu_moe_set_layer.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p),
                                       C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
    L.tr_gpu_moe_layer.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_layer_dev.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                       C.POINTER(Outputs), C.c_void_p]
    L.tr_gpu_moe_launches.argtypes = [C.c_void_p, C.c_int64]
    L.tr_gpu_moe_kernel_name.argtypes = [C.c_void_p, C.c_int64]
    L.tr_gpu_moe_kernel_name.restype = C.c_char_p
    L.tr_gpu_moe_ep_peer_region.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p]
    L.tr_gpu_moe_ep_peer_open.argtypes = [C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_ep_dispatch.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_ep_experts.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
    L.tr_gpu_moe_ep_peer_combine.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                             C.c_void_p]
    L.tr_gpu_moe_set_ffn_norm.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_float, C.c_char_p, C.c_size_t]
    L.tr_gpu_moe_ffn.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_ffn_dev.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.POINTER(Outputs),
                                     C.c_void_p]
    L.tr_gpu_moe_set_prefill.argtypes = [C.c_void_p, C.c_int64]
    L.tr_gpu_moe_ep_pack.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int64, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_experts_dev.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                         C.c_void_p]
    L.tr_gpu_moe_ep_combine.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                        C.c_void_p, C.c_void_p]
    L.tr_gpu_moe_profile.argtypes = [C.c_void_p, C.c_int]
    L.tr_gpu_moe_check.argtypes = [C.c_void_p]
    L.tr_gpu_moe_trace.argtypes = [C.c_void_p, C.c_int]
    L.tr_gpu_moe_trace_read.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
    L.tr_gpu_moe_layer_part.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_int64, C.c_void_p,
                                        C.POINTER(Outputs), C.c_void_p]
    L.tr_gpu_moe_profile_read.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
    L.trmoe_last_error.restype = C.c_char_p
    L.tr_matmul.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p]
    L.tr_matmul_grouped.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
    L.tr_matmul_grouped_s.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                      C.c_void_p]
    L.tr_softmax.argtypes = [C.c_void_p, C.c_int64]
    L.tr_swiglu.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64]
    L.tr_matmul_q4k_noalloc.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                        C.c_void_p]
    L.tr_matmul_s.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
    L.tr_q4x_bytes.argtypes = [C.c_int64]
    L.tr_q4x_bytes.restype = C.c_size_t
    L.tr_q4x_road.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p]
    L.tr_q4x_prepare.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
    L.tr_matmul_q4x_prepared.argtypes = [C.c_void_p, C.POINTER(TrMat), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p]
    L.tr_matmul_q4x_prepared_n.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p]
    L.tr_q4x_fused_calls.restype = C.c_uint64
    L.tr_swiglu_prepare.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
    L.tr_gpu_moe_config_from_gguf.argtypes = [C.c_char_p, C.POINTER(Config), C.POINTER(C.c_float), C.c_char_p,
                                              C.c_size_t]
    L.tr_gpu_moe_load_gguf.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_size_t]
    L.tr_gpu_open.restype = C.c_void_p
    L.tr_gpu_open.argtypes = [C.c_char_p, C.c_size_t]
    L.tr_gpu_close.argtypes = [C.c_void_p]
    L.tr_gpu_name.restype = C.c_char_p
    L.tr_gpu_name.argtypes = [C.c_void_p]
    L.tr_gpu_attn_create.restype = C.c_void_p
    L.tr_gpu_attn_create.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]
    L.tr_gpu_attn_free.argtypes = [C.c_void_p]
    L.tr_gpu_attn_bytes.restype = C.c_uint64
    L.tr_gpu_attn_bytes.argtypes = [C.c_int64] * 4
    L.tr_gpu_attn_write.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]
    L.tr_gpu_attn_decode.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_float, C.c_void_p]
    L.tr_gpu_attn_warm.argtypes = [C.c_void_p, C.c_uint64]
    _lib = L
    return L


def last_error() -> str:
    return lib().trmoe_last_error().decode()


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class GpuMoe:
    """A tr_gpu_moe context: n_layers MoE layers resident on one GPU."""

    def __init__(self, n_layers, n_expert, n_used, n_embd, n_ff, router_type, gate_type, down_type, max_tokens,
                 norm_topk=0, device=0):
        L = lib()
        self.cfg = Config(n_layers, n_expert, n_used, n_embd, n_ff, norm_topk, router_type, gate_type, down_type,
                          max_tokens)
        err = C.create_string_buffer(512)
        self.h = L.tr_gpu_moe_create(C.byref(self.cfg), device, err, 512)
        if not self.h:
            raise RuntimeError(f"tr_gpu_moe_create: {err.value.decode()}")
        self._keep = {}

    @staticmethod
    def bytes_needed(**kw) -> int:
        cfg = Config(kw["n_layers"], kw["n_expert"], kw["n_used"], kw["n_embd"], kw["n_ff"], kw.get("norm_topk", 0),
                     kw["router_type"], kw["gate_type"], kw["down_type"], kw["max_tokens"])
        return int(lib().tr_gpu_moe_bytes(C.byref(cfg)))

    def set_layer(self, layer: int, lay: dict, bias: np.ndarray | None = None):
        E = self.cfg.n_expert
        # an expert whose matrices are None is held by another rank (expert parallelism): not uploaded
        arr = {n: (C.c_void_p * E)(*[None if m is None else m.ctypes.data for m in lay[n]]) for n in ("gate", "up", "down")}
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        err = C.create_string_buffer(512)
        rc = lib().tr_gpu_moe_set_layer(self.h, layer, lay["router"].ctypes.data, _p(b),
                                        C.cast(arr["gate"], C.POINTER(C.c_void_p)),
                                        C.cast(arr["up"], C.POINTER(C.c_void_p)),
                                        C.cast(arr["down"], C.POINTER(C.c_void_p)), err, 512)
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_set_layer: {err.value.decode()}")

    def layer(self, layer: int, normed: np.ndarray, x: np.ndarray, want_sel: bool = True):
        """Host arrays: x is updated in place; returns (sel_id, sel_w) or None."""
        normed = np.ascontiguousarray(normed, dtype=np.float32)
        assert x.dtype == np.float32 and x.flags.c_contiguous
        T = normed.shape[0]
        sid = np.zeros((T, self.cfg.n_used), np.int64) if want_sel else None
        sw = np.zeros((T, self.cfg.n_used), np.float32) if want_sel else None
        rc = lib().tr_gpu_moe_layer(self.h, layer, _p(normed), T, _p(x), _p(sid), _p(sw))
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_layer: {last_error()}")
        return (sid, sw) if want_sel else None

    def set_ffn_norm(self, layer: int, weight: np.ndarray, eps: float):
        """tr_gpu_moe_set_ffn_norm: the layer's ffn_norm weight (n_embd floats) and the model's RMS epsilon."""
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        assert weight.size == self.cfg.n_embd
        err = C.create_string_buffer(512)
        if lib().tr_gpu_moe_set_ffn_norm(self.h, layer, _p(weight), eps, err, 512) != 0:
            raise RuntimeError(f"tr_gpu_moe_set_ffn_norm: {err.value.decode()}")

    def load_gguf(self, path: str):
        """tr_gpu_moe_load_gguf: every layer's router, experts and ffn_norm from an OLMoE GGUF file"""
        err = C.create_string_buffer(512)
        if lib().tr_gpu_moe_load_gguf(self.h, os.fsencode(path), err, 512) != 0:
            raise RuntimeError(f"tr_gpu_moe_load_gguf: {err.value.decode()}")

    @classmethod
    def from_gguf(cls, path: str, max_tokens: int, device: int = 0) -> "GpuMoe":
        """a context made from the file's configuration (tr_gpu_moe_config_from_gguf) and loaded from it"""
        cfg, _ = config_from_gguf(path, max_tokens)
        m = cls(cfg.n_layers, cfg.n_expert, cfg.n_used, cfg.n_embd, cfg.n_ff, cfg.router_type, cfg.gate_type,
                cfg.down_type, max_tokens, norm_topk=cfg.norm_topk, device=device)
        m.load_gguf(path)
        return m

    def ffn(self, layer: int, x: np.ndarray, want_normed: bool = False, want_sel: bool = False):
        """tr_gpu_moe_ffn on host arrays: x (T x n_embd, float32, C order) normalised by the layer's ffn_norm and
        given the layer's output in place; returns (normed or None, sel_id or None, sel_w or None)."""
        assert x.dtype == np.float32 and x.flags.c_contiguous
        T = x.shape[0]
        nrm = np.zeros_like(x) if want_normed else None
        sid = np.zeros((T, self.cfg.n_used), np.int64) if want_sel else None
        sw = np.zeros((T, self.cfg.n_used), np.float32) if want_sel else None
        if lib().tr_gpu_moe_ffn(self.h, layer, T, _p(x), _p(nrm), _p(sid), _p(sw)) != 0:
            raise RuntimeError(f"tr_gpu_moe_ffn: {last_error()}")
        return nrm, sid, sw

    def ffn_ptrs(self, layer: int, n_tok: int, x_ptr: int, host: bool, normed_ptr: int | None = None,
                 outs: dict | None = None, stream: int = 0):
        """Raw-pointer forms: host=True tr_gpu_moe_ffn (host memory, e.g. pinned), else tr_gpu_moe_ffn_dev (device
        pointers, enqueued on `stream`)."""
        if host:
            rc = lib().tr_gpu_moe_ffn(self.h, layer, n_tok, x_ptr, normed_ptr, None, None)
        else:
            o = None
            if outs:
                o = Outputs(*(outs.get(k) for k in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out")))
            rc = lib().tr_gpu_moe_ffn_dev(self.h, layer, n_tok, x_ptr, normed_ptr, C.byref(o) if o else None,
                                          stream or None)
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_ffn: {last_error()}")

    def layer_ptrs(self, layer: int, normed_ptr: int, n_tok: int, x_ptr: int, host: bool):
        """Raw-pointer form of layer() for pinned host buffers (host=True) or device buffers (host=False, on the
        context's stream, not waited for)."""
        if host:
            rc = lib().tr_gpu_moe_layer(self.h, layer, normed_ptr, n_tok, x_ptr, None, None)
        else:
            rc = lib().tr_gpu_moe_layer_dev(self.h, layer, normed_ptr, n_tok, x_ptr, None, None)
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_layer: {last_error()}")

    def layer_dev(self, layer: int, normed_ptr: int, n_tok: int, x_ptr: int, outs: dict | None = None,
                  stream: int = 0):
        """Device pointers (e.g. torch tensors' data_ptr()); enqueued on `stream` (0: the context's own)."""
        o = None
        if outs:
            o = Outputs(*(outs.get(k) for k in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out")))
        rc = lib().tr_gpu_moe_layer_dev(self.h, layer, normed_ptr, n_tok, x_ptr, C.byref(o) if o else None,
                                        stream or None)
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_layer_dev: {last_error()}")

    def layer_part(self, layer: int, part: int, normed_ptr: int, n_tok: int, x_ptr: int, outs: dict | None = None,
                   stream: int = 0):
        """tr_gpu_moe_layer_part: one of the four parts of a layer call (device pointers, enqueued only); outs as in
        layer_dev (part 0 writes logits, sel_id, sel_w, offsets, place)."""
        o = None
        if outs:
            o = Outputs(*(outs.get(k) for k in ("logits", "sel_id", "sel_w", "offsets", "place", "ffn_out")))
        rc = lib().tr_gpu_moe_layer_part(self.h, layer, part, normed_ptr, n_tok, x_ptr, C.byref(o) if o else None,
                                         stream or None)
        if rc != 0:
            raise RuntimeError(f"tr_gpu_moe_layer_part: {last_error()}")

    ZONES = ("router", "gate_up", "act_prep", "down")

    def profile(self, on: bool):
        if lib().tr_gpu_moe_profile(self.h, 1 if on else 0) != 0:
            raise RuntimeError(f"tr_gpu_moe_profile: {last_error()}")

    def profile_read(self) -> dict:
        ms = np.zeros(4, np.float64)
        calls = np.zeros(4, np.int64)
        if lib().tr_gpu_moe_profile_read(self.h, _p(ms), _p(calls), 4) != 0:
            raise RuntimeError(f"tr_gpu_moe_profile_read: {last_error()}")
        return {z: (float(ms[i]), int(calls[i])) for i, z in enumerate(self.ZONES)}

    def check(self):
        """tr_gpu_moe_check: wait for the stream; raise if a kernel gave up on a bounded wait."""
        if lib().tr_gpu_moe_check(self.h) != 0:
            raise RuntimeError(f"tr_gpu_moe_check: {last_error()}")

    def trace(self, on: bool):
        if lib().tr_gpu_moe_trace(self.h, 1 if on else 0) != 0:
            raise RuntimeError(f"tr_gpu_moe_trace: {last_error()}")

    def trace_read(self) -> np.ndarray:
        """the fused kernel's last timeline: ctas x 64 %globaltimer slots (ns, 0: no event)"""
        buf = np.zeros(148 * 8 * 64, np.uint64)
        n = lib().tr_gpu_moe_trace_read(self.h, _p(buf), buf.size)
        if n < 0:
            raise RuntimeError(f"tr_gpu_moe_trace_read: {last_error()}")
        return buf[:n * 64].reshape(n, 64)

    def launches(self, n_tok: int) -> int:
        return int(lib().tr_gpu_moe_launches(self.h, n_tok))

    def kernel_name(self, n_tok: int) -> str:
        """the kernel a call of n_tok tokens runs when it is one kernel ("" otherwise)"""
        return lib().tr_gpu_moe_kernel_name(self.h, n_tok).decode()

    def ep_pack(self, sel_id_ptr, n_tok, n_ranks, cap, normed_ptr, send_rows_ptr, send_ids_ptr, send_counts_ptr,
                place_ptr, scratch_ptr, stream=0):
        """tr_gpu_moe_ep_pack (device pointers; cap 0: packed, cap >= rows: padded per destination)."""
        if lib().tr_gpu_moe_ep_pack(self.h, sel_id_ptr, n_tok, n_ranks, cap, normed_ptr, send_rows_ptr, send_ids_ptr,
                                    send_counts_ptr, place_ptr, scratch_ptr, stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_pack: {last_error()}")

    def ep_peer_region(self, n_ranks: int, rank: int, cap: int) -> bytes:
        """tr_gpu_moe_ep_peer_region: this rank's exchange region; returns its IPC handle (64 bytes)"""
        h = C.create_string_buffer(64)
        if lib().tr_gpu_moe_ep_peer_region(self.h, n_ranks, rank, cap, h) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_peer_region: {last_error()}")
        return h.raw

    def ep_peer_open(self, handles: list):
        """tr_gpu_moe_ep_peer_open: every rank's handle, in rank order"""
        buf = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        if lib().tr_gpu_moe_ep_peer_open(self.h, buf) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_peer_open: {last_error()}")

    def ep_dispatch(self, sel_id_ptr, n_tok, normed_ptr, place_ptr, stream=0):
        if lib().tr_gpu_moe_ep_dispatch(self.h, sel_id_ptr, n_tok, normed_ptr, place_ptr, stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_dispatch: {last_error()}")

    def ep_experts(self, layer, stream=0):
        if lib().tr_gpu_moe_ep_experts(self.h, layer, stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_experts: {last_error()}")

    def ep_peer_combine(self, sel_w_ptr, place_ptr, n_tok, x_ptr, ffn_ptr=None, stream=0):
        if lib().tr_gpu_moe_ep_peer_combine(self.h, sel_w_ptr, place_ptr, n_tok, x_ptr, ffn_ptr, stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_peer_combine: {last_error()}")

    def experts_dev(self, layer, rows_ptr, ids_ptr, n_rows, out_ptr, stream=0):
        """tr_gpu_moe_experts_dev (device pointers)."""
        if lib().tr_gpu_moe_experts_dev(self.h, layer, rows_ptr, ids_ptr, n_rows, out_ptr, stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_experts_dev: {last_error()}")

    def ep_combine(self, sel_w_ptr, place_ptr, back_ptr, n_tok, x_ptr, ffn_ptr=None, stream=0):
        """tr_gpu_moe_ep_combine (device pointers)."""
        if lib().tr_gpu_moe_ep_combine(self.h, sel_w_ptr, place_ptr, back_ptr, n_tok, x_ptr, ffn_ptr,
                                       stream or None) != 0:
            raise RuntimeError(f"tr_gpu_moe_ep_combine: {last_error()}")

    def set_prefill(self, min_tokens: int):
        """tr_gpu_moe_set_prefill: calls of at least min_tokens tokens take the tensor-core road (0: never)."""
        if lib().tr_gpu_moe_set_prefill(self.h, min_tokens) != 0:
            raise RuntimeError(f"tr_gpu_moe_set_prefill: {last_error()}")

    def close(self):
        if self.h:
            lib().tr_gpu_moe_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GpuAttn:
    """A tr_gpu_attn session (Trochilus's GPU attention backend, src/backend/gpu_attn.h) on host arrays: the device
    (tr_gpu_open) and one session's cache of n_ctx positions for n_layers layers of n_head heads of 128."""

    def __init__(self, n_layers: int, n_head: int, n_ctx: int, head_dim: int = 128):
        L = lib()
        err = C.create_string_buffer(512)
        self.g = L.tr_gpu_open(err, 512)
        if not self.g:
            raise RuntimeError(f"tr_gpu_open: {err.value.decode()}")
        self.a = L.tr_gpu_attn_create(self.g, n_layers, n_head, head_dim, n_ctx, err, 512)
        if not self.a:
            L.tr_gpu_close(self.g)
            self.g = None
            raise RuntimeError(f"tr_gpu_attn_create: {err.value.decode()}")
        self.n_head, self.hd = n_head, head_dim

    def name(self) -> str:
        return lib().tr_gpu_name(self.g).decode()

    def write(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray):
        """tr_gpu_attn_write: k, v [n_tok][n_head * head_dim]"""
        k = np.ascontiguousarray(k, dtype=np.float32).reshape(-1, self.n_head * self.hd)
        v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1, self.n_head * self.hd)
        if lib().tr_gpu_attn_write(self.a, layer, pos0, k.shape[0], _p(k), _p(v)) != 0:
            raise RuntimeError(f"tr_gpu_attn_write: {last_error()}")

    def decode(self, layer: int, pos: int, q, k, v, scale: float) -> np.ndarray:
        """tr_gpu_attn_decode: q, k, v [n_head * head_dim]; returns out [n_head][head_dim]"""
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32).ravel() for a in (q, k, v))
        out = np.full((self.n_head, self.hd), np.nan, dtype=np.float32)
        if lib().tr_gpu_attn_decode(self.a, layer, pos, _p(q), _p(k), _p(v), scale, _p(out)) != 0:
            raise RuntimeError(f"tr_gpu_attn_decode: {last_error()}")
        return out

    def warm(self, ns: int):
        if lib().tr_gpu_attn_warm(self.a, ns) != 0:
            raise RuntimeError(f"tr_gpu_attn_warm: {last_error()}")

    def close(self):
        if getattr(self, "a", None):
            lib().tr_gpu_attn_free(self.a)
            self.a = None
        if getattr(self, "g", None):
            lib().tr_gpu_close(self.g)
            self.g = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def config_from_gguf(path: str, max_tokens: int = 1) -> tuple[Config, float]:
    """tr_gpu_moe_config_from_gguf: the context configuration an OLMoE GGUF file gives, and its RMSNorm epsilon"""
    cfg = Config(0, 0, 0, 0, 0, 0, 0, 0, 0, max_tokens)
    eps = C.c_float(0.0)
    err = C.create_string_buffer(512)
    if lib().tr_gpu_moe_config_from_gguf(os.fsencode(path), C.byref(cfg), C.byref(eps), err, 512) != 0:
        raise RuntimeError(f"tr_gpu_moe_config_from_gguf: {err.value.decode()}")
    return cfg, float(eps.value)


def matmul_grouped(type_: int, rows: int, cols: int, mats, offsets, x: np.ndarray, use_s: bool = False):
    """tr_matmul_grouped on host arrays: mats[g] = rows x row_bytes uint8 (GGUF), x = offsets[-1] x cols."""
    n = len(mats)
    ws = (TrMat * n)(*[TrMat(type_, rows, cols, m.ctypes.data) for m in mats])
    off = np.ascontiguousarray(offsets, dtype=np.int64)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.full((int(off[-1]), rows), np.nan, dtype=np.float32)
    if use_s:
        lib().tr_matmul_grouped_s(None, ws, _p(off), n, _p(x), _p(y), None)
    else:
        lib().tr_matmul_grouped(None, ws, _p(off), n, _p(x), _p(y))
    err = last_error()
    if err:
        raise RuntimeError(f"tr_matmul_grouped: {err}")
    return y


def matmul(type_: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray):
    m = TrMat(type_, rows, cols, w.ctypes.data)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.full((x.shape[0], rows), np.nan, dtype=np.float32)
    lib().tr_matmul(None, C.byref(m), _p(x), x.shape[0], _p(y))
    err = last_error()
    if err:
        raise RuntimeError(f"tr_matmul: {err}")
    return y


def matmul_s(type_: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray):
    """tr_matmul_s on host arrays (tr_matmul's result; no scratch)."""
    m = TrMat(type_, rows, cols, w.ctypes.data)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.full((x.shape[0], rows), np.nan, dtype=np.float32)
    lib().tr_matmul_s(None, C.byref(m), _p(x), x.shape[0], _p(y), None)
    err = last_error()
    if err:
        raise RuntimeError(f"tr_matmul_s: {err}")
    return y


def q4x_bytes(cols: int) -> int:
    """tr_q4x_bytes: the bytes of one prepared row's slot"""
    return int(lib().tr_q4x_bytes(cols))


def q4x_road(type_: int, rows: int, cols: int) -> int:
    """tr_q4x_road for weights of this type and shape (the groups and scratch are not consulted)"""
    m = TrMat(type_, rows, cols, None)
    return int(lib().tr_q4x_road(None, C.byref(m), None, 1, None))


def q4x_prepare(x: np.ndarray, xq: np.ndarray | None = None) -> np.ndarray:
    """tr_q4x_prepare: x (n x cols) into slots of tr_q4x_bytes(cols) bytes (a uint8 buffer, made when None)"""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, cols = x.shape
    if xq is None:
        xq = np.zeros(n * q4x_bytes(cols), dtype=np.uint8)
    lib().tr_q4x_prepare(None, _p(x), n, cols, _p(xq))
    return xq


def matmul_q4x_prepared(rows: int, cols: int, mats_list, offsets, xq: np.ndarray, map_=None):
    """tr_matmul_q4x_prepared (one weight) or tr_matmul_q4x_prepared_n (several) on host arrays: mats_list[m][g] =
    weight m's group g (rows x row_bytes uint8, Q4_K); returns (the call's return value, [y_m])."""
    n_w, n = len(mats_list), len(mats_list[0])
    ws = [(TrMat * n)(*[TrMat(Q4_K, rows, cols, mm.ctypes.data) for mm in mats]) for mats in mats_list]
    off = np.ascontiguousarray(offsets, dtype=np.int64)
    mp = None if map_ is None else np.ascontiguousarray(map_, dtype=np.int64)
    ys = [np.full((int(off[-1]), rows), np.nan, dtype=np.float32) for _ in range(n_w)]
    if n_w == 1:
        rc = lib().tr_matmul_q4x_prepared(None, ws[0], _p(off), n, _p(xq), _p(mp), _p(ys[0]), None)
    else:
        wp = (C.c_void_p * n_w)(*[C.cast(w, C.c_void_p) for w in ws])
        yp = (C.c_void_p * n_w)(*[y.ctypes.data for y in ys])
        rc = lib().tr_matmul_q4x_prepared_n(None, wp, n_w, _p(off), n, _p(xq), _p(mp), yp, None)
    err = last_error()
    if err:
        raise RuntimeError(f"tr_matmul_q4x_prepared: {err}")
    return rc, ys


def q4x_fused_calls() -> int:
    return int(lib().tr_q4x_fused_calls())


def swiglu_prepare(x: np.ndarray, y: np.ndarray):
    """tr_swiglu_prepare on host arrays (n_rows x n): returns (x after, the slots)"""
    out = np.array(x, dtype=np.float32, copy=True)
    y = np.ascontiguousarray(y, dtype=np.float32)
    n_rows, n = out.shape
    xq = np.zeros(n_rows * q4x_bytes(n), dtype=np.uint8)
    lib().tr_swiglu_prepare(None, _p(out), _p(y), n_rows, n, _p(xq))
    err = last_error()
    if err:
        raise RuntimeError(f"tr_swiglu_prepare: {err}")
    return out, xq


def kernel_cache_clear():
    """trmoe_kernel_cache_clear: forget every weight the kernel-level calls uploaded."""
    lib().trmoe_kernel_cache_clear()


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().tr_softmax(_p(y), y.size)
    err = last_error()
    if err:
        raise RuntimeError(f"tr_softmax: {err}")
    return y


def swiglu(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    out = np.array(x, dtype=np.float32, copy=True)
    y = np.ascontiguousarray(y, dtype=np.float32)
    lib().tr_swiglu(None, _p(out), _p(y), out.size)
    err = last_error()
    if err:
        raise RuntimeError(f"tr_swiglu: {err}")
    return out
