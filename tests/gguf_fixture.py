"""Writes OLMoE-shaped GGUF files for the loader's tests (tr_gpu_moe_config_from_gguf, tr_gpu_moe_load_gguf), with
gguf-py's writer (an independent implementation of the format): the olmoe.* metadata the reference reads
(src/models/olmoe.c:541-563) and each layer's ffn_norm, router and stacked expert tensors under the reference's names
(olmoe.c:605-641, 895-906). Test infrastructure only."""
from __future__ import annotations

import numpy as np

from trochilus_b200 import gguf_blocks as gb


def write_olmoe_moe(path, layers, norms, eps=1e-5, n_used=2, norm_topk=False, router_type=gb.F32,
                    gate_type=gb.Q8_0, down_type=gb.Q6_K, arch="olmoe", skip=(), reshape=None, extra_kv=None,
                    down_types=None):
    """layers: gguf_blocks.make_layer dicts (router bytes, per-expert gate/up/down); norms: one float32 vector of
    n_embd a layer. skip: tensor names left out; reshape: {name: numpy shape} written instead of the true one;
    extra_kv: {key: value} added as metadata (ints as uint32); down_types: a down type per layer (else down_type)."""
    import gguf
    E = len(layers[0]["gate"])
    F, H = layers[0]["gate"][0].shape[0], len(norms[0])
    w = gguf.GGUFWriter(str(path), arch)
    w.add_uint32("olmoe.block_count", len(layers))
    w.add_uint32("olmoe.embedding_length", H)
    w.add_uint32("olmoe.feed_forward_length", F)
    w.add_uint32("olmoe.attention.head_count", 16)
    w.add_uint32("olmoe.attention.head_count_kv", 16)
    w.add_uint32("olmoe.expert_count", E)
    w.add_uint32("olmoe.expert_used_count", n_used)
    w.add_float32("olmoe.attention.layer_norm_rms_epsilon", eps)
    w.add_bool("olmoe.expert_weights_norm", bool(norm_topk))
    w.add_array("tokenizer.ggml.tokens", ["a", "bc", "def"])  # an array of strings the reader must step over
    for k, v in (extra_kv or {}).items():
        w.add_uint32(k, v)
    for L, (lay, nw) in enumerate(zip(layers, norms)):
        types = {"gate": gate_type, "up": gate_type, "down": down_types[L] if down_types else down_type}
        tensors = {f"blk.{L}.ffn_norm.weight": (np.asarray(nw, dtype=np.float32), None),
                   f"blk.{L}.ffn_gate_inp.weight": (np.ascontiguousarray(lay["router"]), router_type)}
        for part in ("gate", "up", "down"):
            stacked = np.ascontiguousarray(np.stack(lay[part]))  # E x rows x row_bytes: ne = [cols, rows, E]
            tensors[f"blk.{L}.ffn_{part}_exps.weight"] = (stacked, types[part])
        for name, (arr, t) in tensors.items():
            if name in skip:
                continue
            if reshape and name in reshape:
                arr = arr.reshape(reshape[name])
            if t is None:
                w.add_tensor(name, arr)
            else:
                w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def write_olmoe_model(path, n_layers, seed, attn_type=gb.Q8_0, gate_type=gb.Q8_0, down_type=gb.Q8_0,
                      embd_type=gb.Q8_0, head_type=gb.Q8_0, router_type=gb.F32, mode="normal", vocab=50304,
                      n_embd=2048, n_ff=1024, n_head=16, n_expert=64, n_used=8, eps=1e-5, sigma=0.02):
    """A whole OLMoE-architecture model the reference engine loads (src/models/olmoe.c:541-563 metadata, :820-906
    tensors): token_embd, output_norm, output, and per layer attn_norm, attn_q/k/v/output, attn_q_norm, attn_k_norm,
    ffn_norm, ffn_gate_inp and the stacked experts. Norm weights are 1. Every matrix is N(0, sigma) quantized by this
    repo's encoders, except with mode 'random' the experts: random quant blocks with bounded scales (centred for
    Q4_K), quick for the 16-layer configs[1]. No tokenizer: the engine is driven by token ids."""
    import gguf
    rng = np.random.Generator(np.random.PCG64(seed))

    def mat(t, rows, cols, expert=False):
        if expert and mode == "random" and t == gb.Q4_K:
            return _centered_q4k(rows, cols, rng)
        if expert and mode == "random" and t not in (gb.F32, gb.F16, gb.BF16):
            return gb.random_blocks(t, rows, cols, rng)
        out = np.empty((rows, gb.row_bytes(t, cols)), dtype=np.uint8)
        for r0 in range(0, rows, 4096):  # in slices, so that the floats never take much memory
            r1 = min(rows, r0 + 4096)
            out[r0:r1] = gb.quantize(t, rng.normal(0.0, sigma, size=(r1 - r0, cols)).astype(np.float32))
        return out

    w = gguf.GGUFWriter(str(path), "olmoe")
    for key, v in (("block_count", n_layers), ("embedding_length", n_embd), ("feed_forward_length", n_ff),
                   ("attention.head_count", n_head), ("attention.head_count_kv", n_head), ("expert_count", n_expert),
                   ("expert_used_count", n_used), ("context_length", 4096)):
        w.add_uint32(f"olmoe.{key}", v)
    w.add_float32("olmoe.attention.layer_norm_rms_epsilon", eps)
    w.add_float32("olmoe.rope.freq_base", 10000.0)
    w.add_bool("olmoe.expert_weights_norm", False)
    ones = np.ones(n_embd, dtype=np.float32)

    def add(name, arr, t):
        if t == gb.F32 and arr.dtype == np.float32:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, np.ascontiguousarray(arr), raw_dtype=gguf.GGMLQuantizationType(t))

    add("token_embd.weight", mat(embd_type, vocab, n_embd), embd_type)
    add("output_norm.weight", ones, gb.F32)
    add("output.weight", mat(head_type, vocab, n_embd), head_type)
    for L in range(n_layers):
        add(f"blk.{L}.attn_norm.weight", ones, gb.F32)
        for part in ("q", "k", "v", "output"):
            add(f"blk.{L}.attn_{part}.weight", mat(attn_type, n_embd, n_embd), attn_type)
        add(f"blk.{L}.attn_q_norm.weight", ones, gb.F32)
        add(f"blk.{L}.attn_k_norm.weight", ones, gb.F32)
        add(f"blk.{L}.ffn_norm.weight", ones, gb.F32)
        router = rng.normal(0.0, sigma, size=(n_expert, n_embd)).astype(np.float32)
        add(f"blk.{L}.ffn_gate_inp.weight", gb.quantize(router_type, router) if router_type != gb.F32 else router,
            router_type)
        for part, t, rows, cols in (("gate", gate_type, n_ff, n_embd), ("up", gate_type, n_ff, n_embd),
                                    ("down", down_type, n_embd, n_ff)):
            stacked = np.stack([mat(t, rows, cols, expert=True) for _ in range(n_expert)])  # E x rows x row_bytes
            add(f"blk.{L}.ffn_{part}_exps.weight", stacked, t)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def _centered_q4k(rows, cols, rng):
    """Random Q4_K blocks whose weights d sc_j (q - 7.5) are centred (dmin = 7.5 d and m_j = sc_j), so that a deep
    random-init model keeps finite, moving logits; element spread about 0.02 like the N(0, 0.02) configs."""
    out = gb.random_blocks(gb.Q4_K, rows, cols, rng)
    nb = cols // 256
    blk = out.reshape(rows, nb, 144)
    d = rng.uniform(5e-5, 1.2e-4, size=(rows, nb)).astype(np.float16)
    dmin = (d.astype(np.float32) * 7.5).astype(np.float16)
    sc = rng.integers(16, 64, size=(rows, nb, 8))
    blk[..., 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    blk[..., 2:4] = dmin.view(np.uint8).reshape(rows, nb, 2)
    blk[..., 4:16] = gb._pack_q4k_scales(sc, sc)
    return out
