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
