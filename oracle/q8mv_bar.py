"""The reference's GPU bar for the dense Q8_0 GEMV, beside this library's kernel-level tr_matmul on the same shapes.

Trochilus's only GPU kernel on a matmul is q8_mv (tests/bench_gpu_q8.c:1-53, kernel text :269-319): a bit-exact Q8_0
GEMV written as PTX text that the driver compiles at run time, measured by its author on an RTX 4070 Laptop
(docs/MEASUREMENTS.md:2913-2920). `make -C oracle REF=<tree> q8mv` builds that program from its source into
oracle/_ref/bench_gpu_q8; this script runs its `time` mode on this machine's GPU and then times tr_matmul (the call
a relinked engine makes for q, k, v, o and the output head) on the same shapes, the same way as its round trip (b):
pinned x to the device, the product, y back, the stream waited for, host clock, median of the runs.

The model file is synthetic: bench_gpu_q8's time mode reads blk.L.attn_{q,k,v,output}.weight of 16 layers,
output.weight and token_embd.weight (tests/bench_gpu_q8.c:838-870), all Q8_0. Random Q8_0 blocks stand in for the
real checkpoint (the timing does not depend on the values). Test and measurement infrastructure: nothing in the
package imports this.

    python oracle/q8mv_bar.py [--runs 50] [--out results.json]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from trochilus_b200 import gguf_blocks as gb  # noqa: E402

H, V, LAYERS = 2048, 50304, 16
ROLES = ("attn_q", "attn_k", "attn_v", "attn_output")


def write_dense_q8(path: str, seed: int = 5150) -> dict:
    """the tensors bench_gpu_q8's time mode reads, random Q8_0 blocks; returns them (name -> rows x row_bytes)"""
    import gguf
    rng = np.random.Generator(np.random.PCG64(seed))
    mats = {}
    w = gguf.GGUFWriter(path, "olmoe")
    w.add_uint32("olmoe.block_count", LAYERS)
    w.add_uint32("olmoe.embedding_length", H)
    w.add_float32("olmoe.attention.layer_norm_rms_epsilon", 1e-5)

    def add(name, rows):
        a = gb.random_blocks(gb.Q8_0, rows, H, rng)
        mats[name] = a
        w.add_tensor(name, a, raw_dtype=gguf.GGMLQuantizationType(gb.Q8_0))

    add("token_embd.weight", V)
    w.add_tensor("output_norm.weight", np.ones(H, dtype=np.float32))
    add("output.weight", V)
    for L in range(LAYERS):
        w.add_tensor(f"blk.{L}.attn_norm.weight", np.ones(H, dtype=np.float32))
        for r in ROLES:
            add(f"blk.{L}.{r}.weight", H)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return mats


def time_ours(mats: dict, runs: int) -> dict:
    """tr_matmul round trips on the shapes of bench_gpu_q8's time mode, the weights rotating as there (every product
    reads a matrix that is not in L2)"""
    import torch
    from trochilus_b200.moe import TrMat, lib, last_error

    attn = [mats[f"blk.{L}.{r}.weight"] for L in range(LAYERS) for r in ROLES]
    qkv = [np.ascontiguousarray(np.concatenate([mats[f"blk.{L}.{r}.weight"] for r in ROLES[:3]])) for L in range(LAYERS)]
    head = [mats["output.weight"], mats["token_embd.weight"]]
    x = torch.randn((1, H), generator=torch.Generator().manual_seed(42)).pin_memory()
    y = torch.empty((1, V)).pin_memory()
    out = {}
    for name, group, rows in (("2048 x 2048", attn, H), ("6144 x 2048", qkv, 3 * H), ("50304 x 2048", head, V)):
        ms = [TrMat(gb.Q8_0, rows, H, a.ctypes.data) for a in group]
        for m in ms:  # first sight uploads the matrix; then warm calls
            lib().tr_matmul(None, C.byref(m), x.data_ptr(), 1, y.data_ptr())
        for i in range(2 * len(ms)):
            lib().tr_matmul(None, C.byref(ms[i % len(ms)]), x.data_ptr(), 1, y.data_ptr())
        err = last_error()
        if err:
            raise RuntimeError(f"tr_matmul: {err}")
        t = []
        for i in range(runs):
            t0 = time.perf_counter()
            lib().tr_matmul(None, C.byref(ms[i % len(ms)]), x.data_ptr(), 1, y.data_ptr())
            t.append(time.perf_counter() - t0)
        us = float(np.median(t)) * 1e6
        nbytes = rows * gb.row_bytes(gb.Q8_0, H)
        out[name] = {"round_trip_us": us, "GBps": nbytes / (us * 1e-6) / 1e9, "matrices": len(ms), "runs": runs}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--runs", type=int, default=50)
    ap.add_argument("--out", default=None, help="also write the results as JSON here")
    a = ap.parse_args()
    exe = os.path.join(HERE, "_ref", "bench_gpu_q8")
    if not os.path.exists(exe):
        raise SystemExit(f"{exe} is missing: make -C oracle REF=<the reference tree> q8mv")
    res = {}
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "dense_q8_0.gguf")
        t0 = time.time()
        mats = write_dense_q8(path)
        res["gguf_seconds"] = time.time() - t0
        p = subprocess.run([exe, "time", "--model", path, "--runs", str(a.runs)], capture_output=True, text=True,
                           timeout=600)
        res["reference_q8_mv"] = {"rc": p.returncode, "stdout": p.stdout.splitlines(), "stderr": p.stderr[-2000:]}
        print(p.stdout)
        res["ours_tr_matmul"] = time_ours(mats, a.runs)
    if a.out:
        os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)
    print(json.dumps(res["ours_tr_matmul"], indent=1))
    if res["reference_q8_mv"]["rc"] != 0:
        raise SystemExit(f"bench_gpu_q8 exited {res['reference_q8_mv']['rc']}")


if __name__ == "__main__":
    main()
