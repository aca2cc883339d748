"""Reads the fused MoE-layer kernel's timeline (tr_gpu_moe_trace) into per-phase statistics.

    python -m trochilus_b200.timeline [--gate q4_k] [--down q6_k] [--tokens 1] [--calls 20] [--layers 2]

runs a few calls on synthetic weights and prints, over the CTAs of the last call, when each phase ended
(microseconds after the earliest CTA start): router/preparation done, routing seen, copies armed, gate/up
done, first down chunk ready, down done, end.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def summarize(tr: np.ndarray) -> dict:
    t0 = tr[:, 0][tr[:, 0] > 0].min()

    def stat(col_vals):
        v = col_vals[(col_vals > 0) & (col_vals >= t0)]
        if v.size == 0:
            return None
        u = (v.astype(np.float64) - float(t0)) / 1000.0
        return {"min": round(float(u.min()), 2), "median": round(float(np.median(u)), 2), "max": round(float(u.max()), 2)}

    names = (("start", 0), ("router_prep_work_done", 62), ("h_published", 59), ("route_done", 60), ("producer_mask_done", 61), ("producer_on", 49),
             ("producer_walks_set", 51), ("producer_first_copies_out", 3),
             ("phase_a_done", 1), ("sorted_w0", 48), ("routing_seen", 2), ("gate_up_done_w0", 4),
             ("down_first_ready_w0", 5), ("down_done_w0", 6), ("end", 52))
    out = {"ctas": int(tr.shape[0]), **{n: stat(tr[:, slot]) for n, slot in names}}
    med = lambda slot: (stat(tr[:, slot]) or {}).get("median")
    # per chunk of consumer warp 0: (data ready, rows multiplied, counted and released)
    out["cycles_route_token_w0"] = int(np.median(tr[:, 7]))
    out["cycles_sort_w0"] = int(np.median(tr[:, 63]))
    out["w0_gate_up_chunks"] = [(med(8 + j), med(40 + j), med(16 + j)) for j in range(8)]
    out["w0_down_chunks"] = [(med(24 + j), None, med(32 + j)) for j in range(8)]
    cyc = lambda slot: int(np.median(tr[:, slot]))
    # cycles since the CTA's start (thread 0): route count seen, logits loaded, routed, sort begun / done, barrier
    out["cycles_w0"] = {n: cyc(sl) for n, sl in (("route_cnt_seen", 53), ("logits_loaded", 54), ("routed", 55),
                                                 ("sort_begin", 56), ("sorted", 57), ("bar1", 58))}
    return out


def main():
    import torch

    from trochilus_b200 import gguf_blocks as gb
    from trochilus_b200.moe import GpuMoe
    ap = argparse.ArgumentParser()
    ap.add_argument("--gate", default="q4_k")
    ap.add_argument("--down", default="q6_k")
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--calls", type=int, default=20)
    ap.add_argument("--layers", type=int, default=2, help="resident layers, called in turn (16: weights from HBM)")
    ap.add_argument("--per-cta", action="store_true", help="also print each CTA's gate/up-done and end times")
    ap.add_argument("--dump", default=None, help="also save the raw trace (CTAs x 64 slots) to this .npy file")
    a = ap.parse_args()
    types = {"q4_k": gb.Q4_K, "q8_0": gb.Q8_0, "q6_k": gb.Q6_K}
    gt, dt, T = types[a.gate], types[a.down], a.tokens
    m = GpuMoe(a.layers, 64, 8, 2048, 1024, gb.BF16, gt, dt, max_tokens=T)
    for l in range(a.layers):
        m.set_layer(l, gb.make_layer(50 + l, 64, 2048, 1024, gt, dt, gb.BF16, mode="random"))
    normed = torch.randn((a.calls, T, 2048), device="cuda")
    x = torch.randn((T, 2048), device="cuda")
    m.trace(True)
    for i in range(a.calls):
        m.layer_dev(i % a.layers, normed[i].data_ptr(), T, x.data_ptr(), None, stream=torch.cuda.current_stream().cuda_stream)
    tr = m.trace_read()
    m.check()
    print(json.dumps({"gate": a.gate, "down": a.down, "tokens": T, **summarize(tr)}))
    if a.dump:
        np.save(a.dump, tr)
    if a.per_cta:
        t0 = tr[:, 0][tr[:, 0] > 0].min()
        rel = lambda c: [round((float(v) - t0) / 1000.0, 2) if v > t0 else None for v in tr[:, c]]
        print(json.dumps({"gate_up_done": rel(4), "down_first": rel(5), "end": rel(52), "start": rel(0)}))
    m.close()


if __name__ == "__main__":
    main()
