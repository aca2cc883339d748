#!/usr/bin/env python
"""bench.py: Trochilus's OLMoE MoE layer on B200, tokens/s through one MoE layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--tokens T]
                    [--gate q4_k|q8_0] [--down q6_k|q4_k|q8_0]

Default workload: BASELINE.json configs[1]'s MoE layer: OLMoE-1B-7B shape (64 experts, top-8, hidden
2048, expert FFN 1024), Q4_K_M (gate/up Q4_K, down Q6_K), BF16 router, batch-1 decode (T = 1 token a
call). A step is one MoE-layer call (router -> top-8 -> dispatch -> gate/up/SwiGLU -> down -> id-ordered
combine -> residual add) on T tokens. 16 layers are resident in HBM (4.2 GB) and step i runs layer i % 16
on a fresh input row, so every step's 8 experts come from HBM, not from L2 (126 MB).

Arms:
  ours       libtrmoe.so through its C ABI. `value` = T * N / (device time per step); `e2e` = the same
             through tr_gpu_moe_layer with pinned host buffers (copies in and out inside the timed region);
             `roofline` = the dominant zone's algorithmic bytes / its CUDA-event time; `cpu_baseline` =
             Trochilus's own code (oracle/_ref, best SIMD tier, all host cores) on a bounded sample.
             `prefill` = configs[2]'s layer (2048 tokens, Q8_0) on the tensor-core road, same keys, its roofline
             the useful TFLOP/s over the dense TF32 peak (--prefill-tokens 0 skips it; --only-prefill prints it alone).
  reference  Trochilus's own CPU code on this box's host cores, same config (rank 0 only under torchrun).
--only-attention P prints only the decode attention backend's line (tr_gpu_attn_decode, Trochilus's gpu_attn.h on the
B200): one layer of OLMoE's 16 heads of 128 at a context of P positions, wall time per call through the host API,
its K and V bytes against the HBM peak, and Trochilus's own tr_attention_head on one host core beside it.
N > 1: one process per GPU (torchrun), expert parallel (trochilus_b200/ep.py): rank r holds experts
[64 r / N, 64 (r + 1) / N) and owns T tokens a step (weak scaling); each step routes them, sends their rows to the
experts' ranks and back with NCCL all-to-alls (padded blocks: no host sync), and combines. time = max over ranks,
`value` = all ranks' tokens / that time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from trochilus_b200 import gguf_blocks as gb  # noqa: E402

METRIC = "MoE-layer tokens/s (decode & prefill) OLMoE shape Q4_K/Q8_0; % of HBM/TC peak"
TYPES = {"q4_k": gb.Q4_K, "q8_0": gb.Q8_0, "q6_k": gb.Q6_K}
E, K_USED, H, F = 64, 8, 2048, 1024


def args_parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tokens", type=int, default=1)
    p.add_argument("--gate", default="q4_k", choices=["q4_k", "q8_0"])
    p.add_argument("--down", default="q6_k", choices=["q6_k", "q4_k", "q8_0"])
    p.add_argument("--layers", type=int, default=16)
    p.add_argument("--cpu-seconds", type=float, default=8.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--prefill-tokens", type=int, default=2048,
                   help="tokens of the prefill measurement added to the line (configs[2]'s layer); 0: skip it")
    p.add_argument("--prefill-steps", type=int, default=20)
    p.add_argument("--no-extra", action="store_true", help="skip the other configurations (\"configs\" key)")
    p.add_argument("--extra-cpu-seconds", type=float, default=2.0)
    p.add_argument("--ep-tokens", default="1,64",
                   help="N > 1: tokens a rank for the expert-parallel measurements reported under \"ep\" (\"\": none)")
    p.add_argument("--only-prefill", action="store_true", help="run and print only the prefill measurement")
    p.add_argument("--only-attention", type=int, default=0, metavar="P",
                   help="run and print only the decode attention measurement at a context of P positions")
    return p.parse_args()


def bytes_per_expert(gate, down):
    return 2 * F * gb.row_bytes(gate, H) + H * gb.row_bytes(down, F)


def host_layers(gate, down, n_host=2, n_routers=16):
    """n_host distinct layers of host GGUF bytes (random quant blocks with bounded scales) and n_routers
    BF16-rounded N(0, 0.02) routers."""
    lays = [gb.make_layer(1000 + i, E, H, F, gate, down, gb.BF16, mode="random") for i in range(n_host)]
    rng = np.random.Generator(np.random.PCG64(77))
    routers = [gb.quantize(gb.BF16, gb.round_to_bf16(rng.normal(0, 0.02, size=(E, H)).astype(np.float32)))
               for _ in range(n_routers)]
    return lays, routers


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, max, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def wait_first(self, limit_s=3.0):
        t0 = time.time()
        while self.proc and not self.rows and time.time() - t0 < limit_s:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([v.strip() for v in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_reference(args, gate, down, seconds, steps=None, warmup=0, tokens=None, bias=None, names=None, lay=None):
    """Trochilus's own code (oracle/_ref) on all host cores: tokens/s of one MoE layer on T tokens. Either a
    bounded time (seconds) or exactly `steps` layer calls after `warmup`. tokens, bias (the router's per-expert
    bias), names (gate, down) and lay (host layer) default to the bench's own workload."""
    from oracle.oracle import RefLib, make_desc
    T = args.tokens if tokens is None else tokens
    gname, dname = (args.gate, args.down) if names is None else names
    ref = RefLib()
    if lay is None:
        lays, routers = host_layers(gate, down, n_host=1, n_routers=1)
        lay = dict(lays[0])
        lay["router"] = routers[0]
    d, keep = make_desc(lay, H, F, K_USED, 0, gb.BF16, gate, down, bias)
    pool = ref.pool(0)
    st = ref.state(pool, d, T)
    rng = np.random.default_rng(5)
    xs = [rng.normal(size=(T, H)).astype(np.float32) for _ in range(16)]
    res = np.zeros((T, H), np.float32)
    for i in range(warmup):
        ref.moe_layer(d, xs[i % 16], res, pool=pool, state=st)
    n, t0 = 0, time.perf_counter()
    while True:
        ref.moe_layer(d, xs[n % 16], res, pool=pool, state=st)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    cores = ref.pool_size(pool)
    tier = ref.tier()
    ref.state_free(st)
    ref.pool_destroy(pool)
    return {"value": T * n / el, "unit": "tokens/s", "cores": cores, "kind": "reference",
            "sample": f"{n} MoE-layer calls of {T} token(s), {gname}/{dname}, BF16 router"
                      f"{', Zipf router bias' if bias is not None else ''}, {el:.1f} s, Trochilus tier {tier}, "
                      f"tr_pool of {cores} threads"}


def run_reference(args, rank, world):
    gate, down = TYPES[args.gate], TYPES[args.down]
    if rank != 0:
        return
    steps = max(args.steps // 20, 20)
    warm = max(args.warmup, 50)  # the reference's caches and thread pool settled (a call is well under a ms)
    r = cpu_reference(args, gate, down, None, steps=steps, warmup=warm)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": 1000.0 * args.tokens / r["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 lane contract / int64+f64",
            "data": "synthetic", "config": workload_config(args),
            "cpu_baseline": {"kind": "reference", "cores": r["cores"], "sample": r["sample"], "value": r["value"],
                             "unit": "tokens/s"},
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args):
    return {"workload": f"configs[1] MoE layer: OLMoE-1B-7B shape (E=64, top-8, H=2048, F=1024), gate/up "
                        f"{args.gate.upper()}, down {args.down.upper()}, BF16 router, {args.tokens}-token decode "
                        f"call", "tokens_per_step": args.tokens, "layers_resident": args.layers,
            "l2": "inputs larger than L2: each step runs the next of the resident layers (~261 MB each)",
            "weights": "random quant blocks with bounded f16 scales (synthetic), inputs N(0,1)"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def tf32_peak():
    """dense TF32 tensor peak: half the measured dense bf16 (cuBLAS) rate, the ratio of the two dense rates"""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"] / 2.0, "half of measured bf16"
    except (OSError, KeyError, ValueError):
        return 1590.0 / 2.0, "half of fallback bf16"


def run_prefill(args, dev, cpu_seconds):
    """configs[2]'s MoE layer: T = --prefill-tokens tokens, Q8_0 gate/up/down, BF16 router, on the tensor-core road
    (3xTF32 tcgen05 GEMMs). Two resident layers alternate (428 MB of weights each, larger than L2)."""
    import torch
    from trochilus_b200.moe import GpuMoe
    T, NL, steps = args.prefill_tokens, 2, max(args.prefill_steps, 1)
    m = GpuMoe(NL, E, K_USED, H, F, gb.BF16, gb.Q8_0, gb.Q8_0, max_tokens=T, device=dev)
    lays, routers = host_layers(gb.Q8_0, gb.Q8_0, n_host=NL, n_routers=NL)
    for l in range(NL):
        lay = dict(lays[l])
        lay["router"] = routers[l]
        m.set_layer(l, lay)
    del lays
    assert m.launches(T) == 7, "the prefill call did not take the tensor-core road"
    g = torch.Generator(device="cuda")
    g.manual_seed(4321)
    normed = torch.randn((NL, T, H), device="cuda", generator=g)
    x = torch.randn((T, H), device="cuda", generator=g)
    sp = torch.cuda.Stream()  # a stream of its own (handle 0 would mean the context's stream to the C API)
    torch.cuda.synchronize()
    for i in range(3):
        m.layer_dev(i % NL, normed[i % NL].data_ptr(), T, x.data_ptr(), None, stream=sp.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        clk.wait_first()
        torch.cuda.synchronize()
        e0.record(sp)
        for i in range(steps):
            m.layer_dev(i % NL, normed[i % NL].data_ptr(), T, x.data_ptr(), None, stream=sp.cuda_stream)
        e1.record(sp)
        torch.cuda.synchronize()
    m.check()
    ms = e0.elapsed_time(e1) / steps
    flops = 2.0 * T * K_USED * 3 * H * F + 2.0 * T * E * H
    tflops = flops / (ms / 1000.0) / 1e12
    peak, peak_kind = tf32_peak()
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(f"q8_0/q8_0/T{T}/trx_k_pf_gemm (gate/up + down)")
    except (OSError, ValueError):
        pass
    # e2e through the host-pointer call: normed and x in, x out, per call
    hn = torch.randn((T, H)).pin_memory()
    hx = torch.randn((T, H)).pin_memory()
    m.layer_ptrs(0, hn.data_ptr(), T, hx.data_ptr(), host=True)
    n_e2e = max(steps // 2, 2)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        m.layer_ptrs(i % NL, hn.data_ptr(), T, hx.data_ptr(), host=True)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    m.close()
    out = {"workload": f"configs[2] MoE layer: OLMoE shape, Q8_0 gate/up/down, BF16 router, {T}-token prefill call "
                       f"(2 resident layers alternating, 428 MB each)",
           "value": T / (ms / 1000.0), "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "warmup": 3,
           "dtype": "3xTF32 (fp32 semantics, 1e-5)",
           "roofline": {"bound": "tensor", "kernel": "trx_k_pf_gemm (gate/up + down)", "achieved": tflops,
                        "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak, "peak_kind": peak_kind,
                        "flops": flops, "issued_frac": 3.0 * tflops / peak,
                        "note": "useful flops of the whole layer call over its time; the tensor pipe issues 3x these "
                                "(hi.hi, hi.lo, lo.hi): issued_frac", "traffic": traffic,
                        "traffic_note": "dram read+write of the call's two GEMM launches (ncu, profiles/traffic.json)"},
           "e2e": {"value": T / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 2 * T * H * 4,
                   "d2h_bytes_per_step": T * H * 4},
           "clocks": clk.summary()}
    if cpu_seconds > 0:
        try:
            a = argparse.Namespace(**vars(args))
            a.tokens, a.gate, a.down = T, "q8_0", "q8_0"
            out["cpu_baseline"] = cpu_reference(a, gb.Q8_0, gb.Q8_0, cpu_seconds)
        except Exception as exc:
            out["cpu_baseline"] = {"value": None, "sample": f"unavailable: {exc}"}
    return out


def ep_launches(gate, down, rows):
    """our kernels a step of the expert-parallel layer: route 1; pack 2; experts: the fused kernel for up to 64
    received rows, else sort, gather, gate and up 2 each, SwiGLU, down 2, scatter; combine 1"""
    return 1 + 2 + (1 if rows <= 64 else 2 + 2 + 2 + 1 + 2 + 2) + 1


def run_ep(args, rank, world, dist, T=None, steps=None):
    import torch
    from trochilus_b200 import ep
    from trochilus_b200.moe import GpuMoe

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev)
    gate, down = TYPES[args.gate], TYPES[args.down]
    T = args.tokens if T is None else T
    NL = args.layers
    # max_tokens: every row a rank can receive in the padded exchange (world x T k), so its experts take one kernel
    m = GpuMoe(NL, E, K_USED, H, F, gb.BF16, gate, down, max_tokens=T * world * K_USED, device=dev)
    lays, routers = host_layers(gate, down, n_host=2, n_routers=NL)
    for l in range(NL):
        lay = dict(lays[l % len(lays)])
        lay["router"] = routers[l]
        m.set_layer(l, ep.local_layer(lay, E, rank, world))
    del lays
    st = torch.cuda.Stream()
    be = ep.GpuEpBackend(m, st)
    cap = T * K_USED
    g = torch.Generator(device="cuda")
    g.manual_seed(1234 + rank)
    with torch.cuda.stream(st):
        normed = torch.randn((NL, T, H), device="cuda", generator=g)
        x = torch.randn((T, H), device="cuda", generator=g)
        for i in range(max(args.warmup, 3)):
            ep.ep_layer(dist, be, i % NL, normed[i % NL], x, cap=cap)
    torch.cuda.synchronize()
    dist.barrier()
    steps = args.steps if steps is None else steps
    reps = max(steps // NL, 1)
    steps = reps * NL
    # a CUDA graph of NL layer calls (kernels and NCCL all-to-alls; the padded exchange has no host sync)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for l in range(NL):
            ep.ep_layer(dist, be, l, normed[l], x, cap=cap)
    torch.cuda.synchronize()
    dist.barrier()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    with Clocks(dev) as clk:
        clk.wait_first()
        torch.cuda.synchronize()
        start.record(cur)
        for _ in range(reps):
            graph.replay()
        end.record(cur)
        torch.cuda.synchronize()
    del graph  # graphs holding NCCL calls go before the process group does
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ms_step = ms / steps
    value = world * T / (ms_step / 1000.0)
    # bytes: each rank's distinct local experts hit per step (from the routing of every rank's tokens)
    with torch.cuda.stream(st):
        sel = be.route(0, normed[0], x)[0]
    allsel = [torch.empty_like(sel) for _ in range(world)]
    dist.all_gather(allsel, sel)
    ids = torch.cat(allsel).cpu().numpy()
    a, b = ep.expert_range(E, rank, world)
    u_local = len(set(int(e) for e in ids if a <= e < b))
    rank_bytes = u_local * bytes_per_expert(gate, down) + E * gb.row_bytes(gb.BF16, H) + 2 * T * H * 4
    tb = torch.tensor([float(rank_bytes)], device="cuda")
    dist.all_reduce(tb)
    peak, peak_kind = peaks()
    achieved = float(tb.item()) / world / (ms_step / 1000.0) / 1e9
    link_bytes = 2 * world * cap * H * 4 + world * cap * 4  # rows there and back, ids (padded blocks)
    # e2e: pinned host inputs in, the layer, x back, every step
    hn = torch.randn((16, T, H), generator=torch.Generator().manual_seed(99 + rank)).pin_memory()
    hx = torch.empty((T, H)).pin_memory()
    e2e_steps = max(min(steps, 2000), 10)
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(st):
        dn = torch.empty((T, H), device="cuda")
        for i in range(e2e_steps):
            dn.copy_(hn[i % 16], non_blocking=True)
            ep.ep_layer(dist, be, i % NL, dn, x, cap=cap)
            hx.copy_(x, non_blocking=True)
            st.synchronize()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device="cuda")
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    m.close()
    if rank != 0:
        return None
    cfg = workload_config(args)
    cfg["tokens_per_step"] = T
    cfg["parallelism"] = f"ep{world}"
    cfg["experts_per_gpu"] = E // world
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int32/int64+f64 (Q4_K), f32 (Q6_K/Q8_0 lane contract)",
            "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": "expert-parallel layer (route, pack, experts, combine + NCCL)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_gpu": float(tb.item()) / world,
                         "nvlink_bytes_per_gpu": link_bytes,
                         "nvlink_gbs_per_gpu": link_bytes / (ms_step / 1000.0) / 1e9},
            "cpu_baseline": None,
            "e2e": {"value": world * T * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4, "steps": e2e_steps},
            "gpu_launches": ep_launches(gate, down, world * T * K_USED) * steps, "clocks": clk.summary(),
            "timing": f"CUDA graph of {NL} expert-parallel layer calls (kernels + NCCL) replayed {reps} times; CUDA "
                      f"events, max over ranks"}
    return line


# The rest of the metric's configurations: BASELINE.json configs[3] (the isolated layer, all-Q4_K and all-Q8_0, Zipf
# router bias, T in {1, 8, 64, 512, 4096, 16384}), configs[1]'s Q4_K_M layer at more tokens, and configs[4]'s MoE
# step (64 sequences x 4 verify rows = 256 tokens, Q8_0): key, gate, down, tokens a call, Zipf router bias
EXTRA = tuple((f"{n}_zipf_T{t}", g, g, t, True) for n, g in (("q4k", "q4_k"), ("q8_0", "q8_0"))
              for t in (1, 8, 64, 512, 4096, 16384)) + \
        (("q4km_T8", "q4_k", "q6_k", 8, False), ("q4km_T64", "q4_k", "q6_k", 64, False),
         ("q8_0_T256_cfg4", "q8_0", "q8_0", 256, False))


def run_extra(args, dev, cpu_seconds):
    """Each EXTRA configuration on one GPU: CUDA graphs of 4 resident layer calls (two distinct weight sets, each
    larger than L2), the layer's algorithmic bytes and useful flops over its time, and Trochilus's CPU code on the
    same configuration for cpu_seconds."""
    import torch
    from trochilus_b200.moe import GpuMoe
    peak, peak_kind = peaks()
    out, host = {}, {}
    NLX = 4
    for key, gname, dname, T, zipf in EXTRA:
        gate, down = TYPES[gname], TYPES[dname]
        if (gate, down) not in host:  # one set of host layers per type pair
            host.clear()
            host[(gate, down)] = host_layers(gate, down, n_host=2, n_routers=NLX)
        lays, routers = host[(gate, down)]
        bias = gb.zipf_bias(6, E) if zipf else None
        m = GpuMoe(NLX, E, K_USED, H, F, gb.BF16, gate, down, max_tokens=T, device=dev)
        for l in range(NLX):
            lay = dict(lays[l % 2])
            lay["router"] = routers[l]
            m.set_layer(l, lay, bias)
        g = torch.Generator(device="cuda")
        g.manual_seed(4321 + T)
        normed = torch.randn((NLX, T, H), device="cuda", generator=g)
        x = torch.randn((T, H), device="cuda", generator=g)
        sp = torch.cuda.Stream()
        for i in range(3):
            m.layer_dev(i % NLX, normed[i % NLX].data_ptr(), T, x.data_ptr(), None, stream=sp.cuda_stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=sp):
            for l in range(NLX):
                m.layer_dev(l, normed[l].data_ptr(), T, x.data_ptr(), None,
                            stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        cur = torch.cuda.current_stream()  # the stream the replays run on
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        graph.replay()
        e1.record(cur)
        torch.cuda.synchronize()
        reps = max(3, min(400, int(300.0 / max(e0.elapsed_time(e1), 1e-3))))  # about 0.3 s timed
        with Clocks(dev) as clk:
            clk.wait_first()
            torch.cuda.synchronize()
            e0.record(cur)
            for _ in range(reps):
                graph.replay()
            e1.record(cur)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * NLX)
        del graph
        sel = torch.zeros((NLX, T * K_USED), dtype=torch.int64, device="cuda")
        sel_w = torch.zeros((T * K_USED,), device="cuda")
        for l in range(NLX):
            m.layer_dev(l, normed[l].data_ptr(), T, x.data_ptr(), {"sel_id": sel[l].data_ptr(), "sel_w": sel_w.data_ptr()},
                        stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        m.check()
        U = float(np.mean([len(np.unique(r)) for r in sel.cpu().numpy()]))
        nbytes = U * bytes_per_expert(gate, down) + E * gb.row_bytes(gb.BF16, H) + 2 * T * H * 4
        flops = 2.0 * T * K_USED * 3 * H * F + 2.0 * T * E * H
        kname, nl = m.kernel_name(T), m.launches(T)
        m.close()
        entry = {"value": T / (ms / 1000.0), "unit": "tokens/s", "tokens_per_step": T, "ms_per_step": ms,
                 "steps": reps * NLX, "warmup": 3 * NLX + 3, "gate": gname, "down": dname, "zipf_router_bias": zipf,
                 "kernel": kname or f"{nl} kernels a call", "gpu_launches_per_step": nl,
                 "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1000.0) / 1e9, "peak": peak, "unit": "GB/s",
                              "frac": nbytes / (ms / 1000.0) / 1e9 / peak, "peak_kind": peak_kind,
                              "algorithmic_bytes": nbytes, "distinct_experts": U, "traffic": None,
                              "useful_tflops": flops / (ms / 1000.0) / 1e12},
                 "clocks": clk.summary()}
        if cpu_seconds > 0:
            try:
                lay = dict(lays[0])
                lay["router"] = routers[0]
                entry["cpu_baseline"] = cpu_reference(args, gate, down, cpu_seconds, tokens=T, bias=bias,
                                                      names=(gname, dname), lay=lay)
            except Exception as exc:  # the prebuilt reference is missing on this box
                entry["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                                         "sample": f"unavailable: {exc}"}
        out[key] = entry
    return out


def run_ours(args, rank, world, dist):
    import torch
    from trochilus_b200.moe import GpuMoe

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev)
    gate, down = TYPES[args.gate], TYPES[args.down]
    T, NL = args.tokens, args.layers
    m = GpuMoe(NL, E, K_USED, H, F, gb.BF16, gate, down, max_tokens=T, device=dev)
    lays, routers = host_layers(gate, down, n_host=2, n_routers=NL)
    for l in range(NL):
        lay = dict(lays[l % len(lays)])
        lay["router"] = routers[l]
        m.set_layer(l, lay)
    del lays
    g = torch.Generator(device="cuda")
    g.manual_seed(1234 + rank)
    normed = torch.randn((NL, T, H), device="cuda", generator=g)
    x = torch.randn((T, H), device="cuda", generator=g)
    side = torch.cuda.Stream()

    def capture(parts, n=NL):
        """a CUDA graph of n layer calls (call i: layer i mod NL on input row i mod NL): whole calls (parts None, the
        road a user's call takes: one fused kernel for a short pass) or the given parts of the multi-kernel road"""
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            sp = torch.cuda.current_stream().cuda_stream
            for i in range(n):
                l = i % NL
                if parts is None:
                    m.layer_dev(l, normed[l].data_ptr(), T, x.data_ptr(), None, stream=sp)
                else:
                    for part in parts:
                        m.layer_part(l, part, normed[l].data_ptr(), T, x.data_ptr(), stream=sp)
        return graph

    # warm-up outside graphs (first touches), then the graphs
    for i in range(max(args.warmup, 3)):
        m.layer_dev(i % NL, normed[i % NL].data_ptr(), T, x.data_ptr(), None,
                    stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    parts_of = {"route": [0], "gate_up": [0, 1], "act_prep": [0, 1, 2], "parts": [0, 1, 2, 3], "call": None}
    graphs = {k: capture(v) for k, v in parts_of.items()}
    steps = args.steps
    # a short run (up to 4 NL steps) is one graph of exactly its K calls, so that the timed region holds one graph
    # launch; a longer one replays the NL-call graph K // NL times and a graph of the rest. Every graph the timed
    # region replays is replayed (uploaded) before it.
    whole = capture(None, steps) if steps <= 4 * NL else None
    reps, tail_n = (0, 0) if whole is not None else (steps // NL, steps % NL)
    tail = capture(None, tail_n) if tail_n else None
    for _ in range(max(args.warmup // NL, 3)):
        graphs["call"].replay()
        for g_ in (whole, tail):
            if g_ is not None:
                g_.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        clk.wait_first()
        torch.cuda.synchronize()
        start.record(stream)
        if whole is not None:
            whole.replay()
        for _ in range(reps):
            graphs["call"].replay()
        if tail is not None:
            tail.replay()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / steps
    value = world * T / (ms_step / 1000.0)

    # zones: each part's marginal device time per layer call, from graphs of parts 0..z (CUDA events on the
    # replaying stream), warm replays first
    cum = {}
    for k in ("route", "gate_up", "act_prep", "parts"):
        for _ in range(3):
            graphs[k].replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(max(reps, 1)):
            graphs[k].replay()
        e1.record(stream)
        torch.cuda.synchronize()
        cum[k] = e0.elapsed_time(e1) / (max(reps, 1) * NL)
    zone_ms = {"router": cum["route"], "gate_up": cum["gate_up"] - cum["route"],
               "act_prep": cum["act_prep"] - cum["gate_up"], "down": cum["parts"] - cum["act_prep"]}
    del graphs, tail, whole
    # distinct experts per call (computed from the routing each call makes)
    sel = torch.zeros((NL, T * K_USED), dtype=torch.int64, device="cuda")
    sel_w = torch.zeros((T * K_USED,), device="cuda")
    for l in range(NL):
        m.layer_dev(l, normed[l].data_ptr(), T, x.data_ptr(), {"sel_id": sel[l].data_ptr(), "sel_w": sel_w.data_ptr()},
                    stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    used = [len(np.unique(r)) for r in sel.cpu().numpy()]
    U = float(np.mean(used))
    bpe = bytes_per_expert(gate, down)
    router_bytes = E * gb.row_bytes(gb.BF16, H)
    layer_bytes = U * bpe + router_bytes + 2 * T * H * 4
    gate_bytes = U * 2 * F * gb.row_bytes(gate, H) + T * H * 4 + T * K_USED * F * 4
    down_bytes = U * H * gb.row_bytes(down, F) + T * K_USED * F * 4 + 2 * T * H * 4
    zone_bytes = {"router": router_bytes + T * H * 4, "gate_up": gate_bytes,
                  "act_prep": 2 * T * K_USED * F * 4, "down": down_bytes}
    peak, peak_kind = peaks()
    launches = m.launches(T)
    if launches == 1:  # one kernel per call: it is the dominant (only) kernel, its bytes the layer's
        dom = m.kernel_name(T)
        zone_bytes[dom] = layer_bytes
        zone_ms[dom] = ms_step
    else:
        dom = max(zone_ms, key=lambda z: zone_ms[z])
    achieved = zone_bytes[dom] / (zone_ms[dom] / 1000.0) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(f"{args.gate}/{args.down}/T{T}/{dom}")
    except (OSError, ValueError):
        pass
    layer_ms = sum(zone_ms[z] for z in ("router", "gate_up", "act_prep", "down"))

    # e2e through the public host-pointer call, pinned buffers, copies inside the timed region
    n_in = 16
    hn = torch.randn((n_in, T, H), generator=torch.Generator().manual_seed(99)).pin_memory()
    hx = torch.randn((T, H)).pin_memory()
    # (at least 2000 calls, about 80 ms: the host road's steady state, which a short run's handful of calls misses)
    e2e_steps = max(min(args.steps, 4000), 2000)
    hptr, xptr = [hn[j].data_ptr() for j in range(n_in)], hx.data_ptr()  # (no tensor indexing inside the loop)
    for i in range(max(args.warmup, 200)):  # untimed: the host road's first calls run slower (about 8 ms of them)
        m.layer_ptrs(i % NL, hptr[i % n_in], T, xptr, host=True)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        m.layer_ptrs(i % NL, hptr[i % n_in], T, xptr, host=True)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": world * T * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 2 * T * H * 4,
           "d2h_bytes_per_step": T * H * 4, "steps": e2e_steps}

    prefill = None
    if world == 1 and args.prefill_tokens > 0:
        prefill = run_prefill(args, dev, 0 if args.no_cpu_baseline else args.cpu_seconds)
    extra = None
    if world == 1 and not args.no_extra:
        extra = run_extra(args, dev, 0 if args.no_cpu_baseline else args.extra_cpu_seconds)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_reference(args, gate, down, args.cpu_seconds)
        except Exception as exc:  # the prebuilt reference is missing on this box
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {exc}"}
    m.close()
    if rank != 0:
        return None
    cfg = workload_config(args)
    if world > 1:
        cfg["parallelism"] = f"dp{world}"
        cfg["replicas"] = ("each GPU holds every expert of the 16 layers (4.2 GB of its 180 GB) and serves its own "
                           "token stream: no data-path collective")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int32/int64+f64 (Q4_K), f32 (Q6_K/Q8_0 lane contract)",
            "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes": zone_bytes[dom], "avg_ms": zone_ms[dom]},
            "layer_roofline": {"achieved": layer_bytes / (ms_step / 1000.0) / 1e9, "unit": "GB/s",
                               "frac": layer_bytes / (ms_step / 1000.0) / 1e9 / peak, "bytes": layer_bytes,
                               "distinct_experts": U,
                               "multikernel_zone_ms": {z: zone_ms[z] for z in ("router", "gate_up", "act_prep", "down")},
                               "multikernel_ms": layer_ms},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * steps, "clocks": clk.summary(),
            "prefill": prefill, "configs": extra,
            "timing": (f"one CUDA graph of the {steps} layer calls" if steps <= 4 * NL else
                       f"CUDA graphs of {NL} layer calls replayed (+ a graph of the last {tail_n})") +
                      "; zones from graphs of parts 0..z"}
    return line


def run_attention(args):
    """decode attention through the host API: one layer, 16 heads of 128, P positions in the cache, a decode token
    at position P (its k and v stored, positions 0..P attended); the reference's tr_attention_head on one host core
    for the same shape"""
    from trochilus_b200.moe import GpuAttn
    n_head, hd, P = 16, 128, args.only_attention
    rng = np.random.default_rng(3)
    kv = rng.normal(size=(P + 1, n_head * hd)).astype(np.float32)
    q = rng.normal(size=n_head * hd).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    a = GpuAttn(1, n_head, P + 1)
    a.write(0, 0, kv[:P], kv[:P])
    for _ in range(max(args.warmup, 3)):
        a.decode(0, P, q, kv[P], kv[P], scale)
    steps = max(min(args.steps, 2000), 10)
    with Clocks(0) as clk:
        clk.wait_first()
        t0 = time.perf_counter()
        for _ in range(steps):
            out = a.decode(0, P, q, kv[P], kv[P], scale)
        sec = (time.perf_counter() - t0) / steps
    a.close()
    cache_bytes = 2 * n_head * (P + 1) * hd * 4
    peak, peak_kind = peaks()
    achieved = cache_bytes / sec / 1e9
    cpu = None
    try:
        import ctypes as C
        from oracle.oracle import RefLib
        L = RefLib().lib
        L.tr_attention_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                        C.c_int64, C.c_float, C.c_void_p, C.c_void_p]
        keys = np.ascontiguousarray(kv)
        scores = np.zeros(P + 1, dtype=np.float32)
        ref = np.zeros((n_head, hd), dtype=np.float32)
        reps, c0 = 0, time.perf_counter()
        while time.perf_counter() - c0 < min(args.cpu_seconds, 5.0) or reps == 0:
            for h in range(n_head):
                L.tr_attention_head(q[h * hd:].ctypes.data, keys.ctypes.data, keys.ctypes.data, n_head * hd, h * hd,
                                    P + 1, hd, scale, scores.ctypes.data, ref[h].ctypes.data)
            reps += 1
        cpu_us = (time.perf_counter() - c0) / reps * 1e6
        same = bool(np.array_equal(ref.view(np.uint32), out.view(np.uint32)))
        cpu = {"value": cpu_us, "unit": "us", "cores": 1, "kind": "reference",
               "sample": f"{reps} calls of tr_attention_head x {n_head} heads, best tier, one thread",
               "same_bits_as_gpu": same}
    except Exception as exc:  # the reference library is a checker: its absence leaves the baseline out
        cpu = {"value": None, "sample": f"unavailable: {exc}"}
    line = {"metric": f"decode attention, us per layer call (16 heads x 128, {P} cached positions)",
            "value": sec * 1e6, "unit": "us", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
            "higher_is_better": False, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "tr_gpu_attn_decode through the host API (q, k, v in, out back)",
                       "context": P, "n_head": n_head, "head_dim": hd},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "algorithmic_bytes": cache_bytes,
                         "note": "wall time per host call (copies, five launches, synchronisation) over K and V bytes"},
            "cpu_baseline": cpu, "clocks": clk.summary(), "vs_baseline": None}
    print(json.dumps(line), flush=True)


def main():
    args = args_parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1 and args.impl == "ours":
        import datetime

        import torch
        import torch.distributed as dist_
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist_.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = dist_
    if args.only_attention > 0:
        import torch
        torch.cuda.set_device(0)
        run_attention(args)
    elif args.only_prefill:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(run_prefill(args, 0, 0 if args.no_cpu_baseline else args.cpu_seconds)), flush=True)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        # N = 1: the decode layer call on one GPU. N > 1: the same call on N data-parallel replicas (the headline:
        # one-token decode streams are independent), then the north star's expert-parallel layer (64/N experts a
        # GPU, NCCL all-to-all dispatch and combine) at one token a rank and at a throughput batch, under "ep"
        line = run_ours(args, rank, world, dist)
        if world > 1 and args.ep_tokens:
            ep_lines = {}
            for t_ep in [int(v) for v in args.ep_tokens.split(",") if v]:
                r = run_ep(args, rank, world, dist, T=t_ep, steps=min(args.steps, 2048 if t_ep == 1 else 256))
                if r is not None:
                    ep_lines[f"T{t_ep}"] = {k: r[k] for k in ("value", "unit", "ms_per_step", "steps", "roofline",
                                                              "e2e", "gpu_launches", "timing")}
                    ep_lines[f"T{t_ep}"]["tokens_per_rank"] = t_ep
            if line is not None:
                line["ep"] = ep_lines
        if line is not None:
            print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
