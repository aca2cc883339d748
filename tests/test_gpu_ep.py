"""Expert parallelism on the GPU (trochilus_b200/ep.py with libtrmoe.so's tr_gpu_moe_ep_pack, _experts_dev and
_ep_combine): every rank holds E / N experts and routes its own tokens; each rank's output must be bit for bit the
one-GPU layer's on its tokens (the oracle's, and the exact road's of a context holding every expert).

On one GPU the ranks are emulated in one process (the all-to-alls done by slicing); with two or more GPUs a second
test runs real NCCL ranks, one process per GPU."""
import os
import socket

import numpy as np
import pytest

from oracle.oracle import make_desc
from tests.golden.cases import same_bits
from trochilus_b200 import ep
from trochilus_b200 import gguf_blocks as gb

pytestmark = pytest.mark.gpu
E, K, H, F = 64, 8, 2048, 1024


def _contexts(torch, lay, bias, world, T, rt, gt, dt, device=0):
    from trochilus_b200.moe import GpuMoe
    ms = []
    for r in range(world):
        # max_tokens covers every row a rank can receive (world x T k): up to 64 rows take the fused kernel
        m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=T * world * K, device=device)
        m.set_layer(0, ep.local_layer(lay, E, r, world), bias)
        ms.append(m)
    return ms


@pytest.mark.parametrize("world,padded,step", [(2, False, 2), (4, True, 2), (2, True, 1), (2, False, 1), (4, False, 0)])
@pytest.mark.parametrize("rt,gt,dt", [(gb.BF16, gb.Q4_K, gb.Q6_K), (gb.F32, gb.Q8_0, gb.Q8_0)])
def test_ep_emulated_ranks_match_oracle(cuda, oracle, world, padded, step, rt, gt, dt):
    """rank r has 1 + step r tokens: the experts' rows of a rank take the fused kernel (routing given, padding rows
    without an expert) or the kernel-level road, depending on how many arrive"""
    torch = cuda
    lay = gb.make_layer(808 + world, E, H, F, gt, dt, rt, mode="random")
    bias = gb.zipf_bias(6, E)
    d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt, bias)
    Ts = [1 + step * r for r in range(world)]
    ms = _contexts(torch, lay, bias, world, max(Ts), rt, gt, dt)
    st = torch.cuda.Stream()
    bes = [ep.GpuEpBackend(m, st) for m in ms]
    rng = np.random.default_rng(world * 10 + gt)
    normeds = [rng.normal(size=(T, H)).astype(np.float32) for T in Ts]
    xs = [rng.normal(size=(T, H)).astype(np.float32) for T in Ts]
    for rep in range(2):
        torch.cuda.synchronize()
        with torch.cuda.stream(st):  # the kernels' stream is the one torch's copies and slices run on
            dn = [torch.from_numpy(n).cuda() for n in normeds]
            dx = [torch.from_numpy(x.copy()).cuda() for x in xs]
            ffn = [torch.full((T, H), float("nan"), device="cuda") for T in Ts]
            routed = ep.ep_layer_emulated(bes, 0, dn, dx, ffn, padded=padded)
        torch.cuda.synchronize()
        for r in range(world):
            want = oracle.moe_layer(d, normeds[r], xs[r])
            assert same_bits(routed[r][0].cpu().numpy().reshape(-1, K), want["sel_id"]), (r, rep)
            assert same_bits(routed[r][1].cpu().numpy().reshape(-1, K), want["sel_w"]), (r, rep)
            assert same_bits(dx[r].cpu().numpy(), want["x"]), (r, rep)
            assert same_bits(ffn[r].cpu().numpy(), want["ffn_out"]), (r, rep)
    for m in ms:
        m.check()
        m.close()


def test_ep_emulated_long_pass_matches_exact_road(cuda):
    """100 tokens a rank (the many-token router, rows of every expert crossing ranks), against a context holding
    every expert on the exact road"""
    torch = cuda
    from trochilus_b200.moe import GpuMoe
    rt, gt, dt, world, T = gb.BF16, gb.Q8_0, gb.Q6_K, 2, 100
    lay = gb.make_layer(4711, E, H, F, gt, dt, rt, mode="random")
    full = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=T)
    full.set_layer(0, lay)
    ms = _contexts(torch, lay, None, world, T, rt, gt, dt)
    st = torch.cuda.Stream()
    bes = [ep.GpuEpBackend(m, st) for m in ms]
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    dn = [torch.randn((T, H), device="cuda", generator=g) for _ in range(world)]
    x0 = [torch.randn((T, H), device="cuda", generator=g) for _ in range(world)]
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        dx = [x.clone() for x in x0]
        ep.ep_layer_emulated(bes, 0, dn, dx)
    torch.cuda.synchronize()
    for r in range(world):
        want = x0[r].clone()
        full.layer_dev(0, dn[r].data_ptr(), T, want.data_ptr(), None, stream=st.cuda_stream)
        torch.cuda.synchronize()
        assert same_bits(dx[r].cpu().numpy(), want.cpu().numpy()), r
    for m in ms + [full]:
        m.close()


def _nccl_worker(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from trochilus_b200.moe import GpuMoe
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rt, gt, dt = gb.BF16, gb.Q4_K, gb.Q6_K
        lay = gb.make_layer(2024, E, H, F, gt, dt, rt, mode="random")
        m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=2 * world * K, device=rank)  # every row it can receive
        m.set_layer(0, ep.local_layer(lay, E, rank, world))
        st = torch.cuda.Stream()
        be = ep.GpuEpBackend(m, st)
        rng = np.random.default_rng(rank)
        T = 1 + rank
        normed = rng.normal(size=(T, H)).astype(np.float32)
        x = rng.normal(size=(T, H)).astype(np.float32)
        d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt)
        want = Oracle().moe_layer(d, normed, x)
        ok = True
        for padded in (True, False):
            with torch.cuda.stream(st):
                dx = torch.from_numpy(x.copy()).cuda()
                ep.ep_layer(dist, be, 0, torch.from_numpy(normed).cuda(), dx, cap=world * K if padded else None)
            torch.cuda.synchronize()
            ok = ok and same_bits(dx.cpu().numpy(), want["x"])
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
        m.close()
    finally:
        dist.destroy_process_group()


def test_ep_nccl_ranks_match_oracle(cuda, tmp_path):
    torch = cuda
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU: the NCCL ranks need two or more (the emulated ranks above cover the kernels)")
    import torch.multiprocessing as mp
    world = min(n, 4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_nccl_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", r


def _peer_worker(rank, world, port, out_dir):
    """The expert-parallel layer over peer memory (ep.PeerEp): rows and outputs cross NVLink as stores, no NCCL on
    the data path; eager calls and a CUDA graph of a whole call, each rank's output against the oracle"""
    import datetime

    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from trochilus_b200.moe import GpuMoe
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ok = True
    try:
        rt, gt, dt = gb.BF16, gb.Q4_K, gb.Q6_K
        lay = gb.make_layer(2025, E, H, F, gt, dt, rt, mode="random")
        cap = 2 * K  # every rank sends at most 2 tokens x k rows
        m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=world * cap, device=rank)
        m.set_layer(0, ep.local_layer(lay, E, rank, world))
        st = torch.cuda.Stream()
        pe = ep.PeerEp(dist, m, cap, st)
        d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt)
        orc = Oracle()
        rng = np.random.default_rng(rank + 10)
        # the oracle's answers first: the ranks then reach the exchange together (its waits are bounded at 10 s)
        cases = []
        for call in range(3):
            T = 1 + (rank + call) % 2
            normed = rng.normal(size=(T, H)).astype(np.float32)
            x = rng.normal(size=(T, H)).astype(np.float32)
            cases.append((normed, x, orc.moe_layer(d, normed, x)))
        graph_cases = []
        for rep in range(2):
            normed = rng.normal(size=(2, H)).astype(np.float32)
            x = rng.normal(size=(2, H)).astype(np.float32)
            graph_cases.append((normed, x, orc.moe_layer(d, normed, x)["x"]))
        dist.barrier()
        for call, (normed, x, want) in enumerate(cases):
            dn = torch.from_numpy(normed).cuda()
            dx = torch.from_numpy(x.copy()).cuda()
            sid, sw = pe.layer(0, dn, dx)
            torch.cuda.synchronize()
            try:
                m.check()  # a wait that gave up says which flag
            except RuntimeError as exc:
                with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
                    f.write(f"call {call}: {exc}")
                raise
            ok = ok and same_bits(dx.cpu().numpy(), want["x"]) and same_bits(sid.cpu().numpy().reshape(-1, K),
                                                                              want["sel_id"])
        # a CUDA graph of one call, replayed twice on fresh inputs
        T = 2
        dn = torch.zeros((T, H), device="cuda")
        dx = torch.zeros((T, H), device="cuda")
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            pe.layer(0, dn, dx)
        for normed, x, want_x in graph_cases:
            dn.copy_(torch.from_numpy(normed))
            dx.copy_(torch.from_numpy(x))
            torch.cuda.synchronize()
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            ok = ok and same_bits(dx.cpu().numpy(), want_x)
        del g
        m.check()
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
        m.close()
    finally:
        dist.destroy_process_group()


def test_ep_peer_memory_matches_oracle(cuda, tmp_path):
    torch = cuda
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU: the peer-memory exchange needs two or more")
    import torch.multiprocessing as mp
    world = min(n, 4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    try:
        mp.spawn(_peer_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    finally:
        for r in range(world):
            p = tmp_path / f"rank{r}"
            print(f"rank {r}:", p.read_text() if p.exists() else "(no record)")
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", r
