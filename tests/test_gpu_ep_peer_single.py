"""The peer-memory expert-parallel path (ep.PeerEp: tr_gpu_moe_ep_peer_region / _peer_open, _ep_dispatch,
_ep_experts, _ep_peer_combine) with one rank on one GPU: the same kernels and protocol as on several GPUs (rows
and ids into the exchange region, the arrival flag, the fused kernel's bounded wait and return flag, the combine's
wait, the epochs that tell one call's flags from the last) with its own region as the only peer. Eager calls of 1 and
2 tokens, then a CUDA graph of a whole call replayed on fresh inputs, each bit for bit the oracle's layer."""
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


def test_peer_path_one_rank(cuda, oracle):
    torch = cuda
    import torch.distributed as dist
    from trochilus_b200.moe import GpuMoe
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)  # (the handle exchange only)
    try:
        rt, gt, dt = gb.BF16, gb.Q4_K, gb.Q6_K
        lay = gb.make_layer(2026, E, H, F, gt, dt, rt, mode="random")
        cap = 2 * K
        m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=cap)
        m.set_layer(0, lay)
        st = torch.cuda.Stream()
        pe = ep.PeerEp(dist, m, cap, st)
        d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt)
        rng = np.random.default_rng(4)
        for call in range(4):
            T = 1 + call % 2
            normed = rng.normal(size=(T, H)).astype(np.float32)
            x = rng.normal(size=(T, H)).astype(np.float32)
            want = oracle.moe_layer(d, normed, x)
            dn = torch.from_numpy(normed).cuda()
            dx = torch.from_numpy(x.copy()).cuda()
            sid, sw = pe.layer(0, dn, dx)
            torch.cuda.synchronize()
            m.check()
            assert same_bits(dx.cpu().numpy(), want["x"]), call
            assert same_bits(sid.cpu().numpy().reshape(-1, K), want["sel_id"]), call
        T = 2
        dn = torch.zeros((T, H), device="cuda")
        dx = torch.zeros((T, H), device="cuda")
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            pe.layer(0, dn, dx)
        for rep in range(2):
            normed = rng.normal(size=(T, H)).astype(np.float32)
            x = rng.normal(size=(T, H)).astype(np.float32)
            dn.copy_(torch.from_numpy(normed))
            dx.copy_(torch.from_numpy(x))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            assert same_bits(dx.cpu().numpy(), oracle.moe_layer(d, normed, x)["x"]), rep
        del g
        m.check()
        m.close()
    finally:
        dist.destroy_process_group()


def test_peer_wait_gives_up_and_recovers(cuda, oracle):
    """failure detection without a GPU fault: a dispatch whose experts step is left out, so the return flag the
    combine waits for is one that nothing sets. The combine's wait gives up after its bound (10 s), records which
    flag it waited for (error code 6: the combine, source 0), and returns without touching x; tr_gpu_moe_check reports
    it and clears it, and the next call works and matches the oracle"""
    torch = cuda
    import re

    import torch.distributed as dist
    from trochilus_b200.moe import GpuMoe
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        rt, gt, dt = gb.F32, gb.Q8_0, gb.Q8_0
        lay = gb.make_layer(2027, E, H, F, gt, dt, rt, mode="random")
        cap = K
        m = GpuMoe(1, E, K, H, F, rt, gt, dt, max_tokens=cap)
        m.set_layer(0, lay)
        st = torch.cuda.Stream()
        pe = ep.PeerEp(dist, m, cap, st)
        d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt)
        rng = np.random.default_rng(5)

        def one_call():
            normed = rng.normal(size=(1, H)).astype(np.float32)
            x = rng.normal(size=(1, H)).astype(np.float32)
            dn, dx = torch.from_numpy(normed).cuda(), torch.from_numpy(x.copy()).cuda()
            pe.layer(0, dn, dx)
            torch.cuda.synchronize()
            m.check()
            assert same_bits(dx.cpu().numpy(), oracle.moe_layer(d, normed, x)["x"])

        one_call()
        # the steps of a call without its experts
        dn = torch.from_numpy(rng.normal(size=(1, H)).astype(np.float32)).cuda()
        x0 = rng.normal(size=(1, H)).astype(np.float32)
        dx = torch.from_numpy(x0.copy()).cuda()
        sel_id = torch.empty((K,), dtype=torch.int64, device="cuda")
        sel_w = torch.empty((K,), dtype=torch.float32, device="cuda")
        place = torch.empty((K,), dtype=torch.int32, device="cuda")
        sp = st.cuda_stream
        with torch.cuda.stream(st):
            m.layer_part(0, 0, dn.data_ptr(), 1, dx.data_ptr(), {"sel_id": sel_id.data_ptr(), "sel_w": sel_w.data_ptr()},
                         stream=sp)
            m.ep_dispatch(sel_id.data_ptr(), 1, dn.data_ptr(), place.data_ptr(), stream=sp)
            m.ep_peer_combine(sel_w.data_ptr(), place.data_ptr(), 1, dx.data_ptr(), None, stream=sp)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="bounded wait") as info:
            m.check()
        code = int(re.search(r"flag (\d+)", str(info.value)).group(1))
        assert code & 15 == 6 and (code >> 4) & 15 == 0  # the combine's wait, on source 0
        assert same_bits(dx.cpu().numpy(), x0)  # x untouched
        m.check()  # cleared
        one_call()
        one_call()
        m.close()
    finally:
        dist.destroy_process_group()
