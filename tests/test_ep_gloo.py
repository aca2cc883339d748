"""Expert parallelism's exchange (trochilus_b200/ep.py: route, pack, all-to-all, experts, all-to-all, combine) on
gloo ranks on the CPU. The steps run on a CPU backend built on the oracle, so that what is tested here is the
module's protocol: the split sizes, the order rows travel and come back in, and the place of every row. Each rank's
output must equal, bit for bit, the one-process oracle layer on its own tokens (routing ids and weights too)."""
import os
import socket

import numpy as np
import pytest
import torch

from trochilus_b200 import ep
from trochilus_b200 import gguf_blocks as gb

E, K, H, F = 16, 4, 512, 256


class OracleEpBackend:
    """ep.py's backend steps done by the oracle on CPU tensors, for the rank's local experts only."""

    def __init__(self, oracle, lay, bias, rank, world, rt, gt, dt):
        self.o, self.bias, self.rt, self.gt, self.dt = oracle, bias, rt, gt, dt
        self.router = lay["router"]
        loc = ep.local_layer(lay, E, rank, world)
        dummy = {n: next(m for m in loc[n] if m is not None) for n in ("gate", "up", "down")}
        # groups of experts held elsewhere never get rows; any matrix stands in for them
        self.mats = {n: [m if m is not None else dummy[n] for m in loc[n]] for n in ("gate", "up", "down")}
        self.first, self.last = ep.expert_range(E, rank, world)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def route(self, layer, normed, x):
        T = normed.shape[0]
        logits = self.o.matmul_grouped(self.rt, E, H, [self.router], np.array([0, T]), normed.numpy())
        if self.bias is not None:
            logits = (logits + self.bias[None, :]).astype(np.float32)
        ids, ws = self.o.route(logits, K, 0)
        return torch.from_numpy(ids.ravel().copy()), torch.from_numpy(ws.ravel().copy())

    def pack(self, sel_id, normed, world, cap=0):
        sid = sid_all = sel_id.numpy()
        dest = sid // (E // world)
        order = np.argsort(dest, kind="stable")
        counts = np.bincount(dest, minlength=world).astype(np.int32)
        pos = np.arange(sid.size)
        if cap:  # destination d's rows at d cap + their rank
            starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
            pos = dest[order] * cap + (pos - starts[dest[order]])
        place = np.empty(sid.size, np.int32)
        place[order] = pos
        n = world * cap if cap else sid.size
        rows = np.zeros((n, H), np.float32)
        ids = np.full(n, -1, np.int32)
        rows[pos] = normed.numpy()[order // K]
        ids[pos] = sid_all[order]
        return torch.from_numpy(rows), torch.from_numpy(ids), torch.from_numpy(counts), torch.from_numpy(place)

    def experts(self, layer, rows, ids):
        ids_all = ids.numpy()
        out = np.zeros((ids_all.size, H), np.float32)
        sel = np.nonzero(ids_all >= 0)[0]  # the padding (-1) carries no row
        if sel.size == 0:
            return torch.from_numpy(out)
        ids = ids_all[sel]
        assert ids.min() >= self.first and ids.max() < self.last, "a row reached a rank without its expert"
        order = np.argsort(ids, kind="stable")
        off = np.concatenate([[0], np.cumsum(np.bincount(ids, minlength=E))])
        xg = rows.numpy()[sel][order]
        h1 = self.o.matmul_grouped(self.gt, F, H, self.mats["gate"], off, xg)
        h2 = self.o.matmul_grouped(self.gt, F, H, self.mats["up"], off, xg)
        h1 = self.o.swiglu(h1, h2)
        h3 = self.o.matmul_grouped(self.dt, H, F, self.mats["down"], off, h1)
        out[sel[order]] = h3
        return torch.from_numpy(out)

    def combine(self, sel_w, place, back, x, ffn_out=None):
        T = x.shape[0]
        w = sel_w.numpy().reshape(T, K)
        b = back.numpy()[place.numpy()].reshape(T, K, H)
        out = np.zeros((T, H), np.float32)
        for s in range(K):  # out = +0; out += w h3 in slot (= expert id) order, every operation rounded to float
            out = out + (w[:, s, None] * b[:, s]).astype(np.float32)
        x.copy_(torch.from_numpy((x.numpy() + out).astype(np.float32)))
        if ffn_out is not None:
            ffn_out.copy_(torch.from_numpy(out))


def _case(rank):
    rng = np.random.default_rng(100 + rank)
    T = 3 + 2 * rank
    return (rng.normal(size=(T, H)).astype(np.float32), rng.normal(size=(T, H)).astype(np.float32))


def _worker(rank, world, port, rt, gt, dt, padded):
    import torch.distributed as dist
    from oracle.oracle import Oracle, make_desc
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        oracle = Oracle()
        lay = gb.make_layer(555, E, H, F, gt, dt, rt, mode="random")
        bias = gb.zipf_bias(4, E)
        be = OracleEpBackend(oracle, lay, bias, rank, world, rt, gt, dt)
        normed, x = _case(rank)
        xt = torch.from_numpy(x.copy())
        for rep in range(2):  # two calls: nothing is left over from the first
            xr = xt.clone()
            sid, sw = ep.ep_layer(dist, be, 0, torch.from_numpy(normed), xr, cap=(3 + 2 * (world - 1)) * K if padded else None)
            d, keep = make_desc(lay, H, F, K, 0, rt, gt, dt, bias)
            want = oracle.moe_layer(d, normed, x)
            assert np.array_equal(sid.numpy().reshape(-1, K), want["sel_id"]), (rank, rep)
            assert np.array_equal(sw.numpy().reshape(-1, K).view(np.uint32), want["sel_w"].view(np.uint32)), (rank, rep)
            assert np.array_equal(xr.numpy().view(np.uint32), want["x"].view(np.uint32)), (rank, rep)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,padded", [(2, False), (2, True), (4, False), (4, True), (8, True)])
def test_ep_exchange_on_gloo_ranks_matches_one_process(world, padded):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _free_port(), gb.F32, gb.Q8_0, gb.Q6_K, padded), nprocs=world, join=True)


def test_expert_range_and_local_layer():
    assert ep.expert_range(64, 3, 8) == (24, 32)
    with pytest.raises(ValueError):
        ep.expert_range(64, 0, 3)
    lay = {"router": None, "gate": list(range(8)), "up": list(range(8)), "down": list(range(8))}
    loc = ep.local_layer(lay, 8, 1, 2)
    assert loc["gate"] == [None] * 4 + [4, 5, 6, 7]


def _leaver(rank, world, port, out_dir):
    """rank 1 leaves between two layer calls (an exception on the host, none of its collectives in flight); rank 0's
    next exchange must end in an error within the process group's short timeout, not wait for good"""
    import datetime

    import torch.distributed as dist
    from oracle.oracle import Oracle
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    oracle = Oracle()
    lay = gb.make_layer(555, E, H, F, gb.Q8_0, gb.Q6_K, gb.F32, mode="random")
    be = OracleEpBackend(oracle, lay, None, rank, world, gb.F32, gb.Q8_0, gb.Q6_K)
    normed, x = _case(rank)
    cap = (3 + 2 * (world - 1)) * K
    ep.ep_layer(dist, be, 0, torch.from_numpy(normed), torch.from_numpy(x.copy()), cap=cap)
    if rank == 1:
        try:
            raise RuntimeError("rank 1 fails between steps")
        except RuntimeError:
            os._exit(0)  # leaves without a word to the others
    import time
    t0 = time.monotonic()
    try:
        ep.ep_layer(dist, be, 0, torch.from_numpy(normed), torch.from_numpy(x.copy()), cap=cap)
        result = "no error"
    except Exception as exc:  # gloo: the peer's closed connection or the timeout
        result = f"error after {time.monotonic() - t0:.1f} s: {type(exc).__name__}"
    with open(os.path.join(out_dir, "rank0"), "w") as f:
        f.write(result)
    os._exit(0)  # (the group cannot be torn down collectively any more)


def test_ep_rank_leaving_ends_in_an_error_not_a_hang(tmp_path):
    import torch.multiprocessing as mp
    import time
    ctx = mp.spawn(_leaver, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False)
    t0 = time.monotonic()
    while not ctx.join(timeout=5) and time.monotonic() - t0 < 120:  # (returns each time one rank ends)
        pass
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    text = (tmp_path / "rank0").read_text()
    assert text.startswith("error after"), text
    assert float(text.split()[2]) < 60.0, text
