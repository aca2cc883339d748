"""Expert parallelism for the MoE layer: E / N experts per GPU, tokens owned by the rank that holds them.

One layer call on every rank (SPMD, `ep_layer`):

1. route   the rank's own tokens (the router is replicated): top-k ids and weights, exactly;
2. pack    its (token, slot) rows grouped by destination rank (expert // (E / N)), stably, with their expert ids;
3. a2a     counts, then rows and ids, over torch.distributed (NCCL between GPUs; gloo in the CPU tests);
4. experts the expert FFN of the rows that arrived, each with its expert id;
5. a2a     the outputs back, in the order they were sent (short passes: blocks of equal size per destination,
           padded, so that no count has to reach the host);
6. combine x[t] += sum over slots, in increasing expert id, of w * out (the reference's mix_body order,
           src/models/olmoe.c:1432-1446).

Each row's arithmetic is the one-GPU layer's, so every rank's output is bit for bit the one-GPU output for its tokens
(the routing, counting sort and mix of src/models/olmoe.c:1845-1933, split across ranks). The backends carry out
steps 1, 2, 4, 6: `GpuEpBackend` with libtrmoe.so's kernels (tr_gpu_moe_layer_part, _ep_pack, _experts_dev,
_ep_combine); tests substitute a CPU backend built on the oracle to check this module's exchange on gloo ranks.
`ep_layer_emulated` runs the same steps for several ranks in one process (one GPU), exchanging by slicing.
"""
from __future__ import annotations

import torch


def expert_range(E: int, rank: int, world: int) -> tuple[int, int]:
    """the experts [first, last) that rank holds: E / world contiguous experts"""
    if E % world:
        raise ValueError(f"{world} ranks do not divide {E} experts")
    n = E // world
    return rank * n, (rank + 1) * n


def local_layer(lay: dict, E: int, rank: int, world: int) -> dict:
    """a layer dict (gguf_blocks.make_layer's form) with the matrices of experts other ranks hold set to None"""
    a, b = expert_range(E, rank, world)
    out = dict(lay)
    for n in ("gate", "up", "down"):
        out[n] = [m if a <= e < b else None for e, m in enumerate(lay[n])]
    return out


def ep_layer(dist, be, layer: int, normed: torch.Tensor, x: torch.Tensor, ffn_out: torch.Tensor | None = None,
             cap: int | None = None):
    """One expert-parallel MoE layer call on this rank: x (T x H) += the layer's output for this rank's tokens.
    Returns (sel_id, sel_w) of the rank's tokens.

    cap (the padded exchange, for short passes): every rank sends every destination a block of cap rows (unused ids
    -1), so the all-to-alls have equal splits and no count reaches the host. Every rank must pass the same cap, at
    least its T x k rows (e.g. the per-rank token limit x k). None: the counts go first and the rows follow packed."""
    world = dist.get_world_size()
    H = normed.shape[1]
    sel_id, sel_w = be.route(layer, normed, x)
    if cap:
        if sel_id.numel() > cap:
            raise ValueError(f"{sel_id.numel()} rows do not fit the padded blocks of {cap}")
        send_rows, send_ids, _, place = be.pack(sel_id, normed, world, cap)
        recv_rows = be.empty((world * cap, H), torch.float32)
        recv_ids = be.empty((world * cap,), torch.int32)
        dist.all_to_all_single(recv_rows, send_rows)
        dist.all_to_all_single(recv_ids, send_ids)
        out = be.experts(layer, recv_rows, recv_ids)
        back = be.empty((world * cap, H), torch.float32)
        dist.all_to_all_single(back, out)
    else:
        send_rows, send_ids, send_counts, place = be.pack(sel_id, normed, world, 0)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        recv_rows = be.empty((sum(rc), H), torch.float32)
        recv_ids = be.empty((sum(rc),), torch.int32)
        dist.all_to_all_single(recv_rows, send_rows, rc, sc)
        dist.all_to_all_single(recv_ids, send_ids, rc, sc)
        out = be.experts(layer, recv_rows, recv_ids)
        back = be.empty((sum(sc), H), torch.float32)
        dist.all_to_all_single(back, out, sc, rc)
    be.combine(sel_w, place, back, x, ffn_out)
    return sel_id, sel_w


def ep_layer_emulated(bes, layer: int, normeds, xs, ffn_outs=None, padded: bool = False):
    """ep_layer for len(bes) ranks in one process: the same steps, the all-to-alls done by slicing."""
    world = len(bes)
    routed = [be.route(layer, n, x) for be, n, x in zip(bes, normeds, xs)]
    cap = max(r[0].numel() for r in routed) if padded else 0
    packs = [be.pack(r[0], n, world, cap) for be, r, n in zip(bes, routed, normeds)]
    if padded:
        counts = [[cap] * world for _ in range(world)]
        starts = [[d * cap for d in range(world)] for _ in range(world)]
    else:
        counts = [p[2].tolist() for p in packs]
        starts = [[sum(c[:d]) for d in range(world)] for c in counts]
    outs = []
    for d, be in enumerate(bes):  # destination d receives from every source s, in source order
        rows = torch.cat([packs[s][0][starts[s][d]:starts[s][d] + counts[s][d]] for s in range(world)])
        ids = torch.cat([packs[s][1][starts[s][d]:starts[s][d] + counts[s][d]] for s in range(world)])
        outs.append(be.experts(layer, rows, ids))
    for s, be in enumerate(bes):  # source s gets its rows back from every destination, in destination order
        back = []
        for d in range(world):
            o = sum(counts[q][d] for q in range(s))  # where source s's rows start in destination d's buffer
            back.append(outs[d][o:o + counts[s][d]])
        be.combine(routed[s][1], packs[s][3], torch.cat(back), xs[s], None if ffn_outs is None else ffn_outs[s])
    return routed


class GpuEpBackend:
    """The steps on one GPU with libtrmoe.so. m: a GpuMoe holding this rank's experts (tr_gpu_moe_set_layer with
    the others None); all tensors on m's device; work on `stream` (a torch stream, so that NCCL orders after it)."""

    def __init__(self, m, stream: torch.cuda.Stream | None = None):
        self.m = m
        self.stream = stream or torch.cuda.current_stream()
        c = m.cfg
        self.E, self.k, self.H = c.n_expert, c.n_used, c.n_embd
        self.dev = torch.device("cuda", torch.cuda.current_device())

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self.dev)

    def _s(self):
        return self.stream.cuda_stream

    def route(self, layer, normed, x):
        T = normed.shape[0]
        sel_id = self.empty((T * self.k,), torch.int64)
        sel_w = self.empty((T * self.k,), torch.float32)
        with torch.cuda.stream(self.stream):
            self.m.layer_part(layer, 0, normed.data_ptr(), T, x.data_ptr(),
                              {"sel_id": sel_id.data_ptr(), "sel_w": sel_w.data_ptr()}, stream=self._s())
        return sel_id, sel_w

    def pack(self, sel_id, normed, world, cap=0):
        R = sel_id.numel()
        rows = self.empty((world * cap if cap else R, self.H), torch.float32)
        ids = self.empty((world * cap if cap else R,), torch.int32)
        counts = self.empty((world,), torch.int32)
        place = self.empty((R,), torch.int32)
        scratch = self.empty((72 + R,), torch.int32)
        with torch.cuda.stream(self.stream):
            self.m.ep_pack(sel_id.data_ptr(), R // self.k, world, cap, normed.data_ptr(), rows.data_ptr(),
                           ids.data_ptr(), counts.data_ptr(), place.data_ptr(), scratch.data_ptr(), stream=self._s())
        return rows, ids, counts, place

    def experts(self, layer, rows, ids):
        out = self.empty(rows.shape, torch.float32)
        if rows.shape[0]:
            with torch.cuda.stream(self.stream):
                self.m.experts_dev(layer, rows.data_ptr(), ids.data_ptr(), rows.shape[0], out.data_ptr(),
                                   stream=self._s())
        return out

    def combine(self, sel_w, place, back, x, ffn_out=None):
        with torch.cuda.stream(self.stream):
            self.m.ep_combine(sel_w.data_ptr(), place.data_ptr(), back.data_ptr(), x.shape[0], x.data_ptr(),
                              None if ffn_out is None else ffn_out.data_ptr(), stream=self._s())


class PeerEp:
    """The expert-parallel layer over peer memory (libtrmoe.so's tr_gpu_moe_ep_peer_* / _dispatch / _experts /
    _peer_combine): rows go straight into their owner's exchange region over NVLink and come back the same way; no
    collective on the data path, so a CUDA graph can hold whole layer calls. Set up collectively (the IPC handles are
    gathered once with torch.distributed); every rank then calls layer() in step. m: a GpuMoe holding this rank's
    experts, with max_tokens >= world x cap; cap >= the most (token, slot) rows a rank sends in one call."""

    def __init__(self, dist, m, cap: int, stream: torch.cuda.Stream | None = None):
        self.m, self.cap = m, cap
        self.stream = stream or torch.cuda.current_stream()
        world, rank = dist.get_world_size(), dist.get_rank()
        c = m.cfg
        self.k, self.H = c.n_used, c.n_embd
        handle = m.ep_peer_region(world, rank, cap)
        handles = [None] * world
        dist.all_gather_object(handles, handle)
        m.ep_peer_open(handles)
        self.dev = torch.device("cuda", torch.cuda.current_device())

    def layer(self, layer: int, normed: torch.Tensor, x: torch.Tensor, ffn_out: torch.Tensor | None = None):
        """x (T x H) += the layer's output for this rank's tokens; returns (sel_id, sel_w)"""
        T = normed.shape[0]
        sel_id = torch.empty((T * self.k,), dtype=torch.int64, device=self.dev)
        sel_w = torch.empty((T * self.k,), dtype=torch.float32, device=self.dev)
        place = torch.empty((T * self.k,), dtype=torch.int32, device=self.dev)
        sp = self.stream.cuda_stream
        with torch.cuda.stream(self.stream):
            self.m.layer_part(layer, 0, normed.data_ptr(), T, x.data_ptr(),
                              {"sel_id": sel_id.data_ptr(), "sel_w": sel_w.data_ptr()}, stream=sp)
            self.m.ep_dispatch(sel_id.data_ptr(), T, normed.data_ptr(), place.data_ptr(), stream=sp)
            self.m.ep_experts(layer, stream=sp)
            self.m.ep_peer_combine(sel_w.data_ptr(), place.data_ptr(), T, x.data_ptr(),
                                   None if ffn_out is None else ffn_out.data_ptr(), stream=sp)
        return sel_id, sel_w

