"""The ring schedule across processes, on CPU (gloo, world size 2 and 3).

A stand-in stage (exact float64 arithmetic whose result depends on the order
of chunks and on everything already appended to each layer's cache) runs the
same ``Ring`` code as the GPUs; split across ranks it must pick the same ids
as one rank holding every layer.  The routing checks restate test_wire.js:
a lap visits every stage once and terminates at the head; the return leg is
addressed differently from stage 0.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

H, V = 8, 16


class FakeStage:
    """Layers [lo, hi) of a toy model with a per-layer 'cache' (a running sum)."""

    def __init__(self, lo, hi, head):
        self.lo, self.hi, self.head = lo, hi, head
        self.kv = {}
        rng = np.random.default_rng(9)
        self.emb = rng.standard_normal((V, H))
        self.w = rng.standard_normal((8, H)) * 0.3

    def kv_reset(self):
        self.kv = {l: np.zeros(H) for l in range(self.lo, self.hi)}

    def _layers(self, x, pos0, cached, rows=None):
        T = x.numel() // H
        a = x.view(T, H).double().numpy().copy()
        # the cache also moves at every chunk's end (as the value scales do),
        # so the result depends on where the chunks of a pass end
        ends = set(np.cumsum(rows).tolist()) if rows else {T}
        for l in range(self.lo, self.hi):
            for t in range(T):
                if cached:
                    self.kv[l] = self.kv[l] * 0.5 + a[t]
                    ctx = self.kv[l]
                else:
                    ctx = a[: t + 1].sum(0)
                a[t] = np.sin(3.0 * a[t] * self.w[l] + 0.5 * ctx + 0.37 * (pos0 + t))
                if cached and t + 1 in ends:
                    self.kv[l] = self.kv[l] * 0.9 + 0.01
        x.copy_(torch.from_numpy(a.astype(np.float32)).view(-1))
        return x

    def run_layers(self, x):
        return self._layers(x, 0, False)

    def run_layers_chunk(self, x, pos0):
        return self._layers(x, pos0, True)

    def run_layers_chunks(self, x, pos0, rows):
        assert sum(rows) == x.numel() // H and len(rows) > 1
        return self._layers(x, pos0, True, rows)

    def embed_rows(self, ids):
        return torch.from_numpy(self.emb[np.asarray(ids)].astype(np.float32).reshape(-1)).clone()

    def _logits(self, x, row):
        a = x.view(-1, H)[row].double().numpy()
        return self.emb @ a + np.sin(np.arange(V) * (1.0 + 97.0 * a.sum()))

    def logits_at(self, x, rows):
        lg = [self._logits(x, r) for r in rows]
        return [int(np.argmax(l)) for l in lg], lg

    def new_ids(self, n):
        return torch.zeros(max(n, 1), dtype=torch.int32)

    def ids_buffer(self, n):
        return torch.zeros(n, dtype=torch.int32)

    def pick_into(self, x, row, picks, n):
        picks[n] = int(np.argmax(self._logits(x, row)))

    def embed_device(self, picks, n):
        return self.embed_rows([int(picks[n])])

    def broadcast_ids(self, buf):
        import torch.distributed as dist
        dist.broadcast(buf, src=0)


def plan_for(world):
    return {1: [(0, 6)], 2: [(0, 2), (2, 6)], 3: [(0, 1), (1, 4), (4, 6)]}[world]


def run_rank(rank, world, port, prompt, q, wire=False, per_pass=1, window=2):
    import torch.distributed as dist
    import __graft_entry__ as G
    P = G.package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    lo, hi = plan_for(world)[rank]
    st = FakeStage(lo, hi, rank == 0)
    tp = P.pipeline.TorchP2P(P.pipeline.ring_edge_groups(world)) if world > 1 else None
    if tp is not None and wire:
        # every hop as a wire.js activation frame, checked on arrival
        plan = [dict(id=f"rank{i}", index=i) for i in range(world)]
        tp = P.wire.WireTransport(tp, plan, rank, model_hash=0x5EED1234, seq=7)
    ring = P.pipeline.Ring(st, rank, world, H, tp, new_buffer=lambda n: torch.empty(n, dtype=torch.float32))
    marks = []
    picks = ring.generate_chunked(prompt, 5, chunk_size=3, window=window, on_prefill=lambda: marks.append(rank),
                                  per_pass=per_pass)
    assert marks == [rank]  # every rank marks the end of its prefill part once (the bench's timer)
    look = ring.generate_lookahead([4, 4, 4, 7, 4, 4, 4], 4, 12, 4)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        q.put((picks.tolist(), look))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run_world(world, prompt, wire=False, per_pass=1, window=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_rank, args=(r, world, port, prompt, q, wire, per_pass, window))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = q.get(timeout=120)
        for p in procs:
            p.join(60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_ring_matches_single_rank(P, world):
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5]
    ref = run_world(1, prompt)
    assert run_world(world, prompt) == ref
    assert len(ref[0]) == 5 and len(ref[1]) == 7 + 4
    assert len(set(ref[0])) > 1  # the stand-in model is not degenerate


@pytest.mark.parametrize("world", [2, 3])
def test_ring_over_wire_frames_matches_single_rank(P, world):
    """The same schedule with every hop framed, hashed and checked as the
    reference's activation messages (wire.js:100-121) picks the same ids."""
    prompt = [2, 7, 1, 8, 2, 8, 1, 8, 2, 8]
    assert run_world(world, prompt, wire=True) == run_world(1, prompt)


def walk_lap(P, plan):
    ran, addr = [], 0
    for _ in range(100):
        actors = [s["index"] for s in plan if P.pipeline.classify_act(addr, s["index"]) == "mine"]
        assert len(actors) <= 1
        if not actors:
            assert P.pipeline.classify_act(addr, 0) == "return"
            return ran
        ran.append(actors[0])
        addr = P.pipeline.route_after(plan, actors[0])["address"]
    raise AssertionError("lap did not terminate")


def test_lap_visits_every_stage_once(P):
    for n in (1, 2, 3, 5, 8):
        plan = [dict(id=f"p{i}", index=i) for i in range(n)]
        assert walk_lap(P, plan) == list(range(n))


def test_return_leg_is_not_stage_zero(P):
    plan = [dict(id="p0", index=0), dict(id="p1", index=1)]
    last = P.pipeline.route_after(plan, 1)
    assert last["to"] == "p0" and last["isReturn"] and last["address"] != 0
    assert P.pipeline.classify_act(last["address"], 0) == "return"
    assert P.pipeline.classify_act(0, 0) == "mine"


@pytest.mark.parametrize("world,per_pass", [(1, 3), (2, 2), (3, 4)])
def test_chunk_passes_match_one_chunk_per_pass(P, world, per_pass):
    """Several chunks per pass travel the ring together (pipeline.Ring with
    per_pass > 1, ragged chunks of 3 and 2 rows, the last pass short): the
    stand-in stage sees the chunk ends inside each pass, and the ids equal one
    chunk per pass on one rank."""
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7]
    assert run_world(world, prompt, per_pass=per_pass) == run_world(1, prompt)


def test_chunk_passes_grouping(P):
    chunks = P.shard.prefill_chunks(40, 16, 2)["chunks"]  # 14, 13, 13
    assert P.shard.chunk_passes(chunks, 2) == [(0, 27, [14, 13]), (27, 40, [13])]
    assert P.shard.chunk_passes(chunks, 1) == [(0, 14, [14]), (14, 27, [13]), (27, 40, [13])]
    assert P.shard.chunk_passes(chunks, 8) == [(0, 40, [14, 13, 13])]
    big = P.shard.prefill_chunks(2048, 16, 2)["chunks"]
    passes = P.shard.chunk_passes(big, 8)
    assert len(passes) == 16 and all(r == [16] * 8 for _, _, r in passes)
    assert [p[0] for p in passes] == list(range(0, 2048, 128))


def test_more_passes_in_flight_match(P):
    """As many passes in flight as stages (the benchmark's labelled variant;
    the reference keeps two): the same ids."""
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7]
    assert run_world(3, prompt, per_pass=2, window=3) == run_world(1, prompt)
