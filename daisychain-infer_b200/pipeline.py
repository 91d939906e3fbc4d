"""Pipeline stages on 1..8 GPUs of one box: the reference's ring, over NVLink.

The reference hands a T x hidden f32 activation from stage to stage over
WebRTC (public/app.js:705-765, 877-961; wire.js routing :129-138): stage 0 (the
head) embeds, runs its layers and sends; every stage runs its layers and
forwards; the last stage returns to the head, which reads the logits.  Here
each stage is one process on one GPU (torch.distributed, NCCL point-to-point
send/recv of the same f32 buffer), and the lap never leaves the devices:

* chunked prefill (app.js:877-906): prompt chunks from ``prefill_chunks``;
  the head keeps ``window`` (2) chunks in flight, so chunk c+1 runs on stage 0
  while chunk c runs on stage 1; every stage applies its chunks in order and
  appends to its own KV cache;
* decode (app.js:907-921): one token per lap; the head's greedy pick stays on
  the device and feeds the next embedding, so a lap needs no host round trip;
* full-window / lookahead laps (app.js:925-961): the head embeds the window,
  the lap returns the hidden state, the head scores the draft rows.

``Ring`` is written against two small interfaces so its schedule can be tested
on CPU ranks (gloo) with a stand-in stage: a stage with
``embed_rows / run_layers / run_layers_chunk / logits_at`` and a transport
with ``send(tensor, dst, token_idx) / recv(tensor, src, token_idx)`` (the
token index of the hop's first row, which ``wire.WireTransport`` writes into
and checks against the reference's activation frame; ``TorchP2P`` ignores it).
"""
from __future__ import annotations

from . import shard

RETURN = -1  # wire.js:29: the head's return leg is not "stage 0"


def route_after(plan: list, my_index: int) -> dict:
    """wire.js:129-133."""
    is_last = my_index == len(plan) - 1
    nxt = plan[0] if is_last else plan[my_index + 1]
    return dict(to=nxt["id"], address=RETURN if is_last else nxt["index"], isReturn=is_last)


def classify_act(next_index: int, my_index: int) -> str:
    """wire.js:134-138."""
    if next_index == RETURN:
        return "return"
    if next_index == my_index:
        return "mine"
    return "other"


def ring_edge_groups(world: int) -> dict:
    """One process group per directed ring edge i -> (i + 1) % world, so that a
    rank's send to its successor and receive from its predecessor run on
    separate communicators: NCCL orders the point-to-point operations of one
    communicator, and on a single group a pass's return hop would have to
    finish before the next pass could be sent.  Every rank calls this, in the
    same order (group creation is collective).  Returns {(src, dst): group}."""
    import torch.distributed as dist
    edges = {}
    for i in range(world):
        j = (i + 1) % world
        edges[(i, j)] = dist.new_group([i, j])
    return edges


class TorchP2P:
    """Point-to-point transport over torch.distributed (NCCL on GPUs, gloo on CPU);
    with ``edges`` (``ring_edge_groups``) each hop uses its edge's group."""

    def __init__(self, edges: dict | None = None):
        import torch.distributed as dist
        self.dist = dist
        self.edges = edges or {}
        self.me = dist.get_rank() if dist.is_initialized() else 0

    def send(self, t, dst: int, token_idx: int = 0):
        return self.dist.isend(t, dst, group=self.edges.get((self.me, dst)))

    def recv(self, t, src: int, token_idx: int | None = None):
        return self.dist.irecv(t, src, group=self.edges.get((src, self.me)))


class HopBuffers:
    """A ring of hop buffers (up to ``cap`` floats each), so a lap allocates
    nothing per hop: a buffer is handed out again only after the transfer last
    posted on it has completed (``hold`` records that transfer)."""

    def __init__(self, new_buffer, n: int, cap: int):
        self.bufs = [new_buffer(cap) for _ in range(n)]
        self.pending = [None] * n
        self.i = 0

    def take(self, floats: int):
        i = self.i
        self.i = (i + 1) % len(self.bufs)
        if self.pending[i] is not None:
            self.pending[i].wait()
            self.pending[i] = None
        return i, self.bufs[i][:floats]

    def hold(self, i: int, work) -> None:
        self.pending[i] = work

    def drain(self) -> None:
        for i, p in enumerate(self.pending):
            if p is not None:
                p.wait()
                self.pending[i] = None


class Ring:
    """One rank's part of the lap.  ``stage`` holds this rank's layers; rank 0
    is the head.  Every rank runs the same schedule (same chunk list, same
    number of decode laps), so no control messages are needed."""

    def __init__(self, stage, rank: int, world: int, hidden: int, transport=None, device=None, new_buffer=None):
        self.stage, self.rank, self.world, self.hidden = stage, rank, world, hidden
        self.tp = transport
        self.nxt = (rank + 1) % world
        self.prv = (rank - 1) % world
        self.new_buffer = new_buffer  # new_buffer(n_floats) -> tensor on this rank's device
        self.use_graph = True
        self._rings = {}

    def _ring(self, key: str, n: int, cap: int) -> HopBuffers:
        """The hop buffers of one kind of transfer, made once per size."""
        r = self._rings.get(key)
        if r is None or r.bufs[0].numel() < cap or len(r.bufs) < n:
            r = self._rings[key] = HopBuffers(self.new_buffer, n, cap)
        return r

    # ---- chunked prefill + decode --------------------------------------------------
    def _run_pass(self, x, lo: int, rows: list):
        S = self.stage
        return S.run_layers_chunks(x, lo, rows) if len(rows) > 1 else S.run_layers_chunk(x, lo)

    def generate_chunked(self, ids0: list, n_new: int, chunk_size: int = 16, window: int = 2, on_prefill=None,
                         per_pass: int = 1):
        """Returns the device tensor of picked ids on the head (n_new int32), None elsewhere.
        ``on_prefill`` (optional) is called on every rank once its prefill part is issued
        (on the head: when the prefill lap has returned).  ``per_pass`` consecutive
        chunks travel and run together (one pass over each stage's weights; the
        same ids); ``window`` counts such passes in flight."""
        S, H = self.stage, self.hidden
        S.kv_reset()
        chunks = shard.prefill_chunks(len(ids0), chunk_size, window)
        passes = shard.chunk_passes(chunks["chunks"], per_pass)
        last = None
        if self.world == 1:
            for lo, hi, rows in passes:
                last = self._run_pass(S.embed_rows(ids0[lo:hi]), lo, rows)
            if on_prefill:
                on_prefill()
            return self._decode_local(last, len(ids0), n_new)
        cap = chunks["chunkSize"] * max(1, int(per_pass)) * H
        if self.rank == 0:
            flights = []
            backs = self._ring("prefill-return", chunks["window"] + 1, cap)
            for lo, hi, rows in passes:
                x = self._run_pass(S.embed_rows(ids0[lo:hi]), lo, rows)
                sent = self.tp.send(x, self.nxt, token_idx=lo)  # the handle keeps the send (and x) alive
                _, back = backs.take((hi - lo) * H)
                flights.append((sent, self.tp.recv(back, self.prv, token_idx=lo), back))
                if len(flights) >= chunks["window"]:
                    sent_, req, buf = flights.pop(0)
                    sent_.wait()
                    req.wait()
                    last = buf
            while flights:
                sent_, req, buf = flights.pop(0)
                sent_.wait()
                req.wait()
                last = buf
            if on_prefill:
                on_prefill()
            return self._decode_head(last, len(ids0), n_new)
        # a middle or last stage: chunks arrive in order (the inbox of app.js:719-749)
        hops = self._ring("prefill-hop", chunks["window"] + 1, cap)
        for lo, hi, rows in passes:
            i, buf = hops.take((hi - lo) * H)
            self.tp.recv(buf, self.prv, token_idx=lo).wait()
            self._run_pass(buf, lo, rows)
            hops.hold(i, self.tp.send(buf, self.nxt, token_idx=lo))
        if on_prefill:
            on_prefill()
        rows = self._ring("decode-hop", 2, H)
        for n in range(n_new):
            i, buf = rows.take(H)
            self.tp.recv(buf, self.prv, token_idx=len(ids0) + n).wait()
            S.run_layers_chunk(buf, len(ids0) + n)
            rows.hold(i, self.tp.send(buf, self.nxt, token_idx=len(ids0) + n))
        hops.drain()
        rows.drain()
        return None

    def _decode_local(self, last, n_prompt: int, n_new: int):
        S = self.stage
        if hasattr(S, "decode_many"):  # the device loop (one CUDA graph per lap)
            return S.decode_many([S], last, n_new, use_graph=self.use_graph)
        picks = S.new_ids(n_new)
        for n in range(n_new):
            rows = last.numel() // self.hidden
            S.pick_into(last, rows - 1, picks, n)
            last = S.run_layers_chunk(S.embed_device(picks, n), n_prompt + n)
        return picks

    def _decode_head(self, last, n_prompt: int, n_new: int):
        S = self.stage
        picks = S.new_ids(n_new)
        backs = self._ring("decode-return", 2, self.hidden)
        for n in range(n_new):
            rows = last.numel() // self.hidden
            S.pick_into(last, rows - 1, picks, n)
            x = S.run_layers_chunk(S.embed_device(picks, n), n_prompt + n)
            sent = self.tp.send(x, self.nxt, token_idx=n_prompt + n)
            _, back = backs.take(self.hidden)
            self.tp.recv(back, self.prv, token_idx=n_prompt + n).wait()
            sent.wait()
            last = back
        return picks

    # ---- full-window laps ------------------------------------------------------------
    def window_lap(self, win_ids: list):
        """One full-window lap; the head gets the returned hidden state."""
        S, H, T = self.stage, self.hidden, len(win_ids)
        if self.rank == 0:
            x = S.run_layers(S.embed_rows(win_ids))
            if self.world == 1:
                return x
            sent = self.tp.send(x, self.nxt)
            _, back = self._ring("window-return", 2, T * H).take(T * H)
            self.tp.recv(back, self.prv).wait()
            sent.wait()
            return back
        hops = self._ring("window-hop", 2, T * H)
        i, buf = hops.take(T * H)
        self.tp.recv(buf, self.prv).wait()
        S.run_layers(buf)
        hops.hold(i, self.tp.send(buf, self.nxt))
        return None

    def generate_lookahead(self, ids0: list, n_new: int, T: int, max_draft: int = 4):
        """infer.js:464-494 across the ring.  Every rank needs the window size of
        each lap, so the head shares the accepted count over the transport."""
        ids = list(ids0)
        produced = 0
        S = self.stage
        while produced < n_new:
            frame = shard.lookahead_frame(ids, T, max_draft)
            draft = frame["draft"]
            win = [0] * (T - len(frame["win"])) + frame["win"]
            x = self.window_lap(win)
            got = None
            if self.rank == 0:
                rows = shard.draft_rows(T, frame["shown"], len(draft))
                picked, _ = S.logits_at(x, rows)
                got = shard.accept_draft(picked, draft)
            got = self._share_ids(got)
            if not got:
                break
            for t in got:
                ids.append(t)
                produced += 1
                if produced >= n_new:
                    break
        return ids

    def _share_ids(self, got):
        if self.world == 1:
            return got
        import torch
        buf = self.new_ids_host_buffer()
        if self.rank == 0:
            buf.zero_()
            buf[0] = len(got)
            buf[1:1 + len(got)] = torch.tensor(got, dtype=buf.dtype)
        self.stage.broadcast_ids(buf)
        n = int(buf[0].item())
        return [int(v) for v in buf[1:1 + n].tolist()]

    def new_ids_host_buffer(self):
        return self.stage.ids_buffer(16)
