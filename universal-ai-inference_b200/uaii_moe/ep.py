"""Expert-parallel MoE FFN layer: one process per GPU, experts sharded across
ranks, tokens exchanged with two all-to-alls (dispatch, combine).

Rank r of R owns experts [r*E/R, (r+1)*E/R) and brings its own T tokens.  One
forward is

1. ``ep_dispatch`` (device): router + top-k for the local tokens, then each token
   packed once per rank that owns one of its experts (f16 row + top_k
   (local expert | -1, weight) entries), grouped by destination rank;
2. an all-to-all of the per-destination row and entry counts, then one of the
   rows, each a single record (f16 activations, expert ids, weights);
3. ``ep_experts`` (device): the grouped expert GEMM over the received rows,
   producing one row per received row (its weighted expert sum), f16 by default
   (rounded once: half the bytes of the return exchange) or f32;
4. the reverse all-to-all of those rows;
5. ``ep_combine`` (device): each token adds its returned rows in rank order, in f32.

The exchange uses ``torch.distributed.all_to_all_single`` (NCCL over NVLink on
GPUs, gloo for the CPU tests); the device steps go through the library's C ABI.
The reference has no expert parallelism (its MoE op runs in one host process,
libs/uaii-kernels/src/transformer.cpp:564-609); summing per-rank partials first
regroups the top-k sum, which changes rounding only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def record_bytes(D: int, k: int) -> int:
    """Bytes of one exchanged row: f16 x [D], k int32 ids, k f32 weights, padded to 16."""
    return (2 * D + 8 * k + 15) // 16 * 16


class _Chunk:
    """Send-side buffers of one token chunk: one record per row."""

    def __init__(self, T: int, D: int, k: int, R: int, dev):
        cap = max(T * min(k, R), 1)
        self.T = T
        self.rec = torch.empty((cap, record_bytes(D, k)), dtype=torch.uint8, device=dev)
        self.token = torch.empty((cap,), dtype=torch.int32, device=dev)
        self.row_of = torch.empty((max(T, 1), R), dtype=torch.int32, device=dev)
        self.counts = torch.empty((2, R), dtype=torch.int32, device=dev)  # rows, entries per destination


class ExpertParallelFFN:
    """Expert-parallel forward of one MoE FFN layer.

    ``backend`` provides ``ep_dispatch``, ``ep_experts`` and ``ep_combine`` with
    the signatures of :class:`uaii_moe.Backend`; ``router_layer`` is a layer
    struct carrying the router weight, d_model, the global expert count, top_k
    and norm_topk; ``local_layer`` carries this rank's experts (n_experts =
    E / world).  ``group`` is the torch.distributed process group (default: world).
    ``return_f16`` sends the per-rank partial rows back as f16 (default: on CUDA).

    ``chunks`` > 1 splits the local tokens: every chunk is dispatched up front
    (one host read of all split sizes), then the exchanges run asynchronously so
    that the experts of chunk i overlap the rows of chunk i+1 in flight and the
    return of chunk i overlaps the experts of chunk i+1.
    """

    def __init__(self, backend, router_layer, local_layer, d_model: int, n_experts: int, top_k: int,
                 rank: int, world: int, group=None, device="cuda", chunks: int = 2, min_chunk: int = 256,
                 return_f16: bool | None = None):
        if n_experts % world != 0:
            raise ValueError("the world size must divide the expert count")
        self.be = backend
        self.router_layer = router_layer
        self.local_layer = local_layer
        self.D, self.E, self.k = d_model, n_experts, top_k
        self.rank, self.world = rank, world
        self.group = group
        self.device = torch.device(device)
        self.chunks, self.min_chunk = max(1, chunks), min_chunk
        self.return_f16 = self.device.type == "cuda" if return_f16 is None else bool(return_f16)
        self._bufs = {}
        self.last_exchange = None  # (rows sent per rank, rows received per rank, entries received), all chunks

    def _chunk_bufs(self, i: int, T: int) -> _Chunk:
        b = self._bufs.get(i)
        if b is None or b.T != T:
            b = _Chunk(T, self.D, self.k, self.world, self.device)
            self._bufs[i] = b
        return b

    def forward(self, x: torch.Tensor, y: torch.Tensor, probs: torch.Tensor | None = None) -> torch.Tensor:
        """The collectives and buffer allocations are ordered on the backend's stream;
        x must be ready on it (or on a stream it waits for) when forward is called."""
        stream = getattr(self.be, "stream", None)
        if self.device.type == "cuda" and stream is not None:
            ext = torch.cuda.ExternalStream(stream, device=self.device) if stream else \
                torch.cuda.default_stream(self.device)
            with torch.cuda.stream(ext):
                return self._forward(x, y, probs)
        return self._forward(x, y, probs)

    def _forward(self, x: torch.Tensor, y: torch.Tensor, probs: torch.Tensor | None = None) -> torch.Tensor:
        T = int(x.shape[0])
        D, k, R = self.D, self.k, self.world
        rb = record_bytes(D, k)
        n = self.chunks if T >= self.chunks * self.min_chunk else 1
        bounds = [T * c // n for c in range(n + 1)]
        parts = []
        for c in range(n):  # 1. dispatch every chunk on the device
            t0, t1 = bounds[c], bounds[c + 1]
            b = self._chunk_bufs(c, t1 - t0)
            self.be.ep_dispatch_records(self.router_layer, x[t0:t1], t1 - t0, self.rank, R, b.rec, rb, b.token,
                                        b.row_of, b.counts[0], b.counts[1], None if probs is None else probs[t0:t1])
            parts.append(b)
        # 2. rows / entries per destination of every chunk -> per source (one exchange, one host read)
        meta_send = torch.stack([b.counts.t() for b in parts], dim=1).reshape(R, 2 * n).to(torch.int64)
        meta_recv = torch.empty_like(meta_send)
        dist.all_to_all_single(meta_recv, meta_send.contiguous(), group=self.group)
        host = torch.cat([meta_send.reshape(-1), meta_recv.reshape(-1)]).cpu().view(2, R, n, 2).tolist()
        dev = self.device
        plans = []
        for c, b in enumerate(parts):
            send_rows = [host[0][r][c][0] for r in range(R)]
            recv_rows = [host[1][r][c][0] for r in range(R)]
            entries = sum(host[1][r][c][1] for r in range(R))
            plans.append((send_rows, recv_rows, entries))
        self.last_exchange = (
            [sum(p[0][r] for p in plans) for r in range(R)], [sum(p[1][r] for p in plans) for r in range(R)],
            sum(p[2] for p in plans))
        # 3. rows of every chunk in flight (one all-to-all of records per chunk)
        recv, works = [], []
        for (send_rows, recv_rows, entries), b in zip(plans, parts):
            ns, nr = sum(send_rows), sum(recv_rows)
            rrec = torch.empty((max(nr, 1), rb), dtype=torch.uint8, device=dev)
            works.append(dist.all_to_all_single(rrec[:nr], b.rec[:ns], output_split_sizes=recv_rows,
                                                input_split_sizes=send_rows, group=self.group, async_op=True))
            recv.append(rrec)
        # 4. experts of chunk c as soon as its rows are in, return its rows asynchronously
        backs, rworks = [], []
        for c, ((send_rows, recv_rows, entries), rrec) in enumerate(zip(plans, recv)):
            works[c].wait()
            ns, nr = sum(send_rows), sum(recv_rows)
            rdt = torch.float16 if self.return_f16 else torch.float32
            y_part = torch.empty((max(nr, 1), D), dtype=rdt, device=dev)
            if nr:
                if self.return_f16:
                    self.be.ep_experts_records_f16(self.local_layer, rrec, rb, nr, entries, y_part)
                else:
                    self.be.ep_experts_records(self.local_layer, rrec, rb, nr, entries, y_part)
            y_back = torch.empty((max(ns, 1), D), dtype=rdt, device=dev)
            rworks.append(dist.all_to_all_single(y_back[:ns], y_part[:nr], output_split_sizes=send_rows,
                                                 input_split_sizes=recv_rows, group=self.group, async_op=True))
            backs.append(y_back)
        # 5. combine each chunk in rank order
        for c, b in enumerate(parts):
            rworks[c].wait()
            t0, t1 = bounds[c], bounds[c + 1]
            if self.return_f16:
                self.be.ep_combine_f16(backs[c], b.row_of, t1 - t0, R, D, y[t0:t1])
            else:
                self.be.ep_combine(backs[c], b.row_of, t1 - t0, R, D, y[t0:t1])
        return y
