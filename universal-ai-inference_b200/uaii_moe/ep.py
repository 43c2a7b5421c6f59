"""Expert-parallel MoE FFN layer: one process per GPU, experts sharded across
ranks, tokens exchanged with two all-to-alls (dispatch, combine).

Rank r of R owns experts [r*E/R, (r+1)*E/R) and brings its own T tokens.  One
forward is

1. ``ep_dispatch`` (device): router + top-k for the local tokens, then each token
   packed once per rank that owns one of its experts (f16 row + top_k
   (local expert | -1, weight) entries), grouped by destination rank;
2. an all-to-all of the per-destination row and entry counts, then of the rows
   (f16 activations, expert ids, weights);
3. ``ep_experts`` (device): the grouped expert GEMM over the received rows,
   producing one f32 row per received row (its weighted expert sum);
4. the reverse all-to-all of those rows;
5. ``ep_combine`` (device): each token adds its returned rows in rank order.

The exchange uses ``torch.distributed.all_to_all_single`` (NCCL over NVLink on
GPUs, gloo for the CPU tests); the device steps go through the library's C ABI.
The reference has no expert parallelism (its MoE op runs in one host process,
libs/uaii-kernels/src/transformer.cpp:564-609); summing per-rank partials first
regroups the top-k sum, which changes rounding only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelFFN:
    """Expert-parallel forward of one MoE FFN layer.

    ``backend`` provides ``ep_dispatch``, ``ep_experts`` and ``ep_combine`` with
    the signatures of :class:`uaii_moe.Backend`; ``router_layer`` is a layer
    struct carrying the router weight, d_model, the global expert count, top_k
    and norm_topk; ``local_layer`` carries this rank's experts (n_experts =
    E / world).  ``group`` is the torch.distributed process group (default: world).
    """

    def __init__(self, backend, router_layer, local_layer, d_model: int, n_experts: int, top_k: int,
                 rank: int, world: int, group=None, device="cuda"):
        if n_experts % world != 0:
            raise ValueError("the world size must divide the expert count")
        self.be = backend
        self.router_layer = router_layer
        self.local_layer = local_layer
        self.D, self.E, self.k = d_model, n_experts, top_k
        self.rank, self.world = rank, world
        self.group = group
        self.device = torch.device(device)
        self._cap = -1
        self.last_exchange = None  # (rows sent per rank, rows received per rank, entries received)

    def _buffers(self, T: int):
        cap = T * min(self.k, self.world)
        if cap != self._cap:
            dev, D, k, R = self.device, self.D, self.k, self.world
            self.send_x16 = torch.empty((max(cap, 1), D), dtype=torch.float16, device=dev)
            self.send_ids = torch.empty((max(cap, 1), k), dtype=torch.int32, device=dev)
            self.send_w = torch.empty((max(cap, 1), k), dtype=torch.float32, device=dev)
            self.send_token = torch.empty((max(cap, 1),), dtype=torch.int32, device=dev)
            self.row_of = torch.empty((max(T, 1), R), dtype=torch.int32, device=dev)
            self.counts = torch.empty((2, R), dtype=torch.int32, device=dev)  # rows, entries per destination
            self._cap = cap

    def forward(self, x: torch.Tensor, y: torch.Tensor, probs: torch.Tensor | None = None) -> torch.Tensor:
        T = int(x.shape[0])
        D, k, R = self.D, self.k, self.world
        self._buffers(T)
        self.be.ep_dispatch(self.router_layer, x, T, self.rank, R, self.send_x16, self.send_ids, self.send_w,
                            self.send_token, self.row_of, self.counts[0], self.counts[1], probs)
        # rows and entries per destination -> per source
        meta_send = self.counts.t().contiguous().to(torch.int64)  # [R, 2]
        meta_recv = torch.empty_like(meta_send)
        dist.all_to_all_single(meta_recv, meta_send, group=self.group)
        both = torch.cat([meta_send[:, 0], meta_recv[:, 0], meta_recv[:, 1]]).cpu().tolist()
        send_rows, recv_rows, recv_entries = both[:R], both[R:2 * R], both[2 * R:]
        n_send, n_recv, entries = sum(send_rows), sum(recv_rows), sum(recv_entries)
        self.last_exchange = (send_rows, recv_rows, entries)
        dev = self.device
        recv_x16 = torch.empty((max(n_recv, 1), D), dtype=torch.float16, device=dev)
        recv_ids = torch.empty((max(n_recv, 1), k), dtype=torch.int32, device=dev)
        recv_w = torch.empty((max(n_recv, 1), k), dtype=torch.float32, device=dev)
        dist.all_to_all_single(recv_x16[:n_recv], self.send_x16[:n_send], output_split_sizes=recv_rows,
                               input_split_sizes=send_rows, group=self.group)
        dist.all_to_all_single(recv_ids[:n_recv], self.send_ids[:n_send], output_split_sizes=recv_rows,
                               input_split_sizes=send_rows, group=self.group)
        dist.all_to_all_single(recv_w[:n_recv], self.send_w[:n_send], output_split_sizes=recv_rows,
                               input_split_sizes=send_rows, group=self.group)
        y_part = torch.empty((max(n_recv, 1), D), dtype=torch.float32, device=dev)
        if n_recv:
            self.be.ep_experts(self.local_layer, recv_x16, recv_ids, recv_w, n_recv, entries, y_part)
        y_back = torch.empty((max(n_send, 1), D), dtype=torch.float32, device=dev)
        dist.all_to_all_single(y_back[:n_send], y_part[:n_recv], output_split_sizes=send_rows,
                               input_split_sizes=recv_rows, group=self.group)
        self.be.ep_combine(y_back, self.row_of, T, R, D, y)
        return y
