"""Expert-parallel orchestration (uaii_moe.ep) with two gloo ranks on CPU.

The device steps (dispatch packing, expert products, combine) are replaced by
a CPU restatement with the same contract as the C ABI (one row per (token,
destination rank) grouped by rank in token order, top_k (local expert | -1,
weight) entries per row, per-rank partials added in rank order), whose expert
math comes from the oracle.  The tests check that the exchange (count
all-to-all, row all-to-alls both ways, combine) reproduces the single-process
layer, and that a rank that fails mid-layer makes the other rank's collective
end with an error instead of waiting forever.
"""
from __future__ import annotations

import datetime
import os
import queue
import socket
import sys
import traceback

import numpy as np
import pytest

torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_case(seed: int = 5):
    rng = np.random.default_rng(seed)
    D, E, I, k, T = 64, 8, 32, 3, 7
    w_router = (rng.standard_normal((E, D)) * 0.3).astype(np.float32)
    G = (rng.standard_normal((E, I, D)) * 0.05).astype(np.float32)
    U = (rng.standard_normal((E, I, D)) * 0.05).astype(np.float32)
    Dn = (rng.standard_normal((E, D, I)) * 0.05).astype(np.float32)
    return D, E, I, k, T, w_router, G, U, Dn


def _tokens(rank: int, T: int, D: int) -> np.ndarray:
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((T, D)).astype(np.float32)
    return x.astype(np.float16).astype(np.float32)  # the exchange carries f16 rows


class FakeEpBackend:
    """CPU restatement of uaii_moe_ep_{dispatch,experts,combine} (test only)."""

    def __init__(self, oracle, w_router, G, U, Dn, k: int, world: int):
        self.o, self.w, self.G, self.U, self.Dn, self.k = oracle, w_router, G, U, Dn, k
        self.E = G.shape[0]
        self.epr = self.E // world

    def ep_dispatch(self, layer, x, T, rank, world, send_x16, send_ids, send_w, send_token, row_of, send_counts,
                    send_entries, probs=None):
        xn = x.numpy()
        _, pr, _ = self.o.router(np.ascontiguousarray(xn), self.w)
        sel = [self.o.topk(pr[t], self.k, 1) for t in range(T)]
        groups = [[t for t in range(T) if any(int(e) // self.epr == d for e in sel[t][0])] for d in range(world)]
        row = 0
        row_of.fill_(-1)
        for d in range(world):
            send_counts[d] = len(groups[d])
            send_entries[d] = sum(int(int(e) // self.epr == d) for t in groups[d] for e in sel[t][0])
            for t in groups[d]:
                ids, w = sel[t]
                send_x16[row] = torch.from_numpy(xn[t]).to(torch.float16)
                for r in range(self.k):
                    mine = int(ids[r]) // self.epr == d
                    send_ids[row, r] = int(ids[r]) - d * self.epr if mine else -1
                    send_w[row, r] = float(w[r]) if mine else 0.0
                send_token[row] = t
                row_of[t, d] = row
                row += 1
        if probs is not None:
            probs.copy_(torch.from_numpy(pr))

    def ep_experts(self, layer, recv_x16, recv_ids, recv_w, rows, entries, y_part):
        first = layer  # the fake's "layer" is this rank's first global expert
        assert int((recv_ids[:rows] >= 0).sum()) == entries
        for i in range(rows):
            xr = recv_x16[i].to(torch.float32).numpy()[None, :]
            acc = np.zeros(xr.shape[1], np.float32)
            for r in range(self.k):
                e = int(recv_ids[i, r])
                if e < 0:
                    continue
                g = first + e
                ye, _, _ = self.o.experts_f32(xr, self.G[g:g + 1], self.U[g:g + 1], self.Dn[g:g + 1],
                                              np.ones((1, 1), np.float32), 1)
                acc = acc + np.float32(recv_w[i, r]) * ye[0]
            y_part[i] = torch.from_numpy(acc.astype(np.float32))

    @staticmethod
    def _fields(rec, D, k):  # views of the record columns (same layout as the C ABI)
        return (rec[:, :2 * D].view(torch.float16), rec[:, 2 * D:2 * D + 4 * k].view(torch.int32),
                rec[:, 2 * D + 4 * k:2 * D + 8 * k].view(torch.float32))

    def ep_dispatch_records(self, layer, x, T, rank, world, send_rec, rec_bytes, send_token, row_of, send_counts,
                            send_entries, probs=None):
        assert rec_bytes == send_rec.shape[1] and rec_bytes % 16 == 0
        x16, ids, w = self._fields(send_rec, x.shape[1], self.k)
        self.ep_dispatch(layer, x, T, rank, world, x16, ids, w, send_token, row_of, send_counts, send_entries, probs)

    def ep_experts_records(self, layer, recv_rec, rec_bytes, rows, entries, y_part):
        x16, ids, w = self._fields(recv_rec, y_part.shape[1], self.k)
        self.ep_experts(layer, x16, ids, w, rows, entries, y_part)

    def ep_experts_records_f16(self, layer, recv_rec, rec_bytes, rows, entries, y_part):
        self.ep_experts_records(layer, recv_rec, rec_bytes, rows, entries, y_part)  # y_part is f16: rounded once

    def ep_combine_f16(self, y_back, row_of, T, world, D, y):
        self.ep_combine(y_back.to(torch.float32), row_of, T, world, D, y)

    def ep_combine(self, y_back, row_of, T, world, D, y):
        for t in range(T):
            acc = torch.zeros(D, dtype=torch.float32)
            for d in range(world):
                r = int(row_of[t, d])
                if r >= 0:
                    acc = acc + y_back[r]
            y[t] = acc


def _worker(rank: int, world: int, port: int, q, fail_rank: int, chunks: int = 1, f16: bool = False):
    try:
        sys.path.insert(0, REPO)
        sys.path.insert(0, os.path.join(REPO, "universal-ai-inference_b200"))
        import torch.distributed as dist

        from oracle.oracle import Oracle
        from uaii_moe.ep import ExpertParallelFFN

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        D, E, I, k, T, w_router, G, U, Dn = _layer_case()
        fake = FakeEpBackend(Oracle(), w_router, G, U, Dn, k, world)
        if rank == fail_rank:  # the device step of this rank fails before the exchange
            def broken(*a, **kw):
                raise RuntimeError("planted dispatch failure")
            fake.ep_dispatch = broken
        ep = ExpertParallelFFN(fake, None, rank * (E // world), D, E, k, rank, world, device="cpu", chunks=chunks,
                               min_chunk=1, return_f16=f16)
        x = torch.from_numpy(_tokens(rank, T, D))
        y = torch.zeros((T, D), dtype=torch.float32)
        try:
            ep.forward(x, y)
            q.put((rank, "ok", y.numpy(), ep.last_exchange))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error", f"{type(e).__name__}: {e}", None))
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass
    except Exception:  # noqa: BLE001
        q.put((rank, "crash", traceback.format_exc(), None))


def _run(world: int, fail_rank: int = -1, timeout: float = 120.0, chunks: int = 1, f16: bool = False):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank, chunks, f16)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, payload, extra = q.get(timeout=timeout)
            out[rank] = (status, payload, extra)
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
    return out


@pytest.mark.parametrize("chunks,f16", [(1, False), (3, False), (1, True)])  # 3: chunks with overlapped exchanges
def test_ep_two_ranks_match_single_process(oracle, chunks, f16):
    D, E, I, k, T, w_router, G, U, Dn = _layer_case()
    out = _run(2, chunks=chunks, f16=f16)
    assert set(out) == {0, 1}, out
    for rank in (0, 1):
        status, y, exch = out[rank]
        assert status == "ok", y
        x = _tokens(rank, T, D)
        _, pr, _ = oracle.router(x, w_router)
        y_ref, _, _ = oracle.experts_f32(x, G, U, Dn, pr, k)
        err = np.abs(y - y_ref).max() / max(np.abs(y_ref).max(), 1e-30)
        assert err < (1.5e-3 if f16 else 1e-5), (rank, err)  # f16 return rows: one rounding per rank row
        send_rows, recv_rows, entries = exch
        assert sum(send_rows) >= T and sum(send_rows) <= 2 * T  # each token goes to 1 or 2 ranks
        assert entries >= sum(recv_rows)


def test_ep_rank_failure_surfaces_as_error_not_hang():
    out = _run(2, fail_rank=1, timeout=90.0)
    assert 1 in out and out[1][0] == "error" and "planted" in out[1][1]
    # rank 0's exchange must end (error from the collective or the closed peer), not wait forever
    assert 0 in out and out[0][0] in ("error", "crash"), out.get(0)
