"""Expert-parallel host logic on CPU: two gloo ranks run ExpertParallelMoE with CPU stand-ins for
the device steps (the oracle's per-expert arithmetic), and the result must equal the single-process
oracle layer bit for bit — dispatch order, split sizes, re-slotting, return and combine order."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ref

E, H, I, T, TOPK = 8, 256, 128, 24, 4


class RefOps:
    """CPU stand-ins for CudaOps with the oracle's arithmetic (test infrastructure)."""

    def align(self, ids, E_):
        flat = ids.flatten().long()
        n = flat.numel()
        valid = (flat >= 0) & (flat < E_)
        key = torch.where(valid, flat, torch.full_like(flat, E_))
        order = torch.argsort(key, stable=True)
        counts = torch.bincount(flat[valid], minlength=E_).to(torch.int32)
        offsets = torch.cat([torch.zeros(1, dtype=torch.int32), counts.cumsum(0).to(torch.int32)])
        nv = int(valid.sum())
        inv = torch.full((n,), -1, dtype=torch.int32)
        inv[order[:nv]] = torch.arange(nv, dtype=torch.int32)
        return counts, offsets, order.to(torch.int32), inv

    def gather_rows(self, src, idx, div, n):
        return src[idx[:n].long() // div]

    def layout(self, recv_counts, R):
        S, El = recv_counts.shape
        c = recv_counts.long()
        src_start = torch.cat([torch.zeros(1, dtype=torch.long), c.sum(1).cumsum(0)[:-1]])
        recv_base = src_start[:, None] + torch.cat([torch.zeros(S, 1, dtype=torch.long),
                                                    c.cumsum(1)[:, :-1]], dim=1)
        rows = []
        for e in range(El):
            for s in range(S):
                rows.extend(range(int(recv_base[s, e]), int(recv_base[s, e] + c[s, e])))
        rows = torch.tensor(rows, dtype=torch.int32)
        offsets = torch.cat([torch.zeros(1, dtype=torch.long), c.sum(0).cumsum(0)]).to(torch.int32)
        inv = torch.empty(R, dtype=torch.int32)
        inv[rows.long()] = torch.arange(R, dtype=torch.int32)
        return offsets, rows, inv

    def grouped(self, xrows, rows, offsets, weights, tokens_per_expert, flags):
        gu_q, gu_s, gu_z, dn_q, dn_s, dn_z = weights
        R = rows.numel()
        out3 = torch.zeros(R, xrows.shape[1], dtype=torch.float16)
        for e in range(gu_q.shape[0]):
            a, b = int(offsets[e]), int(offsets[e + 1])
            if a == b:
                continue
            x = xrows[rows[a:b].long()].half().float()
            wgu = ref.dequant_w4(gu_q[e], gu_s[e], gu_z[e], 128).float()
            wdn = ref.dequant_w4(dn_q[e], dn_s[e], dn_z[e], 64).float()
            gu = x @ wgu.T
            act = (ref.gelu_tanh(gu[:, :I]) * gu[:, I:]).half().float()
            out3[a:b] = (act @ wdn.T).half()
        return out3

    def combine(self, out3, inv, w, T_, out_dtype):
        tk = w.shape[1]
        o3 = torch.zeros(T_ * tk, out3.shape[1], dtype=torch.float16)
        valid = inv >= 0
        o3[valid] = out3[inv[valid].long()]
        o3 = o3.float().view(T_, tk, -1)
        wf = w.float()
        vm = valid.view(T_, tk)
        y = torch.zeros(T_, out3.shape[1], dtype=torch.float32)
        for j in range(tk):
            y = y + torch.where(vm[:, j, None], wf[:, j, None] * o3[:, j], torch.zeros(()))
        return y.to(out_dtype)


def _data():
    import workloads
    W = workloads.moe_weights(E, H, I, seed=3)
    g = torch.Generator().manual_seed(4)
    hidden = (torch.randn(T, H, generator=g) * 0.5).half()
    ids, w = workloads.random_routing(T, E, TOPK, seed=4)
    ids[5, 1] = E  # a dropped pair (id out of range)
    return W, hidden, ids, w


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ep_moe
        W, hidden, ids, w = _data()
        local = ep_moe.shard_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                     W["dn_z"], rank, world)
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        layer = ep_moe.ExpertParallelMoE(*local, E_total=E, ops=RefOps(), int_zeros=False)
        y = layer(hidden[sl], ids[sl], w[sl], out_dtype=torch.float16)
        torch.save(y, os.path.join(out_dir, f"y{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, world, out_dir, attempts=3):
    """mp.spawn with a fresh rendezvous port per attempt: the port _free_port() released can be
    taken by another process before rank 0 binds it (EADDRINUSE), which says nothing about the
    code under test."""
    for i in range(attempts):
        try:
            mp.spawn(fn, args=(world, _free_port(), out_dir), nprocs=world, join=True)
            return
        except Exception as exc:  # the ranks' error arrives as ProcessRaisedException text
            if "EADDRINUSE" not in str(exc) or i == attempts - 1:
                raise


@pytest.mark.parametrize("world", [1, 2])
def test_expert_parallel_matches_single_process(world):
    W, hidden, ids, w = _data()
    want = ref.moe_layer(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"],
                         ids, w, out_dtype=torch.float16)
    with tempfile.TemporaryDirectory() as d:
        _spawn(_worker, world, d)
        got = torch.cat([torch.load(os.path.join(d, f"y{r}.pt")) for r in range(world)])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def _straggler_worker(rank, world, port, out_dir):
    """Rank 1 joins the process group but never enters the layer's collectives; rank 0 must get
    an error from its first exchange once the group's timeout passes, not hang."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        time.sleep(12)            # longer than the timeout, then leave without a collective
        return
    import ep_moe
    W, hidden, ids, w = _data()
    local = ep_moe.shard_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                 W["dn_z"], rank, world)
    layer = ep_moe.ExpertParallelMoE(*local, E_total=E, ops=RefOps(), int_zeros=False)
    t0 = time.monotonic()
    outcome = "returned"
    try:
        layer(hidden[:T // 2], ids[:T // 2], w[:T // 2], out_dtype=torch.float16)
    except Exception as exc:  # gloo reports the timeout as a RuntimeError subclass
        outcome = type(exc).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.1f}")


def test_rank_that_never_joins_is_reported_on_the_host():
    with tempfile.TemporaryDirectory() as d:
        _spawn(_straggler_worker, 2, d)
        outcome, secs = open(os.path.join(d, "rank0.txt")).read().split()
    assert outcome != "returned"
    assert float(secs) < 11.0      # ended by the 3 s group timeout, before the straggler left


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_relabel_is_a_permutation_that_spreads_the_tasks(world):
    import math
    import ep_moe
    g = torch.Generator().manual_seed(world)
    # Zipf-like pairs per expert, as the router's bias gives them
    counts = [int(600 / (1 + e) ** 0.8 + torch.randint(0, 8, (1,), generator=g)) for e in range(E)]
    relabel, order = ep_moe.balanced_relabel(counts, world)
    assert sorted(relabel) == list(range(E)) and sorted(order) == list(range(E))
    assert all(order[relabel[e]] == e for e in range(E))
    tasks = [math.ceil(c / 32) for c in counts]
    per_rank = [sum(tasks[order[lab]] for lab in range(r, E, world)) for r in range(world)]
    rr = [sum(tasks[r::world]) for r in range(world)]
    assert max(per_rank) - min(per_rank) <= max(tasks)       # greedy bound
    assert max(per_rank) <= max(rr)                          # never worse than round-robin
    # the labels a rank holds are exactly the experts shard_experts(order=...) gives it
    W, _, _, _ = _data()
    for r in range(world):
        local = ep_moe.shard_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                     W["dn_z"], r, world, interleaved=True, order=order)
        want = torch.stack([W["gu_q"][order[lab]] for lab in range(r, E, world)])
        assert torch.equal(local[0], want)
