"""Expert parallelism on the GPU through the C ABI: the EP layer at one rank equals the
single-GPU layer bit for bit (every engine), the re-slotting kernel equals the host reference,
and on two GPUs (NCCL, skipped with fewer) each rank's output equals the single-GPU layer's."""
import os
import socket
import tempfile

import pytest
import torch

from oracle import ref
from test_ep_host import RefOps

pytestmark = pytest.mark.gpu


def _case(E, H, I, T, tk, seed, dev):
    import workloads
    W = workloads.moe_weights(E, H, I, seed=seed, device=dev)
    inp = workloads.moe_inputs(T, H, E, seed=seed + 1, device=dev)
    import moe_router
    ids, w, _ = moe_router.route_topk(inp["hidden"], inp["router_w"], tk, bias=inp["bias"])
    xp = ref.kperm(inp["hidden"])  # the MoE K-interleave the RMSNorm kernel would write
    return W, inp["hidden"], xp.contiguous(), ids, w


@pytest.mark.parametrize("engine", ["auto", "ws", "tc"])
def test_ep_one_rank_matches_layer_bitwise(cuda, engine):
    import ep_moe
    import fused_moe_w4_v2
    W, hidden, xp, ids, w = _case(128, 2816, 704, 256, 8, 31, cuda)
    args = (W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"])
    want = fused_moe_w4_v2.moe_forward(hidden, *args, ids, w, hidden_perm=xp, engine=engine)
    layer = ep_moe.ExpertParallelMoE(*args, E_total=128, engine=engine)
    got = layer(xp, ids, w, out_dtype=torch.float16)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_ep_layout_kernel_matches_reference(cuda):
    import ep_moe
    g = torch.Generator().manual_seed(9)
    for S, El in ((4, 32), (8, 16), (1, 128), (3, 5)):
        cnt = torch.randint(0, 40, (S, El), generator=g, dtype=torch.int32)
        cnt[0, 0] = 0
        R = int(cnt.sum())
        o_ref, r_ref, i_ref = RefOps().layout(cnt, R)
        o, r, i = ep_moe.CudaOps().layout(cnt.to(cuda), R)
        assert torch.equal(o.cpu(), o_ref) and torch.equal(r.cpu(), r_ref) and torch.equal(i.cpu(), i_ref)


def test_gather_rows_and_combine_kernels(cuda):
    import ep_moe
    ops = ep_moe.CudaOps()
    g = torch.Generator().manual_seed(10)
    src = torch.randn(50, 2816, generator=g).half().to(cuda)
    idx = torch.randint(-1, 200, (70,), generator=g, dtype=torch.int32).to(cuda)
    got = ops.gather_rows(src, idx, 4, 70)
    want = torch.where((idx >= 0)[:, None], src[(idx.clamp(min=0) // 4).long()], torch.zeros((), dtype=src.dtype, device=cuda))
    assert torch.equal(got, want)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, world, out_dir, attempts=3, extra=()):
    """mp.spawn with a fresh rendezvous port per attempt: the port _free_port() released can be
    taken by another process before rank 0 binds it (EADDRINUSE), which says nothing about the
    code under test."""
    import torch.multiprocessing as mp
    for i in range(attempts):
        try:
            mp.spawn(fn, args=(world, _free_port(), out_dir) + tuple(extra), nprocs=world,
                     join=True)
            return
        except Exception as exc:  # the ranks' error arrives as ProcessRaisedException text
            if "EADDRINUSE" not in str(exc) or i == attempts - 1:
                raise


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import ep_moe
        W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, dev)
        local = ep_moe.shard_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                     W["dn_z"], rank, world)
        sl = slice(rank * 256, (rank + 1) * 256)
        layer = ep_moe.ExpertParallelMoE(*local, E_total=128)
        y = layer(xp[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous(), out_dtype=torch.float16)
        torch.save(y.cpu(), os.path.join(out_dir, f"y{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_bitwise_equal_single_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import fused_moe_w4_v2
    world = 2
    W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, cuda)
    want = fused_moe_w4_v2.moe_forward(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                       W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp,
                                       engine="auto").cpu()
    with tempfile.TemporaryDirectory() as d:
        _spawn(_worker, world, d)
        got = torch.cat([torch.load(os.path.join(d, f"y{r}.pt")) for r in range(world)])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def _worker_p2p(rank, world, port, out_dir, balanced=False):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import ep_moe
        W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, dev)
        relabel = order = None
        if balanced:  # owners dealt by the job-wide pairs per expert (every rank sees all ids)
            counts = torch.bincount(ids.flatten().long(), minlength=128).tolist()
            relabel, order = ep_moe.balanced_relabel(counts, world)
            if world == 1:  # one rank: any permutation must still give the same rows
                relabel = [(e * 37) % 128 for e in range(128)]
                order = [0] * 128
                for e, lab in enumerate(relabel):
                    order[lab] = e
        local = ep_moe.shard_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"],
                                     W["dn_z"], rank, world, interleaved=True, order=order)
        sl = slice(rank * 256, (rank + 1) * 256)
        layer = ep_moe.P2PExpertParallelMoE(*local, E_total=128, relabel=relabel)
        # three layers in a row through the same exchange region (epochs, reuse of the rows)
        ys = [layer(xp[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous(),
                    out_dtype=torch.float16).clone() for _ in range(3)]
        torch.cuda.synchronize()
        err = layer.check_errors()
        same = all(torch.equal(ys[0].view(torch.int16), y.view(torch.int16)) for y in ys[1:])
        torch.save({"y": ys[0].cpu(), "err": err, "same": same}, os.path.join(out_dir, f"p{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_p2p(world, balanced=False):
    import fused_moe_w4_v2
    W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, torch.device("cuda", 0))
    want = fused_moe_w4_v2.moe_forward(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                       W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp,
                                       engine="auto").cpu()
    with tempfile.TemporaryDirectory() as d:
        _spawn(_worker_p2p, world, d, extra=(balanced,))
        res = [torch.load(os.path.join(d, f"p{r}.pt")) for r in range(world)]
    for r in res:
        assert r["err"] == 0 and r["same"]
    got = torch.cat([r["y"] for r in res])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("balanced", [False, True])
def test_ep_p2p_one_rank_bitwise_equal_single_gpu(cuda, balanced):
    """The NVLink exchange at one rank (stores into its own region) equals the single-GPU layer,
    also with the experts relabelled (a permutation applied inside the counting sort)."""
    _run_p2p(1, balanced)


@pytest.mark.parametrize("balanced", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_p2p_multi_gpu_bitwise_equal_single_gpu(cuda, world, balanced):
    """2, 4 and 8 ranks (one canvas each, 128 / world experts per rank) through the NVLink
    exchange, three layers in a row: bit-identical to the single-GPU layer on all the tokens."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_p2p(world, balanced)


def test_p2p_barrier_gives_up_and_the_plan_is_empty(cuda):
    """A peer that never arrives, on one GPU: this GPU plays rank 0 of 2 and the peer's region
    is a local buffer nothing writes.  The barrier gives up after its 2 s limit and reports
    KNX_DEV_TIMEOUT; the counts step then writes the empty plan, the dispatch stores nothing into
    the peers' rows, and the context stays usable."""
    import time
    import _knx
    import fused_moe_w4
    lib = _knx.load()
    E, El, world, H, tk, T = 8, 4, 2, 64, 2, 4
    i64 = dict(dtype=torch.int64, device=cuda)
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(world)]
    cnt = [torch.zeros(world * E, dtype=torch.int32, device=cuda) for _ in range(world)]
    rows = [torch.full((T * tk, H), 3.0, dtype=torch.float16, device=cuda) for _ in range(world)]
    peer_flags = torch.tensor([f.data_ptr() for f in flags], **i64)
    peer_cnt = torch.tensor([c.data_ptr() for c in cnt], **i64)
    peer_rows = torch.tensor([r.data_ptr() for r in rows], **i64)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    st = _knx.stream_of(cuda.index or 0)
    p = _knx.ptr
    torch.cuda.synchronize()
    t0 = time.monotonic()
    assert lib.knx_ep_p2p_barrier(p(peer_flags), 0, world, 1, p(err), st) == 0
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(err.item()) & _knx.KNX_DEV_TIMEOUT
    assert 1.5 < waited < 30.0, waited
    assert int(flags[1][0].item()) == 1          # this rank's epoch reached the peer's flag
    err.zero_()
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, E, (T, tk), generator=g, dtype=torch.int32).to(cuda)
    counts, offsets, sorted_pair, _ = fused_moe_w4.moe_align_unpadded(ids, E)
    nplan = lib.knx_ep_p2p_plan_ints(E, El, world)
    plan = torch.full((nplan,), 7, dtype=torch.int32, device=cuda)
    assert lib.knx_ep_p2p_counts(p(counts.to(torch.int32)), E, El, 0, world, p(peer_cnt),
                                 p(peer_flags), 2, p(plan), p(err), st) == 0
    torch.cuda.synchronize()
    assert int(err.item()) & _knx.KNX_DEV_TIMEOUT
    assert (plan[:E] == -1).all()                          # no destination for any expert
    assert (plan[E:E + El + 2 + El * world] == 0).all()    # no receive rows, no segments
    xp = torch.randn(T, H, device=cuda).half()
    assert lib.knx_ep_p2p_dispatch(p(xp), H, tk, p(sorted_pair), p(offsets), E, El, p(plan),
                                   p(peer_rows), T * tk, st) == 0
    torch.cuda.synchronize()
    assert all(bool((r == 3.0).all()) for r in rows)
    assert torch.ones(8, device=cuda).sum().item() == 8.0
