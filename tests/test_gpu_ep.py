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
    import torch.multiprocessing as mp
    import fused_moe_w4_v2
    world = 2
    W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, cuda)
    want = fused_moe_w4_v2.moe_forward(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                       W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp,
                                       engine="auto").cpu()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _free_port(), d), nprocs=world, join=True)
        got = torch.cat([torch.load(os.path.join(d, f"y{r}.pt")) for r in range(world)])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def _worker_p2p(rank, world, port, out_dir):
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
                                     W["dn_z"], rank, world, interleaved=True)
        sl = slice(rank * 256, (rank + 1) * 256)
        layer = ep_moe.P2PExpertParallelMoE(*local, E_total=128)
        # three layers in a row through the same exchange region (epochs, reuse of the rows)
        ys = [layer(xp[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous(),
                    out_dtype=torch.float16).clone() for _ in range(3)]
        torch.cuda.synchronize()
        err = int(layer.ex.err.item())
        same = all(torch.equal(ys[0].view(torch.int16), y.view(torch.int16)) for y in ys[1:])
        torch.save({"y": ys[0].cpu(), "err": err, "same": same}, os.path.join(out_dir, f"p{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_p2p(world):
    import torch.multiprocessing as mp
    import fused_moe_w4_v2
    W, hidden, xp, ids, w = _case(128, 2816, 704, 256 * world, 8, 41, torch.device("cuda", 0))
    want = fused_moe_w4_v2.moe_forward(hidden, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                       W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp,
                                       engine="auto").cpu()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker_p2p, args=(world, _free_port(), d), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"p{r}.pt")) for r in range(world)]
    for r in res:
        assert r["err"] == 0 and r["same"]
    got = torch.cat([r["y"] for r in res])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_ep_p2p_one_rank_bitwise_equal_single_gpu(cuda):
    """The NVLink exchange at one rank (stores into its own region) equals the single-GPU layer."""
    _run_p2p(1)


def test_ep_p2p_two_gpus_bitwise_equal_single_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_p2p(2)
