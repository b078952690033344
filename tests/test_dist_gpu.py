"""GPU parity of the multi-GPU partitions (kq.dist) with libkq doing the
math: world 1 in-process (the MoE stage entry points kq_moe_route /
kq_moe_experts_q4_0 / kq_moe_combine), and world 2 over NCCL in spawned
processes when two GPUs are visible. Bar for fp32 outputs: rel-L2 <= 1e-3 and
per element |out - ref| <= 1e-2 |ref| + 1e-3 rms(ref) against the oracle."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _moe_case(rng, T, E, H, I):
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    wg = np.stack([Q.make_q4_0_blocks(rng, I, H) for _ in range(E)])
    wu = np.stack([Q.make_q4_0_blocks(rng, I, H) for _ in range(E)])
    wd = np.stack([Q.make_q4_0_blocks(rng, H, I) for _ in range(E)])
    return x, logits, wg, wu, wd


def test_moe_stages_world1(cuda):
    import kq
    from kq import dist as kd

    rng = np.random.default_rng(3)
    T, E, topk, H, I = 200, 8, 2, 256, 512
    x, logits, wg, wu, wd = _moe_case(rng, T, E, H, I)
    idx, wts = kq.moe_route(torch.from_numpy(logits).to(cuda), topk)
    ridx, rw = Q.moe_route(logits, topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=1e-5, atol=1e-6)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out = kd.moe_expert_parallel(t(x), t(logits), t(wg), t(wu), t(wd), E, topk)
    fused = kq.moe_q4_0(t(x), t(logits), t(wg), t(wu), t(wd), topk=topk)
    ref = Q.moe_forward(x, logits, list(wg), list(wu), list(wd), topk, H, I, Q.SUM_DQ)
    Q.check_close(out.cpu().numpy(), ref)
    Q.check_close(fused.cpu().numpy(), ref)


def test_nsharded_gemm_world1(cuda):
    from kq import dist as kd

    rng = np.random.default_rng(8)
    M, N, K = 16, 1024, 512
    w = Q.make_blocks("q4_0", rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = kd.NShardedGemm(torch.from_numpy(w.reshape(N, -1)).to(cuda), N, K, wtype="q4_0", act_mode="sum_dq")
    out = g(torch.from_numpy(x).to(cuda))
    Q.check_close(out.cpu().numpy(), Q.gemm_f32act("q4_0", w.reshape(-1), x, M, N, K, Q.SUM_DQ))


# ---------------------------------------------------------------------------
# two ranks over NCCL
# ---------------------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, which):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from kq import dist as kd

        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        if which == "gemm":
            rng = np.random.default_rng(12)
            M, N, K = 64, 2048, 1024
            w = Q.make_blocks("q8_0", rng, N, K)
            x = rng.standard_normal((M, K)).astype(np.float32)
            shard = kd.NShardedGemm.shard_weight(torch.from_numpy(w.reshape(N, -1)), N, world, rank).to(dev)
            out = kd.NShardedGemm(shard, N, K, wtype="q8_0", act_mode="sum_dq")(t(x))
            if rank == 0:
                Q.check_close(out.cpu().numpy(), Q.gemm_f32act("q8_0", w.reshape(-1), x, M, N, K, Q.SUM_DQ))
        elif which == "moe":
            rng = np.random.default_rng(13)
            T_per, E, topk, H, I = 96, 8, 2, 256, 512
            x, logits, wg, wu, wd = _moe_case(rng, T_per * world, E, H, I)
            first, per = kd.expert_range(E, world, rank)
            sl = slice(rank * T_per, (rank + 1) * T_per)
            out = kd.moe_expert_parallel(t(x[sl]), t(logits[sl]), t(wg[first:first + per]), t(wu[first:first + per]),
                                         t(wd[first:first + per]), E, topk)
            ref = Q.moe_forward(x, logits, list(wg), list(wu), list(wd), topk, H, I, Q.SUM_DQ,
                                tokens=np.arange(sl.start, sl.stop))
            Q.check_close(out.cpu().numpy(), ref)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("which", ["gemm", "moe"])
def test_two_ranks_nccl(cuda, which):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, _free_port(), which), nprocs=2, join=True, start_method="spawn")
