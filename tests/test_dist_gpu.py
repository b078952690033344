"""GPU parity of the multi-GPU partitions (kq.dist) with libkq doing the
math: world 1 in-process (the MoE stage entry points kq_moe_route /
kq_moe_experts_q4_0 / kq_moe_combine), and world 2 over NCCL in spawned
processes when two GPUs are visible. Bar for fp32 outputs: rel-L2 <= 1e-3 and
per element |out - ref| <= 1e-2 |ref| + 1e-3 rms(ref), against the oracle for
the GEMMs and, for the expert-parallel MoE, against the single-GPU fused
operator on the whole batch (stage-checked against the oracle in
test_moe_gpu.py): every expert sees the same rows either way, so the two runs
quantise identical intermediates."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _assert_close(out, ref, what=""):
    ok, msg = Q.check_close(out, ref)
    assert ok, f"{what} {msg}"


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
    _assert_close(out.cpu().numpy(), fused.cpu().numpy().astype(np.float64), "expert-parallel vs fused")


@pytest.mark.parametrize("mode", ["sum_dq", "sum_x"])
def test_moe_experts_q8_1_rows_bit_exact(cuda, mode):
    """kq_moe_experts_q4_0_q8_1 on rows quantised to q8_1 bytes equals
    kq_moe_experts_q4_0 on the fp32 rows bit for bit (same codes and fp16
    scales reach the same expert GEMMs), and the expert-parallel path with its
    q8_1 wire equals the fused operator."""
    import kq
    from kq import dist as kd

    rng = np.random.default_rng(5)
    T, E, H, I = 150, 4, 256, 512
    x, logits, wg, wu, wd = _moe_case(rng, T, E, H, I)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    er = t(rng.integers(0, E, size=T).astype(np.int32))
    y32 = kq.moe_experts_q4_0(t(x), er, t(wg), t(wu), t(wd), act_mode=mode)
    a8 = kq.quantize_q8_1(t(x), mode).reshape(T, -1)
    y8 = kq.moe_experts_q4_0_q8_1(a8, er, t(wg), t(wu), t(wd), act_mode=mode)
    assert np.array_equal(y32.cpu().numpy().view(np.uint32), y8.cpu().numpy().view(np.uint32))
    stats = {}
    out = kd.moe_expert_parallel(t(x), t(logits), t(wg), t(wu), t(wd), E, 2, act_mode=mode, stats=stats)
    fused = kq.moe_q4_0(t(x), t(logits), t(wg), t(wu), t(wd), topk=2, act_mode=mode)
    assert stats["wire"] == "q8_1"
    _assert_close(out.cpu().numpy(), fused.cpu().numpy().astype(np.float64), "expert-parallel (q8_1 rows) vs fused")


def test_nsharded_gemm_world1(cuda):
    from kq import dist as kd

    rng = np.random.default_rng(8)
    M, N, K = 16, 1024, 512
    w = Q.make_blocks("q4_0", rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = kd.NShardedGemm(torch.from_numpy(w.reshape(N, -1)).to(cuda), N, K, wtype="q4_0", act_mode="sum_dq")
    out = g(torch.from_numpy(x).to(cuda))
    _assert_close(out.cpu().numpy(), Q.gemm_f32act("q4_0", w.reshape(-1), x, M, N, K, Q.SUM_DQ))


@pytest.mark.parametrize("wtype,M,N,K", [("q4_0", 1, 512, 1024), ("q8_0", 4, 256, 512), ("q8_0", 200, 384, 1024),
                                         ("q4_1", 130, 136, 512)])
def test_scatter_epilogue_world1(cuda, wtype, M, N, K):
    """kq_gemm_f32act_scatter into two destinations at a column offset inside
    wider rows: every destination gets the same (correct) columns, nothing else
    is touched."""
    import kq

    rng = np.random.default_rng(M + N)
    w = Q.make_blocks(wtype, rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    ldo, col0 = N + 24, 12
    outs = [torch.full((M, ldo), -7.0, device=cuda) for _ in range(2)]
    kq.gemm_f32act_scatter(torch.from_numpy(w).to(cuda), torch.from_numpy(x).to(cuda), [o.data_ptr() for o in outs],
                           ldo, col0, M, N, K, wtype, "sum_dq")
    ref = Q.gemm_f32act(wtype, w, x, M, N, K, Q.SUM_DQ)
    for o in outs:
        o = o.cpu().numpy()
        ok, msg = Q.check_close(o[:, col0:col0 + N], ref)
        assert ok, msg
        assert np.all(o[:, :col0] == -7.0) and np.all(o[:, col0 + N:] == -7.0)


def test_peer_buffer_and_p2p_gemm_world1(cuda):
    from kq import dist as kd

    rng = np.random.default_rng(4)
    M, N, K = 64, 1024, 512
    w = Q.make_blocks("q8_0", rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = kd.NShardedGemm(torch.from_numpy(w.reshape(N, -1)).to(cuda), N, K, wtype="q8_0", mode="p2p")
    y = g(torch.from_numpy(x).to(cuda))
    ok, msg = Q.check_close(y.cpu().numpy(), Q.gemm_f32act("q8_0", w.reshape(-1), x, M, N, K, Q.SUM_DQ))
    g.close()
    assert ok, msg


# ---------------------------------------------------------------------------
# two ranks over NCCL (this file run by torchrun as a script; see _ranks_main)
# ---------------------------------------------------------------------------

def _ranks_main(which: str) -> None:
    """One rank of a two-rank case; launched by test_two_ranks_nccl through
    torch.distributed.run with a bounded runtime. Prints progress per rank."""
    import datetime
    import sys

    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    say = lambda *a: print(f"[rank {rank}]", *a, flush=True)  # noqa: E731
    failures = []
    try:
        import kq
        from kq import dist as kd

        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        if which in ("gemm", "gemm_p2p"):
            rng = np.random.default_rng(12)
            mode = "p2p" if which == "gemm_p2p" else "nccl"
            for (M, N, K) in ((64, 2048, 1024), (3, 1024, 512)):   # tensor-core and GEMV epilogues
                w = Q.make_blocks("q8_0", rng, N, K)
                x = rng.standard_normal((M, K)).astype(np.float32)
                shard = kd.NShardedGemm.shard_weight(torch.from_numpy(w.reshape(N, -1)), N, world, rank).to(dev)
                g = kd.NShardedGemm(shard, N, K, wtype="q8_0", act_mode="sum_dq", mode=mode)
                for rep in range(3):   # alternating buffers
                    out = g(t(x)).cpu().numpy()
                    ok, msg = Q.check_close(out, Q.gemm_f32act("q8_0", w.reshape(-1), x, M, N, K, Q.SUM_DQ))
                    say(which, M, N, K, rep, msg)
                    if not ok:
                        failures.append((M, N, K, rep, msg))
                dist.barrier()
                g.close()
        elif which == "moe":
            rng = np.random.default_rng(13)
            T_per, E, topk, H, I = 96, 8, 2, 256, 512
            x, logits, wg, wu, wd = _moe_case(rng, T_per * world, E, H, I)
            first, per = kd.expert_range(E, world, rank)
            sl = slice(rank * T_per, (rank + 1) * T_per)
            stats = {}
            out = kd.moe_expert_parallel(t(x[sl]), t(logits[sl]), t(wg[first:first + per]), t(wu[first:first + per]),
                                         t(wd[first:first + per]), E, topk, stats=stats)
            # the fused single-GPU operator on the whole batch with every expert
            ref = kq.moe_q4_0(t(x), t(logits), t(wg), t(wu), t(wd), topk=topk)[sl]
            ok, msg = Q.check_close(out.cpu().numpy(), ref.cpu().numpy().astype(np.float64))
            say("moe", stats, msg)
            if not ok:
                failures.append(msg)
        # every rank reaches this point on every path: the exit status carries the verdict
        dist.barrier()
    finally:
        dist.destroy_process_group()
    say("failures:", failures)
    sys.exit(1 if failures else 0)


@pytest.mark.parametrize("which", ["gemm", "gemm_p2p", "moe"])
def test_two_ranks_nccl(cuda, which):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import subprocess
    import sys

    env = dict(os.environ, NCCL_NVLS_ENABLE="0", KQ_DIST_CASE=which,
               PYTHONPATH=os.pathsep.join([p for p in sys.path if p]))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.abspath(__file__)]
    try:
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240, start_new_session=True)
    except subprocess.TimeoutExpired as e:
        pytest.fail(f"two-rank case {which} did not finish in 240 s:\n{e.stdout}\n{e.stderr}")
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


if __name__ == "__main__":
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), os.path.join(os.path.dirname(here), "k-search_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    _ranks_main(os.environ["KQ_DIST_CASE"])
