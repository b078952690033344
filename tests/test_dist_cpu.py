"""Host logic of the multi-GPU partitions (kq.dist) on CPU: world_size-2
``gloo`` process groups, with the per-rank compute injected from the oracle
so that only the sharding and exchange logic is under test. Each sharded
result must equal the single-device oracle on the same inputs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kq import dist as kd
from oracle import quant as Q


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world, *args):
    port = _free_port()
    mp.start_processes(_entry, args=(fn, world, port) + args, nprocs=world, join=True, start_method="spawn")


def _entry(rank, fn, world, port, *args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# pure host logic
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("n,world,align", [(11008, 8, 128), (14336, 3, 128), (100, 4, 1), (5, 8, 1), (160, 2, 32)])
def test_split_range_covers(n, world, align):
    parts = [kd.split_range(n, world, r, align) for r in range(world)]
    pos = 0
    for s, c in parts:
        assert s == pos and c >= 0
        if c and s + c < n:
            assert (s + c) % align == 0
        pos += c
    assert pos == n
    counts = [c for _, c in parts]
    assert max(counts) - min(counts) <= align


def test_plan_decode_balance():
    rng = np.random.default_rng(0)
    L = rng.integers(64, 8193, size=32)
    for world in (1, 2, 4, 8):
        plan = kd.plan_decode(L, Hkv=8, world=world)
        seen = sorted((u.seq, u.head0) for us in plan.units for u in us)
        assert seen == [(b, 0) for b in range(32)]              # 8 KV heads: whole sequences
        load = plan.load()
        assert sum(load) == int(L.sum()) * 8
        # longest-first greedy: makespan <= mean + largest unit
        assert max(load) <= sum(load) / world + int(L.max()) * 8
    plan = kd.plan_decode([100, 50], Hkv=16, world=4)          # two 8-head groups per sequence
    assert sorted((u.seq, u.head0, u.heads) for us in plan.units for u in us) == \
        [(0, 0, 8), (0, 8, 8), (1, 0, 8), (1, 8, 8)]
    plan = kd.plan_decode([10], Hkv=6, world=2)                 # group = largest divisor <= 8
    assert [u.heads for us in plan.units for u in us] == [6]


def test_expert_range():
    assert [kd.expert_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 2), (4, 2), (6, 2)]
    with pytest.raises(ValueError):
        kd.expert_range(8, 3, 0)


# ---------------------------------------------------------------------------
# N-sharded GEMM + all-gather
# ---------------------------------------------------------------------------

def _oracle_gemm(weight, x, M, n, K, wtype, act_mode):
    mode = {"sum_x": Q.SUM_X, "sum_dq": Q.SUM_DQ, "f32": Q.ACT_F32}[act_mode]
    out = Q.gemm_f32act(wtype, weight.numpy().reshape(-1), x.numpy(), M, n, K, mode)
    return torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32))


def _gemm_rank(rank, world, wtype, M, N, K, align):
    rng = np.random.default_rng(11)
    w = Q.make_blocks(wtype, rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wt = torch.from_numpy(w.reshape(N, -1))
    shard = kd.NShardedGemm.shard_weight(wt, N, world, rank, align)
    g = kd.NShardedGemm(shard, N, K, wtype=wtype, act_mode="sum_dq", align=align, gemm_fn=_oracle_gemm)
    out = g(torch.from_numpy(x))
    ref = Q.gemm_f32act(wtype, w.reshape(-1), x, M, N, K, Q.SUM_DQ).astype(np.float32)
    np.testing.assert_array_equal(out.numpy(), ref)


@pytest.mark.parametrize("wtype,M,N,K,align", [("q4_0", 3, 256, 128, 64), ("q8_0", 2, 160, 64, 32)])
def test_nsharded_gemm_gloo(wtype, M, N, K, align):
    _spawn(_gemm_rank, 2, wtype, M, N, K, align)


# ---------------------------------------------------------------------------
# sequence-sharded decode (+ optional gather)
# ---------------------------------------------------------------------------

def _decode_rank(rank, world):
    rng = np.random.default_rng(5)
    B, Hq, Hkv, D = 6, 8, 2, 64
    L = rng.integers(1, 40, size=B)
    L[2] = 0                                                     # an empty sequence
    scale = 1.0 / np.sqrt(D)
    q = rng.standard_normal((B, Hq, D)).astype(np.float16)
    ks = [Q.quantize_q8_0(rng.standard_normal((int(l) * Hkv, D)).astype(np.float32)) for l in L]
    vs = [Q.quantize_q8_0(rng.standard_normal((int(l) * Hkv, D)).astype(np.float32)) for l in L]
    plan = kd.plan_decode(L, Hkv, world)
    mine = [u.seq for u in plan.units[rank]]
    cu = np.concatenate([[0], np.cumsum([L[b] for b in mine])]).astype(np.int32)
    k_loc = np.concatenate([ks[b].reshape(-1) for b in mine] + [np.zeros(0, np.uint8)])
    v_loc = np.concatenate([vs[b].reshape(-1) for b in mine] + [np.zeros(0, np.uint8)])

    def decode_fn(qq, k, v, cu_, Bl, Hq_, Hkv_, D_, max_seqlen, sc):
        o = Q.flash_decode_ragged(qq.numpy(), k.numpy(), v.numpy(), cu_.numpy(), Hq_, Hkv_, D_, sc)
        return torch.from_numpy(o.astype(np.float16))

    out = kd.decode_shard(torch.from_numpy(q[mine]), torch.from_numpy(k_loc), torch.from_numpy(v_loc),
                          torch.from_numpy(cu), Hq, Hkv, D, scale, int(L.max()), decode_fn=decode_fn)
    full = kd.gather_decode_outputs(out, plan, rank, B)
    cu_all = np.concatenate([[0], np.cumsum(L)]).astype(np.int32)
    ref = Q.flash_decode_ragged(q, np.concatenate([k.reshape(-1) for k in ks]),
                                np.concatenate([v.reshape(-1) for v in vs]), cu_all, Hq, Hkv, D, scale)
    np.testing.assert_array_equal(full.numpy(), ref.astype(np.float16))


def test_decode_shard_gloo():
    _spawn(_decode_rank, 2)


# ---------------------------------------------------------------------------
# expert-parallel MoE with all-to-all dispatch and combine
# ---------------------------------------------------------------------------

def _moe_rank(rank, world, T_per, E, topk, H, I):
    rng = np.random.default_rng(21)
    T = T_per * world
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    wg = [Q.make_q4_0_blocks(rng, I, H) for _ in range(E)]
    wu = [Q.make_q4_0_blocks(rng, I, H) for _ in range(E)]
    wd = [Q.make_q4_0_blocks(rng, H, I) for _ in range(E)]
    first, per = kd.expert_range(E, world, rank)
    t0 = rank * T_per
    xs, ls = x[t0:t0 + T_per], logits[t0:t0 + T_per]

    def route_fn(lg, k):
        idx, w = Q.moe_route(lg.numpy(), k)
        return torch.from_numpy(idx), torch.from_numpy(w)      # fp64 weights: the oracle's combine

    def experts_fn(xr, er, g, u, d, am):
        xr, er = xr.numpy(), er.numpy()
        y = np.zeros((xr.shape[0], H), dtype=np.float64)
        for e in range(per):
            sel = np.nonzero(er == e)[0]
            if len(sel) == 0:
                continue
            xt = np.ascontiguousarray(xr[sel])
            m = len(sel)
            gg = Q.gemm_f32act("q4_0", wg[first + e], xt, m, I, H, Q.SUM_DQ)
            uu = Q.gemm_f32act("q4_0", wu[first + e], xt, m, I, H, Q.SUM_DQ)
            h = (Q.silu(gg) * uu.astype(np.float64)).astype(np.float32)
            y[sel] = Q.gemm_f32act("q4_0", wd[first + e], h, m, H, I, Q.SUM_DQ)
        return torch.from_numpy(y)

    def combine_fn(y, w):
        return (y.view(T_per, topk, H) * w.unsqueeze(-1)).sum(dim=1)

    stats = {}
    out = kd.moe_expert_parallel(torch.from_numpy(xs), torch.from_numpy(ls), None, None, None, E, topk,
                                 route_fn=route_fn, experts_fn=experts_fn, combine_fn=combine_fn, stats=stats)
    ref = Q.moe_forward(x, logits, wg, wu, wd, topk, H, I, Q.SUM_DQ, tokens=np.arange(t0, t0 + T_per))
    assert stats["send_rows"] == T_per * topk
    np.testing.assert_allclose(out.numpy(), ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("T_per,E,topk", [(12, 4, 2), (3, 8, 2), (7, 2, 1)])
def test_moe_expert_parallel_gloo(T_per, E, topk):
    _spawn(_moe_rank, 2, T_per, E, topk, 64, 96)


def _moe_q8_rank(rank, world, T_per, E, topk, H, I):
    """As _moe_rank, with the rows travelling as q8_1 blocks (the default wire
    for "sum_dq"): quant_fn and experts_q8_fn stand in for libkq."""
    rng = np.random.default_rng(22)
    T = T_per * world
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    wg = [Q.make_q4_0_blocks(rng, I, H) for _ in range(E)]
    wu = [Q.make_q4_0_blocks(rng, I, H) for _ in range(E)]
    wd = [Q.make_q4_0_blocks(rng, H, I) for _ in range(E)]
    first, per = kd.expert_range(E, world, rank)
    t0 = rank * T_per
    xs, ls = x[t0:t0 + T_per], logits[t0:t0 + T_per]
    nb = H // 32

    def route_fn(lg, k):
        idx, w = Q.moe_route(lg.numpy(), k)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def quant_fn(xx, am):
        assert am == "sum_dq"
        return torch.from_numpy(Q.quantize_q8_1(xx.numpy(), Q.SUM_DQ).reshape(xx.shape[0], -1))

    def experts_q8_fn(ar, er, g, u, d, am):
        ar, er = ar.numpy().reshape(-1, nb, 36), er.numpy()
        da = ar[:, :, 0:2].copy().view(np.float16)[:, :, 0].astype(np.float32)
        sa = ar[:, :, 2:4].copy().view(np.float16)[:, :, 0].astype(np.float32)
        qa = ar[:, :, 4:].copy().view(np.int8)
        y = np.zeros((ar.shape[0], H), dtype=np.float64)
        for e in range(per):
            sel = np.nonzero(er == e)[0]
            if len(sel) == 0:
                continue
            m = len(sel)
            gg = Q.gemm_codes("q4_0", wg[first + e], qa[sel], da[sel], sa[sel], m, I, H)
            uu = Q.gemm_codes("q4_0", wu[first + e], qa[sel], da[sel], sa[sel], m, I, H)
            h = (Q.silu(gg) * uu.astype(np.float64)).astype(np.float32)
            y[sel] = Q.gemm_f32act("q4_0", wd[first + e], h, m, H, I, Q.SUM_DQ)
        return torch.from_numpy(y)

    def combine_fn(y, w):
        return (y.view(T_per, topk, H) * w.unsqueeze(-1)).sum(dim=1)

    stats = {}
    out = kd.moe_expert_parallel(torch.from_numpy(xs), torch.from_numpy(ls), None, None, None, E, topk,
                                 route_fn=route_fn, combine_fn=combine_fn, stats=stats, quant_fn=quant_fn,
                                 experts_q8_fn=experts_q8_fn)
    ref = Q.moe_forward(x, logits, wg, wu, wd, topk, H, I, Q.SUM_DQ, tokens=np.arange(t0, t0 + T_per))
    assert stats["wire"] == "q8_1" and stats["row_bytes"] == nb * 36
    np.testing.assert_allclose(out.numpy(), ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("T_per,E,topk", [(12, 4, 2), (3, 8, 2)])
def test_moe_expert_parallel_q8_1_rows_gloo(T_per, E, topk):
    """Expert-parallel dispatch of q8_1 rows (36 bytes per 32 values instead of
    128) gives the single-device oracle's result exactly."""
    _spawn(_moe_q8_rank, 2, T_per, E, topk, 64, 96)


# ---------------------------------------------------------------------------
# failure detection on the host: a rank that leaves between steps
# ---------------------------------------------------------------------------

def _leaver_rank(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import time
    rk, wd, _ = kd.init_from_env(backend="gloo", timeout_s=3.0)
    t = torch.ones(8)
    dist.all_reduce(t)  # step 1: every rank takes part
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)  # step 2: the peer is gone
        q.put(("completed", time.monotonic() - t0, float(t[0])))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put((type(e).__name__, time.monotonic() - t0, str(e)[:200]))
    os._exit(0)  # no collective teardown with a dead peer


def test_rank_leaving_between_steps_errors_instead_of_hanging():
    """kq.dist.init_from_env gives the group a short timeout: after rank 1
    exits between two steps, rank 0's next collective ends with an error (the
    peer's closed connection or the timeout) within seconds instead of
    hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind, secs, detail = q.get(timeout=90)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert kind != "completed", detail
    assert secs < 30, (kind, secs, detail)
