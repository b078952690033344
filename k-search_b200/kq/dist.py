"""Multi-GPU sharding of the quantized-inference path: one process per GPU,
``torch.distributed`` (NCCL) for the exchanges, libkq kernels for the math.

Three partitions, one per operator family:

* GEMM / GEMV (``NShardedGemm``): the output dimension N is split into
  contiguous row ranges of the weight matrix (a q4_0/q4_1/q8_0 matrix is N rows
  of K/32 blocks, so a shard is one contiguous byte range). Every rank holds the
  fp32 activations, quantises them itself (the q8_1 codes are a function of the
  row alone, so every rank stages identical codes) and computes its [M, N/G]
  columns; one all-gather assembles [M, N].
* Flash decode (``plan_decode`` / ``decode_shard``): units are (sequence,
  KV-head group); ranks own whole units, balanced by KV length (longest first
  onto the least-loaded rank). No collective: each rank's outputs are final.
  ``gather_decode_outputs`` is the optional all-gather when one rank needs
  every output.
* MoE (``moe_expert_parallel``): expert-parallel. Rank r owns experts
  [r·E/G, (r+1)·E/G). Tokens stay data-parallel: each rank routes its own
  tokens, sends every (token, slot) pair to the owner of its expert (one
  all-to-all of row counts, one of rows and expert ids), runs its experts on
  what it received, and returns the rows (a second all-to-all), after which
  the weighted combine runs where the token lives.

Compute functions are parameters (defaulting to libkq's) so that the
exchange logic is testable on CPU with the ``gloo`` backend.

The GGML formats and formulas are those of KernelEvalPlus
(``llm_kernel_test/reference/gemm_ref.py``, ``quantize.py``); the reference
itself is single-device and has no sharded counterpart.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch
import torch.distributed as dist

__all__ = [
    "init_from_env", "split_range", "PeerBuffer", "NShardedGemm", "DecodeUnit", "plan_decode", "decode_shard",
    "gather_decode_outputs", "moe_expert_parallel", "expert_range",
]


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, torch.device]:
    """Join the process group torchrun describes (RANK, WORLD_SIZE, LOCAL_RANK,
    MASTER_ADDR/PORT); binds this process to GPU LOCAL_RANK when CUDA is
    present. A short timeout makes ranks that wait on a missing peer fail
    instead of hanging. Returns (rank, world, device)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if dev.type == "cuda" else "gloo")
        kw = {"device_id": dev} if backend == "nccl" else {}
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, dev


def split_range(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous balanced split of [0, n): (start, count) of ``rank``. Shard
    boundaries are multiples of ``align`` (the last shard takes the rest)."""
    if n < 0 or world < 1 or not 0 <= rank < world or align < 1:
        raise ValueError(f"bad split n={n} world={world} rank={rank} align={align}")
    units = -(-n // align)
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    start, stop = min(u0 * align, n), min(u1 * align, n)
    return start, stop - start


# ---------------------------------------------------------------------------
# GEMM: output dimension N sharded, all-gather of output columns
# ---------------------------------------------------------------------------

class _CudaArray:
    """Zero-copy view of a device allocation for torch.as_tensor."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (ptr, False), "version": 3}


class PeerBuffer:
    """An fp32 buffer of `numel` elements on every rank, each mapped into every
    other rank's address space with CUDA IPC (one process per GPU, one node).
    `ptrs[r]` is rank r's buffer as seen from this process; `local` is this
    rank's buffer as a tensor. The library owns the memory (kq_peer_alloc);
    close() unmaps and frees it."""

    def __init__(self, numel: int, device: torch.device, group=None):
        import ctypes
        from ._lib import check, lib

        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self._group = group
        self._lib, self._check = lib, check
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(device):
            check(lib().kq_peer_alloc(numel * 4, ctypes.byref(ptr), handle), "kq_peer_alloc")
        self._own = ptr.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                check(lib().kq_peer_open(hb, ctypes.byref(p)), "kq_peer_open")
                self.ptrs.append(p.value)
                self._opened.append(p.value)
        self.local = torch.as_tensor(_CudaArray(self._own, numel), device=device)
        self.numel = numel

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers, then (after a
        barrier, so no mapping of it remains) frees its own."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        for p in self._opened:
            self._check(self._lib().kq_peer_close(p), "kq_peer_close")
        self._opened = []
        self.local = None
        if self.world > 1:
            dist.barrier(group=self._group)
        self._check(self._lib().kq_peer_free(self._own), "kq_peer_free")
        self._own = None


def _default_gemm(weight, x, M, N, K, wtype, act_mode):
    from . import ops
    return ops.gemm_f32act(weight, x, M, N, K, wtype=wtype, act_mode=act_mode)


class NShardedGemm:
    """out[M, N] = x[M, K] · W[N, K]^T with W's N rows split over the ranks.

    ``weight_shard`` holds this rank's rows ``split_range(N, world, rank,
    align)`` as raw GGML blocks (uint8, rows × K/32 × block bytes). Each call
    quantises x on the fly, computes the local [M, n_r] columns and
    all-gathers them; shards of unequal width are padded to the widest for the
    collective and trimmed. ``gemm_fn(weight, x, M, n, K, wtype, act_mode)``
    is the per-rank compute (libkq by default). ``mode="p2p"`` instead stores
    the columns straight into every rank's output over peer mappings (see
    _forward_p2p); ``push_min_rows`` (p2p only) switches calls with more rows
    than that to local stores plus one strided copy per peer."""

    def __init__(self, weight_shard: torch.Tensor, N: int, K: int, wtype: str = "q4_0", act_mode: str = "sum_dq",
                 group=None, align: int = 128, gemm_fn: Callable | None = None, mode: str = "nccl",
                 push_min_rows: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.N, self.K, self.wtype, self.act_mode = N, K, wtype, act_mode
        self.splits = [split_range(N, self.world, r, align) for r in range(self.world)]
        self.n_local = self.splits[self.rank][1]
        self.n_max = max(c for _, c in self.splits)
        self.weight = weight_shard
        self.gemm_fn = gemm_fn or _default_gemm
        if mode not in ("nccl", "p2p"):
            raise ValueError("mode is 'nccl' or 'p2p'")
        self.mode = mode
        self.push_min_rows = push_min_rows
        self._bufs: list[PeerBuffer] = []   # p2p: two full-width outputs, used alternately
        self._buf_rows = 0
        self._calls = 0

    @staticmethod
    def shard_weight(weight_full: torch.Tensor, N: int, world: int, rank: int, align: int = 128) -> torch.Tensor:
        """This rank's contiguous row range of a full [N, ...] block matrix."""
        s, c = split_range(N, world, rank, align)
        return weight_full.reshape(N, -1)[s:s + c].contiguous()

    def local(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's columns, fp32 [M, n_local]."""
        M = x.shape[0]
        return self.gemm_fn(self.weight, x, M, self.n_local, self.K, self.wtype, self.act_mode)

    def close(self) -> None:
        for b in self._bufs:
            b.close()
        self._bufs = []

    def _forward_p2p(self, x: torch.Tensor) -> torch.Tensor | None:
        """The output lands in every rank's full-width buffer (CUDA IPC
        mappings of two alternating buffers) without a collective on the data:
        the GEMM's epilogue stores this rank's columns into every rank's
        buffer (kq_gemm_f32act_scatter: P2P stores over NVLink, overlapped
        with the MMAs of the next tiles). With push_min_rows set and more rows
        than that, the epilogue writes the local buffer only and one strided
        copy per peer (copy engines, one stream each) pushes the block
        afterwards. A one-element all-reduce then orders all of it before
        anything later on any rank's stream. The returned tensor is valid
        only until this object's next call: a peer that has passed that
        call's all-reduce may already be storing into the other buffer's
        successor, and a call with more rows than any before frees both
        buffers before allocating larger ones. Copy it out to keep it. None
        if the shape has no scatter epilogue."""
        from . import ops
        from ._lib import KQError, check, lib
        M = x.shape[0]
        if M > self._buf_rows:
            self.close()
            self._buf_rows = max(M, 2 * self._buf_rows)
            self._bufs = [PeerBuffer(self._buf_rows * self.N, x.device, self.group) for _ in range(2)]
        buf = self._bufs[self._calls & 1]
        s, c = self.splits[self.rank]
        push = self.push_min_rows is not None and M > self.push_min_rows and self.world > 1
        dests = [buf.ptrs[self.rank]] if push else buf.ptrs
        try:
            ops.gemm_f32act_scatter(self.weight, x, dests, self.N, s, M, c, self.K, self.wtype, self.act_mode,
                                    stream_of=x)
        except KQError as e:
            if e.status == 2:  # KQ_ERR_UNSUPPORTED: no scatter epilogue for this shape
                return None
            raise
        self._calls += 1
        if push and c > 0:
            main = torch.cuda.current_stream(x.device)
            if not hasattr(self, "_streams"):
                self._streams = [torch.cuda.Stream(x.device) for _ in range(self.world)]
            ready = torch.cuda.Event()
            ready.record(main)
            done = []
            pitch = self.N * 4
            for d in range(self.world):
                if d == self.rank:
                    continue
                st = self._streams[d]
                st.wait_event(ready)
                check(lib().kq_copy_2d(buf.ptrs[d] + s * 4, pitch, buf.ptrs[self.rank] + s * 4, pitch, c * 4, M,
                                       st.cuda_stream), "kq_copy_2d")
                ev = torch.cuda.Event()
                ev.record(st)
                done.append(ev)
            for ev in done:
                main.wait_event(ev)
        if self.world > 1:
            if not hasattr(self, "_flag"):
                self._flag = torch.zeros(1, dtype=torch.int32, device=x.device)
            dist.all_reduce(self._flag, group=self.group)
        return buf.local[:M * self.N].view(M, self.N)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        M = x.shape[0]
        if self.mode == "p2p":
            y = self._forward_p2p(x)
            if y is not None:
                if out is None:
                    return y
                out.copy_(y)
                return out
        part = self.local(x)
        if self.world == 1:
            if out is None:
                return part
            out.copy_(part)
            return out
        if self.n_local != self.n_max:
            padded = torch.zeros((M, self.n_max), dtype=part.dtype, device=part.device)
            padded[:, :self.n_local] = part
            part = padded
        gathered = torch.empty((self.world * M, self.n_max), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(gathered, part.contiguous(), group=self.group)
        gathered = gathered.view(self.world, M, self.n_max)
        if out is None:
            out = torch.empty((M, self.N), dtype=part.dtype, device=part.device)
        if all(c == self.n_max for _, c in self.splits):
            out.view(M, self.world, self.n_max).copy_(gathered.permute(1, 0, 2))
        else:
            for r, (s, c) in enumerate(self.splits):
                out[:, s:s + c] = gathered[r, :, :c]
        return out

    __call__ = forward


# ---------------------------------------------------------------------------
# Flash decode: (sequence, KV-head group) units, no collective
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class DecodeUnit:
    seq: int           # batch index
    head0: int         # first KV head of the group
    heads: int         # KV heads in the group
    cost: int          # KV rows × heads (what the decode streams)


@dataclass
class DecodePlan:
    world: int
    units: list[list[DecodeUnit]] = field(default_factory=list)   # per rank

    def load(self) -> list[int]:
        return [sum(u.cost for u in us) for us in self.units]


def plan_decode(seqlens: Sequence[int], Hkv: int, world: int, head_group: int = 8) -> DecodePlan:
    """Assign (sequence, KV-head group) units to ranks, longest first onto the
    least-loaded rank (ties to the lower rank). KV heads are grouped
    ``head_group`` at a time (the decode kernel's fast path reads 8 KV heads per
    token row), falling back to smaller groups that divide Hkv."""
    if world < 1 or Hkv < 1:
        raise ValueError("world and Hkv must be positive")
    hg = max(g for g in range(1, min(head_group, Hkv) + 1) if Hkv % g == 0)
    units = [DecodeUnit(b, h0, hg, int(L) * hg) for b, L in enumerate(seqlens) for h0 in range(0, Hkv, hg)]
    units.sort(key=lambda u: (-u.cost, u.seq, u.head0))
    plan = DecodePlan(world, [[] for _ in range(world)])
    load = [0] * world
    for u in units:
        r = min(range(world), key=lambda i: (load[i], i))
        plan.units[r].append(u)
        load[r] += u.cost
    for us in plan.units:
        us.sort(key=lambda u: (u.seq, u.head0))
    return plan


def _default_decode(q, k, v, cu, B, Hq, Hkv, D, max_seqlen, scale):
    from . import ops
    return ops.flash_decode_ragged(q, k, v, cu, Hkv, max_seqlen=max_seqlen, scale=scale)


def decode_shard(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cu_seqlens: torch.Tensor,
                 Hq: int, Hkv: int, D: int, scale: float, max_seqlen: int,
                 decode_fn: Callable | None = None) -> torch.Tensor:
    """Decode this rank's sequences: q fp16 [B_r, Hq, D] and a local cache
    (q8_0, [rows, Hkv, D] blocks) holding only those sequences; the math is
    the single-GPU kernel's, so per-unit results are those of one GPU."""
    fn = decode_fn or _default_decode
    return fn(q, k_cache, v_cache, cu_seqlens, q.shape[0], Hq, Hkv, D, max_seqlen, scale)


def gather_decode_outputs(local_out: torch.Tensor, plan: DecodePlan, rank: int, B: int, group=None) -> torch.Tensor:
    """All-gather per-rank decode outputs into [B, Hq, D] on every rank.
    Requires whole-sequence units (head group == Hkv), as ``plan_decode``
    produces when Hkv <= head_group. ``local_out`` rows follow
    ``plan.units[rank]`` order."""
    world = plan.world
    seqs = [[u.seq for u in us] for us in plan.units]
    if any(len(set(s)) != len(s) for s in seqs):
        raise ValueError("gather_decode_outputs needs whole-sequence units")
    rows_max = max(len(s) for s in seqs)
    tail = tuple(local_out.shape[1:])
    send = torch.zeros((rows_max,) + tail, dtype=local_out.dtype, device=local_out.device)
    send[:local_out.shape[0]] = local_out
    if world == 1:
        gathered = send.unsqueeze(0)
    else:
        gathered = torch.empty((world * rows_max,) + tail, dtype=local_out.dtype, device=local_out.device)
        dist.all_gather_into_tensor(gathered, send, group=group)
        gathered = gathered.view((world, rows_max) + tail)
    out = torch.empty((B,) + tail, dtype=local_out.dtype, device=local_out.device)
    for r, s in enumerate(seqs):
        if s:
            out[torch.tensor(s, device=out.device)] = gathered[r, :len(s)]
    return out


# ---------------------------------------------------------------------------
# MoE: expert parallel, all-to-all dispatch and combine
# ---------------------------------------------------------------------------

def expert_range(E: int, world: int, rank: int) -> tuple[int, int]:
    """Experts owned by ``rank``: [first, first + count). E must divide evenly."""
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    c = E // world
    return rank * c, c


def _ops():
    from . import ops
    return ops


def moe_expert_parallel(x: torch.Tensor, router_logits: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                        w_down: torch.Tensor, E: int, topk: int = 2, act_mode: str = "sum_dq", group=None,
                        route_fn: Callable | None = None, experts_fn: Callable | None = None,
                        combine_fn: Callable | None = None, stats: dict | None = None,
                        quant_fn: Callable | None = None, experts_q8_fn: Callable | None = None) -> torch.Tensor:
    """Expert-parallel grouped MoE FFN for this rank's tokens.

    x fp32 [T_r, H] and router_logits fp32 [T_r, E] are this rank's tokens;
    w_gate / w_up / w_down hold only this rank's experts (``expert_range``),
    laid out as for ``ops.moe_q4_0``. Returns fp32 [T_r, H], the same values
    the single-GPU operator gives for these tokens.

    Dispatched rows travel as q8_1 blocks (H/32 blocks of 36 bytes: codes plus
    fp16 d and s, 1.125 bytes per value instead of 4) when act_mode is
    "sum_x" or "sum_dq": each token is quantised once where it lives and the
    owning rank runs its experts on the received codes, which are the codes
    the single-GPU operator forms (its staging holds the same fp16 d and s).
    Mode "f32" keeps fp32 d and s, so its rows travel as fp32.

    route_fn(logits, topk) -> (idx int32 [T, k], wts fp32 [T, k]);
    experts_fn(x_rows, local_expert int32 [P], w_gate, w_up, w_down, act_mode) -> [P, H] (fp32 rows);
    quant_fn(x, act_mode) -> uint8 [T, H/32 * 36] and
    experts_q8_fn(a_rows uint8, local_expert, w_gate, w_up, w_down, act_mode) -> [P, H] (q8_1 rows);
    combine_fn(y [T*k, H], wts) -> [T, H]. Defaults: libkq. Injecting
    experts_fn alone selects fp32 rows."""
    use_q8 = act_mode in ("sum_x", "sum_dq") and (experts_q8_fn is not None or experts_fn is None)
    needs_ops = not route_fn or not combine_fn or (use_q8 and not (quant_fn and experts_q8_fn)) or \
        (not use_q8 and not experts_fn)
    ops = _ops() if needs_ops else None
    route_fn = route_fn or (lambda lg, k: ops.moe_route(lg, k))
    experts_fn = experts_fn or (lambda xr, er, g, u, d, am: ops.moe_experts_q4_0(xr, er, g, u, d, act_mode=am))
    quant_fn = quant_fn or (lambda xx, am: ops.quantize_q8_1(xx, am))
    experts_q8_fn = experts_q8_fn or (
        lambda ar, er, g, u, d, am: ops.moe_experts_q4_0_q8_1(ar, er, g, u, d, act_mode=am))
    combine_fn = combine_fn or (lambda y, w: ops.moe_combine(y, w))
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    first, per = expert_range(E, world, rank)
    T, H = x.shape
    idx, wts = route_fn(router_logits, topk)
    flat = idx.reshape(-1).to(torch.int64)                        # pair p = t * topk + k
    dest = torch.div(flat, per, rounding_mode="floor")
    order = torch.argsort(dest, stable=True)                      # pairs grouped by owning rank
    send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
    rows = quant_fn(x, act_mode).reshape(T, -1) if use_q8 else x   # what travels per token
    x_send = rows.index_select(0, torch.div(order, topk, rounding_mode="floor"))
    e_send = (flat - dest * per).index_select(0, order).to(torch.int32)
    if world == 1:
        x_recv, e_recv, recv_counts = x_send, e_send, send_counts
    else:
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        x_recv = torch.empty((sum(rc), rows.shape[1]), dtype=rows.dtype, device=x.device)
        e_recv = torch.empty((sum(rc),), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(x_recv, x_send, rc, sc, group=group)
        dist.all_to_all_single(e_recv, e_send, rc, sc, group=group)
    if x_recv.shape[0]:
        fn = experts_q8_fn if use_q8 else experts_fn
        y_recv = fn(x_recv, e_recv, w_gate, w_up, w_down, act_mode)
    else:
        y_recv = torch.empty((0, H), dtype=x.dtype, device=x.device)
    if world == 1:
        y_back = y_recv
    else:
        y_back = torch.empty((int(send_counts.sum()), H), dtype=y_recv.dtype, device=x.device)
        dist.all_to_all_single(y_back, y_recv, sc, rc, group=group)
    y_pairs = torch.empty((T * topk, H), dtype=y_back.dtype, device=x.device)
    y_pairs[order] = y_back
    if stats is not None:
        stats.update(send_rows=int(send_counts.sum()), recv_rows=int(recv_counts.sum()),
                     recv_counts=recv_counts.tolist(), row_bytes=int(rows.shape[1] * rows.element_size()),
                     wire="q8_1" if use_q8 else "f32")
    return combine_fn(y_pairs, wts)
