"""GPU parity of flash-attention decode over q8_0 / q4_0 / fp16 KV caches.

Bar: rel-L2 <= 1e-3 and per element |out - ref| <= 1e-2 |ref| + 1e-3 rms(ref)
against the fp64 oracle on the same q8_0 bytes; fp16 outputs are compared
after the oracle's fp64 result (the fp16 rounding of the output is inside
the bar). Plus the harness's NMSE <= 0.05 gate against unquantised K/V.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_golden_fixture(cuda):
    import kq
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "flash_attn.npz"))
    B, S, H, D = (int(g[k]) for k in "BSHD")
    got = kq.flash_attn_q8_0(_t(g["q"], cuda), _t(g["k_q8_0"], cuda), _t(g["v_q8_0"], cuda), B, S, H, D).cpu().numpy()
    ok, msg = Q.check_close(got, g["ref_on_q8_0"])
    assert ok, msg
    assert Q.nmse(got, g["ref_on_fp32"]) < 0.05


@pytest.mark.parametrize("B,S,H,D", [(1, 512, 32, 128), (8, 1000, 4, 128), (3, 4096, 2, 64), (2, 1, 3, 32),
                                     (16, 300, 2, 256), (2, 100, 3, 96), (6, 2000, 5, 160),
                                     # tensor-core path (D = 128, heads in groups of 8): partial tiles,
                                     # partial query groups, one-token cache, many query groups
                                     (5, 77, 8, 128), (12, 1000, 16, 128), (3, 1, 8, 128), (4, 33, 32, 128),
                                     (512, 64, 8, 128), (9, 8192, 8, 128)])
def test_mha_parity(cuda, B, S, H, D):
    import kq
    rng = np.random.default_rng(B * S + H)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kf = rng.standard_normal((S * H, D)).astype(np.float32)
    vf = rng.standard_normal((S * H, D)).astype(np.float32)
    k, v = Q.quantize_q8_0(kf), Q.quantize_q8_0(vf)
    got = kq.flash_attn_q8_0(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D))
    assert ok, msg


def test_harness_void_entry(cuda):
    import kq
    rng = np.random.default_rng(5)
    B, S, H, D = 2, 512, 32, 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kf = rng.standard_normal((S, H, D)).astype(np.float32)
    vf = rng.standard_normal((S, H, D)).astype(np.float32)
    k, v = Q.quantize_q8_0(kf.reshape(-1, D)), Q.quantize_q8_0(vf.reshape(-1, D))
    out = torch.empty((B, H, D), dtype=torch.float32, device=cuda)
    qd, kd, vd = _t(q, cuda), _t(k, cuda), _t(v, cuda)
    torch.cuda.synchronize()
    kq.lib().kq_flash_attn_q8_0(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), B, S, H, D)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D))
    assert ok, msg
    # harness gate: attention on the unquantised caches
    ref = np.einsum("bhs,shd->bhd", _softmax(np.einsum("bhd,shd->bhs", q, kf) / np.sqrt(D)), vf)
    assert Q.nmse(got, ref) < 0.05


_FA_DEFS = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                      "flash_attention_definitions.json")))["definitions"]


def _cache(fmt, x, D):
    """fp32 [S, H, D] -> cache bytes as the harness builds them (op_test_handler.py:489-534)."""
    if fmt == "q8_0":
        return Q.quantize_q8_0(x.reshape(-1, D))
    if fmt == "q4_0":
        return Q.quantize_q4_0(x.reshape(-1, D))
    return x.astype(np.float16)


@pytest.mark.parametrize("fmt", ["q4_0", "f16"])
@pytest.mark.parametrize("B,S,H,D", [(1, 512, 32, 128), (8, 1000, 4, 128), (3, 4096, 2, 64), (2, 1, 3, 32),
                                     (16, 300, 2, 256), (5, 77, 28, 128), (2, 100, 3, 96), (1, 8192, 28, 128)])
def test_mha_parity_kv_formats(cuda, fmt, B, S, H, D):
    import kq
    rng = np.random.default_rng(B * S + H + len(fmt))
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    v = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    got = kq.flash_attn(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D, fmt).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D, fmt))
    assert ok, msg


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "f16"])
def test_mha_unaligned_caches(cuda, fmt):
    """Caches that start 2 bytes past an aligned address (the ABI asks for
    2-byte alignment only): the fp16 vector loads give way to element loads."""
    import kq
    rng = np.random.default_rng(3)
    B, S, H, D = 3, 700, 4, 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    v = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    nb = k.nbytes
    kbuf = torch.zeros(nb + 16, dtype=torch.uint8, device=cuda)
    vbuf = torch.zeros(nb + 16, dtype=torch.uint8, device=cuda)
    kbuf[2:2 + nb] = _t(np.frombuffer(k.tobytes(), dtype=np.uint8), cuda)
    vbuf[2:2 + nb] = _t(np.frombuffer(v.tobytes(), dtype=np.uint8), cuda)
    got = kq.flash_attn(_t(q, cuda), kbuf[2:2 + nb], vbuf[2:2 + nb], B, S, H, D, fmt).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D, fmt))
    assert ok, msg


@pytest.mark.parametrize("defn", _FA_DEFS, ids=lambda d: os.path.basename(d["definition"])[:-5])
def test_definition_flash_attention(cuda, defn):
    """Every flash_attention definition the reference ships, at each of its
    batch sizes, through the harness mirror (KV format decided from the
    definition as the harness decides it). Queries are independent, so the
    full batch runs and up to four query rows are checked against the oracle
    on the cache bytes and against the harness's NMSE gate on fp32 K/V."""
    import kq
    S, H, D = defn["S"], defn["H"], defn["D"]
    spec = {"inputs": {"key_cache": {"dtype": defn["key_cache_dtype"]}}, "variant": defn["variant"],
            "tags": defn["tags"]}
    fmt = kq.harness.flash_attention_kv_format(spec)
    rng = np.random.default_rng(S + H + len(defn["definition"]))
    kf = rng.standard_normal((S, H, D)).astype(np.float32)
    vf = rng.standard_normal((S, H, D)).astype(np.float32)
    k, v = _cache(fmt, kf, D), _cache(fmt, vf, D)
    kd, vd = _t(k, cuda), _t(v, cuda)
    for B in defn["B"]:
        q = rng.standard_normal((B, H, D)).astype(np.float32)
        got = kq.harness.flash_attention_forward(_t(q, cuda), kd, vd, B, S, H, D, fmt).cpu().numpy()
        rows = np.unique(np.array([0, B // 3, (2 * B) // 3, B - 1]))
        ok, msg = Q.check_close(got[rows], Q.flash_decode_mha(q[rows], k, v, S, H, D, fmt))
        assert ok, f"B={B}: {msg}"
        ref = np.einsum("bhs,shd->bhd", _softmax(np.einsum("bhd,shd->bhs", q[rows], kf) / np.sqrt(D)), vf)
        assert Q.nmse(got[rows], ref) < 0.05, f"B={B}"


@pytest.mark.parametrize("fmt,entry", [("q4_0", "kq_flash_attn_q4_0"), ("f16", "kq_flash_attn_f16")])
def test_harness_void_entry_kv_formats(cuda, fmt, entry):
    import kq
    rng = np.random.default_rng(11)
    B, S, H, D = 3, 512, 28, 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    v = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    out = torch.empty((B, H, D), dtype=torch.float32, device=cuda)
    qd, kd, vd = _t(q, cuda), _t(k, cuda), _t(v, cuda)
    torch.cuda.synchronize()
    getattr(kq.lib(), entry)(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), B, S, H, D)
    torch.cuda.synchronize()
    assert kq.lib().kq_last_error() == b""
    ok, msg = Q.check_close(out.cpu().numpy(), Q.flash_decode_mha(q, k, v, S, H, D, fmt))
    assert ok, msg


def _softmax(x):
    x = x - x.max(-1, keepdims=True)
    e = np.exp(x)
    return e / e.sum(-1, keepdims=True)


def _ragged_case(rng, lens, Hq, Hkv, D):
    B = len(lens)
    cu = np.zeros(B + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    T = int(cu[-1])
    q = rng.standard_normal((B, Hq, D)).astype(np.float16)
    k = Q.quantize_q8_0(rng.standard_normal((max(T, 1) * Hkv, D)).astype(np.float32))
    v = Q.quantize_q8_0(rng.standard_normal((max(T, 1) * Hkv, D)).astype(np.float32))
    return q, k, v, cu


RAGGED_CASES = [
    ([64, 8192, 1000, 3], 32, 8, 128),
    ([1, 2, 300, 257], 8, 8, 64),
    ([500, 0, 77], 16, 2, 128),        # an empty sequence
    ([4096] * 4, 32, 4, 128),
    # TMA fast path (Hkv = 8, D = 128): g = 4, 2, 1; empty and one-token sequences
    ([100, 33, 1, 0, 257], 32, 8, 128),
    ([7, 4097, 64], 16, 8, 128),
    ([31, 32, 33], 8, 8, 128),
    ([2000, 5], 32, 16, 128),
    # stream schedule: fewer tiles than CTAs, tile-boundary lengths, two and
    # four KV-head groups per token row, many sequences (ranges crossing items)
    ([1, 2, 3], 32, 8, 128),
    ([15, 16, 17, 0, 48, 1], 8, 8, 128),
    ([300, 700], 32, 32, 128),
    ([129, 4000, 64], 64, 16, 128),
    (list(np.random.default_rng(3).integers(0, 600, size=200)), 32, 8, 128),
]


@pytest.mark.parametrize("lens,Hq,Hkv,D", RAGGED_CASES)
def test_ragged_parity(cuda, lens, Hq, Hkv, D):
    import kq
    rng = np.random.default_rng(sum(lens) + Hq)
    q, k, v, cu = _ragged_case(rng, lens, Hq, Hkv, D)
    scale = 1.0 / np.sqrt(D)
    got = kq.flash_decode_ragged(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), Hkv, scale=scale)
    got = got.float().cpu().numpy()
    ref = Q.flash_decode_ragged(q, k, v, cu, Hq, Hkv, D, scale)
    ok, msg = Q.check_close(got, ref)
    assert ok, msg


def test_ragged_garbage_rows_masked(cuda):
    """Cache rows past the last sequence (total_rows > cu_seqlens[B]) hold
    arbitrary bytes, here NaN scales: a tile that reaches into them must mask
    them out (scores to -inf, p * d_v to zero), not propagate them."""
    import kq
    rng = np.random.default_rng(17)
    lens, Hq, Hkv, D = [37, 250, 9], 32, 8, 128
    q, k, v, cu = _ragged_case(rng, lens, Hq, Hkv, D)
    pad = np.full((40 * Hkv, D // 32, 34), 0xFF, dtype=np.uint8)  # fp16 0xFFFF = NaN, codes -1
    kp = np.concatenate([k.reshape(-1, D // 32, 34), pad]).reshape(-1)
    vp = np.concatenate([v.reshape(-1, D // 32, 34), pad]).reshape(-1)
    scale = 1.0 / np.sqrt(D)
    got = kq.flash_decode_ragged(_t(q, cuda), _t(kp, cuda), _t(vp, cuda), _t(cu, cuda), Hkv, scale=scale)
    ok, msg = Q.check_close(got.float().cpu().numpy(), Q.flash_decode_ragged(q, k, v, cu, Hq, Hkv, D, scale))
    assert ok, msg


def _seq_rows(x, cu, b, Hkv, D):
    """Cache bytes of sequence b alone (rows cu[b] .. cu[b+1] - 1)."""
    r = x.reshape(-1, Hkv, D // 32, 34)
    return np.ascontiguousarray(r[cu[b]:cu[b + 1]]).reshape(-1)


def test_full_size_config3_sampled_sequences(cuda):
    """configs[3] at full size: B = 32 sequences with lengths U[64, 8192]
    (seeded), Hq = 32, Hkv = 8, D = 128, fp16 queries and output. The whole
    batch runs in one call; the fp64 oracle checks the shortest, the longest
    and four more sequences (each sequence's output depends only on its own
    rows)."""
    import kq
    rng = np.random.default_rng(99)
    B, Hq, Hkv, D = 32, 32, 8, 128
    lens = rng.integers(64, 8193, size=B).astype(np.int32)
    cu = np.zeros(B + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    T = int(cu[-1])
    dev = cuda
    g = torch.Generator(device=dev).manual_seed(7)
    kd = kq.quantize_rows(torch.randn((T * Hkv, D), generator=g, device=dev), "q8_0")
    vd = kq.quantize_rows(torch.randn((T * Hkv, D), generator=g, device=dev), "q8_0")
    q = rng.standard_normal((B, Hq, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    got = kq.flash_decode_ragged(_t(q, dev), kd, vd, _t(cu, dev), Hkv, scale=scale).float().cpu().numpy()
    kh, vh = kd.cpu().numpy(), vd.cpu().numpy()
    pick = sorted({int(np.argmin(lens)), int(np.argmax(lens)), 0, 7, 19, B - 1})
    for b in pick:
        one = np.array([0, lens[b]], dtype=np.int32)
        ref = Q.flash_decode_ragged(q[b:b + 1], _seq_rows(kh, cu, b, Hkv, D), _seq_rows(vh, cu, b, Hkv, D), one,
                                    Hq, Hkv, D, scale)
        ok, msg = Q.check_close(got[b:b + 1], ref)
        assert ok, f"sequence {b} (L={lens[b]}): {msg}"


@pytest.mark.parametrize("path", ["tma", "generic"])
def test_earlier_decode_paths_opt_in(cuda, path):
    """KQ_FA_PATH=tma (the CUDA-core TMA decode) and =generic (the split-KV
    kernel) against the oracle on the ragged cases, in a child process (the
    path is chosen once per process)."""
    import os
    import subprocess
    import sys
    code = (
        "import sys; sys.path[:0] = %r\n"
        "import test_flash_decode_gpu as T, torch\n"
        "dev = torch.device('cuda:0')\n"
        "for fn in (T.test_ragged_parity, ):\n"
        "    for args in T.RAGGED_CASES:\n"
        "        fn(dev, *args)\n"
        "print('ok')\n" % ([os.path.dirname(os.path.abspath(__file__))] + [p for p in sys.path if p],))
    env = dict(os.environ, KQ_FA_PATH=path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("B,S,H", [(1, 8192, 32), (1, 512, 28), (2, 17, 32), (3, 16, 8), (4, 1, 32), (5, 300, 32),
                                   (8, 512, 32), (2, 8192, 32), (1, 1000, 2), (3, 777, 6)])
def test_small_batch_mha(cuda, B, S, H):
    """Harness batches too small to fill the GPU through the stream kernel
    (below 20 stream tiles per SM with one or two queries per head, below 4
    with more) run the small-batch kernel (fa_small.cu): one warp per
    (KV head, token chunk); every case here is below its bound. Covers one to five
    queries per head (a second query group at B = 5, 8), lengths at and
    around the 16-token tile, a one-token cache, and even head counts below 8
    that the stream kernel does not take."""
    import kq
    rng = np.random.default_rng(B * 7 + S + H)
    D = 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = Q.quantize_q8_0(rng.standard_normal((S * H, D)).astype(np.float32))
    v = Q.quantize_q8_0(rng.standard_normal((S * H, D)).astype(np.float32))
    got = kq.flash_attn_q8_0(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D))
    assert ok, msg
    assert kq.device_error() == 0


@pytest.mark.parametrize("lens,Hq,Hkv", [([8192], 32, 8), ([1], 32, 8), ([16], 8, 8), ([4097], 16, 8),
                                         ([300, 0], 32, 8), ([2000], 4, 2), ([33, 700], 8, 4)])
def test_small_batch_ragged(cuda, lens, Hq, Hkv):
    """Single sequences and small ragged batches (the common one-user decode
    step) on the small-batch kernel: g = 1, 2 and 4 queries per KV head, an
    empty sequence, one-token and tile-boundary lengths."""
    import kq
    rng = np.random.default_rng(sum(lens) + Hq + Hkv)
    D = 128
    q, k, v, cu = _ragged_case(rng, lens, Hq, Hkv, D)
    scale = 1.0 / np.sqrt(D)
    got = kq.flash_decode_ragged(_t(q, cuda), _t(k, cuda), _t(v, cuda), _t(cu, cuda), Hkv, scale=scale)
    ok, msg = Q.check_close(got.float().cpu().numpy(), Q.flash_decode_ragged(q, k, v, cu, Hq, Hkv, D, scale))
    assert ok, msg


@pytest.mark.parametrize("B,S,H", [(512, 64, 32), (300, 65, 32), (512, 1, 32), (1024, 100, 24), (512, 777, 28),
                                   (320, 2048, 32), (512, 3000, 28)])
def test_batch_mha(cuda, B, S, H):
    """Harness batches whose (64-query tile, head) CTAs fill the GPU run the
    tensor-core flash attention (fa_batch.cu). Partial query tiles (B = 300,
    320), lengths at and around the 64-token tile, a one-token cache, odd
    multiples of the head pair (H = 24, 28), and caches split into token
    chunks merged by the combine kernel (S = 2048 at B = 320: 3 chunks;
    S = 3000 at H = 28: 5 chunks, the last ending on a partial tile)."""
    import kq
    rng = np.random.default_rng(B + S + H)
    D = 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = Q.quantize_q8_0(rng.standard_normal((S * H, D)).astype(np.float32))
    v = Q.quantize_q8_0(rng.standard_normal((S * H, D)).astype(np.float32))
    got = kq.flash_attn_q8_0(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D))
    assert ok, msg
    assert Q.nmse(got, Q.flash_decode_mha(q, k, v, S, H, D)) < 0.05
    assert kq.device_error() == 0


@pytest.mark.parametrize("fmt", ["q4_0", "f16"])
@pytest.mark.parametrize("B,S,H", [(512, 64, 32), (300, 65, 32), (512, 1, 32), (1024, 100, 24), (512, 777, 28),
                                   (320, 2048, 32), (1920, 129, 5), (512, 3000, 28)])
def test_batch_mha_kv_formats(cuda, fmt, B, S, H):
    """Harness batches over q4_0 and fp16 caches run the batch kernel too
    (fa_batch.cu): q4_0 through the exact int8 QK on the nibble codes and the
    split V, fp16 with the split query over the cache read in place. Partial
    query tiles, lengths around the 64-token tile, a one-token cache, and for
    fp16 an odd head count (H = 5; the block formats need an even one)."""
    import kq
    if fmt == "q4_0" and H % 2:
        pytest.skip("block-quantised caches take the batch kernel with an even head count only")
    rng = np.random.default_rng(B + S + H + len(fmt))
    D = 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    v = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    got = kq.flash_attn(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D, fmt).cpu().numpy()
    ref = Q.flash_decode_mha(q, k, v, S, H, D, fmt)
    ok, msg = Q.check_close(got, ref)
    assert ok, msg
    assert kq.device_error() == 0


@pytest.mark.parametrize("fmt", ["q4_0", "f16"])
@pytest.mark.parametrize("B,S,H", [(1, 8192, 32), (8, 4096, 28), (3, 17, 32), (5, 1, 2), (2, 2049, 3), (4, 300, 7),
                                   (64, 1000, 8)])
def test_small_batch_kv_formats(cuda, fmt, B, S, H):
    """Harness batches too small for the batch kernel over q4_0 and fp16
    caches run the small-batch kernel (fa_small.cu): q4_0 nibbles as int8
    codes for the dp4a QK and decoded in PV, fp16 rows through 128-byte
    swizzled boxes with fp32 QK. One to four queries per group (and several
    groups), partial tiles, a one-token cache, odd head counts for fp16."""
    import kq
    if fmt == "q4_0" and H % 2:
        pytest.skip("block-quantised caches take the small-batch kernel with an even head count only")
    rng = np.random.default_rng(B * 7 + S + H + len(fmt))
    D = 128
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    v = _cache(fmt, rng.standard_normal((S, H, D)).astype(np.float32), D)
    got = kq.flash_attn(_t(q, cuda), _t(k, cuda), _t(v, cuda), B, S, H, D, fmt).cpu().numpy()
    ok, msg = Q.check_close(got, Q.flash_decode_mha(q, k, v, S, H, D, fmt))
    assert ok, msg
    assert kq.device_error() == 0


@pytest.mark.parametrize("lens,Hq,Hkv", [([8192], 32, 8), ([64] * 32 + [4096] * 8, 32, 8)])
def test_decode_after_producer(cuda, lens, Hq, Hkv):
    """The decode kernels are programmatic dependents of whatever precedes
    them: each call here directly follows torch's copy of fresh queries into
    the query buffer, and must see them (small-batch and stream kernels)."""
    import kq
    rng = np.random.default_rng(len(lens) + Hq)
    D = 128
    _, k, v, cu = _ragged_case(rng, lens, Hq, Hkv, D)
    kd, vd, cud = _t(k, cuda), _t(v, cuda), _t(cu, cuda)
    qd = torch.empty((len(lens), Hq, D), dtype=torch.float16, device=cuda)
    scale = 1.0 / np.sqrt(D)
    for it in range(3):
        q = (rng.standard_normal((len(lens), Hq, D)) * (1 + it)).astype(np.float16)
        qd.copy_(_t(q, cuda))
        got = kq.flash_decode_ragged(qd, kd, vd, cud, Hkv, scale=scale).float().cpu().numpy()
        ok, msg = Q.check_close(got, Q.flash_decode_ragged(q, k, v, cu, Hq, Hkv, D, scale))
        assert ok, f"iteration {it}: {msg}"
