"""GPU parity of the decode step's attention kernels through the C ABI
(draco_rope_kv_append, draco_attention_cached).

* RoPE + cache append: bit-exact against the oracle's apply_rope
  (draco/runtime/cpu/ops.py:86-95 restated), the value rows copied unchanged;
* cached attention: within 1e-5 relative L2 of a float64 softmax(q K^T /
  sqrt(d)) V (the reference computes the scores in float64,
  draco/runtime/cpu/attention.py), per token, across 32-key chunk edges,
  with grouped-query heads and tokens outside the cache (zero output);
* the one-launch decode form (draco_attention_decode): bit-identical outputs
  and caches to RoPE + append followed by the cached attention, q untouched,
  the workspace's status word and counters left at zero.
"""

import numpy as np
import pytest

from oracle import llama_decode as D

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from dracort_b200 import _native as N  # noqa: E402
from dracort_b200.gguf_executor import rope_tables  # noqa: E402

ATTN_TOL = 1e-5


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def O_rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def _attention_ref(q, kc, vc, seq, pos):
    """float64 attention of each token over its slot's keys 0..pos."""
    n, heads, hd = q.shape
    kvh = kc.shape[1]
    out = np.zeros((n, heads, hd))
    for i in range(n):
        if pos[i] < 0 or pos[i] >= kc.shape[2]:
            continue
        for h in range(heads):
            K = kc[seq[i], h // (heads // kvh), :pos[i] + 1].astype(np.float64)
            V = vc[seq[i], h // (heads // kvh), :pos[i] + 1].astype(np.float64)
            s = K @ q[i, h].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[i, h] = (p / p.sum()) @ V
    return out


@pytest.mark.parametrize("heads,kv_heads,hd", [(8, 4, 32), (32, 32, 128), (4, 1, 64)])
def test_rope_kv_append_is_bit_exact(heads, kv_heads, hd):
    rng = np.random.default_rng(hd + heads)
    n, cap, slots = 5, 80, 3
    q = rng.standard_normal((n, heads, hd)).astype(np.float32)
    k = rng.standard_normal((n, kv_heads, hd)).astype(np.float32)
    v = rng.standard_normal((n, kv_heads, hd)).astype(np.float32)
    seq = np.array([0, 2, 1, 2, 0], dtype=np.int32)
    pos = np.array([0, 7, 31, 32, 79], dtype=np.int32)
    cos, sin = rope_tables(hd, cap, 10000.0)
    qd, kd, vd = _cuda(q), _cuda(k), _cuda(v)
    kc = torch.zeros((slots, kv_heads, cap, hd), device="cuda")
    vc = torch.zeros_like(kc)
    cd, sd, seqd, posd = _cuda(cos), _cuda(sin), _cuda(seq), _cuda(pos)
    lib = N.load()
    rc = lib.draco_rope_kv_append(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                  cd.data_ptr(), sd.data_ptr(), seqd.data_ptr(), posd.data_ptr(), n, heads, kv_heads,
                                  hd, cap, slots, None)
    assert rc == 0, N.last_error()
    torch.cuda.synchronize()
    ocos, osin = D.build_rope_cache(hd, cap, 10000.0)
    q_ref = D.apply_rope(q, ocos, osin, pos)
    k_ref = D.apply_rope(k, ocos, osin, pos)
    assert np.array_equal(qd.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))
    kc_h, vc_h = kc.cpu().numpy(), vc.cpu().numpy()
    for i in range(n):
        assert np.array_equal(kc_h[seq[i], :, pos[i]].view(np.uint32), k_ref[i].view(np.uint32))
        assert np.array_equal(vc_h[seq[i], :, pos[i]], v[i])


def _run_attention(q, kc, vc, seq, pos, max_pos, ws_bytes=None):
    n, heads, hd = q.shape
    slots, kvh, cap, _ = kc.shape
    lib = N.load()
    need = lib.draco_attention_workspace_bytes(n, heads, hd, max_pos)
    ws = torch.zeros(max(int(ws_bytes if ws_bytes is not None else need), 16), dtype=torch.uint8, device="cuda")
    qd, kd, vd, seqd, posd = _cuda(q), _cuda(kc), _cuda(vc), _cuda(seq), _cuda(pos)
    out = torch.full((n, heads, hd), float("nan"), device="cuda")
    rc = lib.draco_attention_cached(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), seqd.data_ptr(), posd.data_ptr(),
                                    max_pos, out.data_ptr(), n, heads, kvh, hd, cap, slots, ws.data_ptr(),
                                    ws_bytes if ws_bytes is not None else ws.numel(), None)
    return rc, out


@pytest.mark.parametrize("heads,kv_heads,hd", [(8, 4, 32), (32, 32, 128), (4, 1, 64), (2, 2, 256)])
def test_attention_cached_matches_float64(heads, kv_heads, hd):
    rng = np.random.default_rng(7 * hd + heads)
    slots, cap = 3, 1100
    kc = rng.standard_normal((slots, kv_heads, cap, hd)).astype(np.float32)
    vc = rng.standard_normal((slots, kv_heads, cap, hd)).astype(np.float32)
    # positions on both sides of the 32-key chunk edges, one past the last full chunk
    pos = np.array([0, 1, 30, 31, 32, 33, 63, 64, 500, 1023, 1024, 1099], dtype=np.int32)
    seq = (np.arange(len(pos)) % slots).astype(np.int32)
    q = (rng.standard_normal((len(pos), heads, hd)) * 2).astype(np.float32)
    rc, out = _run_attention(q, kc, vc, seq, pos, cap - 1)
    assert rc == 0, N.last_error()
    ref = _attention_ref(q, kc, vc, seq, pos)
    got = out.cpu().numpy()
    for i in range(len(pos)):
        assert O_rel(got[i], ref[i]) < ATTN_TOL, i


def test_attention_bound_and_tokens_outside_the_cache():
    rng = np.random.default_rng(3)
    slots, kvh, cap, hd, heads = 2, 2, 128, 64, 4
    kc = rng.standard_normal((slots, kvh, cap, hd)).astype(np.float32)
    vc = rng.standard_normal((slots, kvh, cap, hd)).astype(np.float32)
    q = rng.standard_normal((5, heads, hd)).astype(np.float32)
    # max_pos 63: position 64 and above count as outside, as do a bad slot and a negative position
    pos = np.array([10, 63, 64, 5, -1], dtype=np.int32)
    seq = np.array([0, 1, 0, 7, 1], dtype=np.int32)
    rc, out = _run_attention(q, kc, vc, seq, pos, 63)
    assert rc == 0, N.last_error()
    got = out.cpu().numpy()
    ref = _attention_ref(q[:2], kc, vc, seq[:2], pos[:2])
    assert O_rel(got[:2], ref) < ATTN_TOL
    assert np.all(got[2:] == 0.0)


def test_attention_argument_errors():
    q = np.zeros((2, 4, 64), dtype=np.float32)
    kc = np.zeros((1, 2, 96, 64), dtype=np.float32)
    seq = np.zeros(2, dtype=np.int32)
    pos = np.array([3, 4], dtype=np.int32)
    lib = N.load()
    need = lib.draco_attention_workspace_bytes(2, 4, 64, 95)
    # status word, 8 counters, 96 positions = three 32-key chunk records of hd + 4 floats
    assert need == 16 + 32 + 2 * 4 * 3 * (64 + 4) * 4
    rc, _ = _run_attention(q, kc, kc, seq, pos, 95, ws_bytes=need - 4)
    assert rc == N.DRACO_ERR_WORKSPACE and "workspace" in N.last_error()
    rc, _ = _run_attention(q, kc, kc, seq, pos, 96)  # max_pos beyond the capacity
    assert rc == N.DRACO_ERR_SHAPE
    assert lib.draco_attention_workspace_bytes(2, 4, 64, -1) == 0
    q6 = np.zeros((2, 4, 6), dtype=np.float32)
    kc6 = np.zeros((1, 2, 96, 6), dtype=np.float32)
    rc, _ = _run_attention(q6, kc6, kc6, seq, pos, 95)  # head_dim not a multiple of 4
    assert rc == N.DRACO_ERR_SHAPE and "head_dim" in N.last_error()


def _workspace(n, heads, hd, max_pos):
    need = N.load().draco_attention_workspace_bytes(n, heads, hd, max_pos)
    return torch.zeros(int(need), dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("heads,kv_heads,hd", [(8, 4, 32), (32, 32, 128), (4, 1, 64), (2, 2, 256)])
def test_decode_form_equals_rope_then_cached_attention(heads, kv_heads, hd):
    rng = np.random.default_rng(11 * hd + heads)
    slots, cap = 9, 1100
    # one token per slot, positions on both sides of the chunk edges (0 = an empty history)
    pos = np.array([0, 5, 31, 32, 33, 64, 1023, 1024, 1099], dtype=np.int32)
    seq = np.array([3, 0, 8, 1, 7, 2, 6, 4, 5], dtype=np.int32)
    n = len(pos)
    kc0 = torch.from_numpy(rng.standard_normal((slots, kv_heads, cap, hd)).astype(np.float32)).cuda()
    vc0 = torch.from_numpy(rng.standard_normal((slots, kv_heads, cap, hd)).astype(np.float32)).cuda()
    q = torch.from_numpy(rng.standard_normal((n, heads, hd)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((n, kv_heads, hd)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((n, kv_heads, hd)).astype(np.float32)).cuda()
    cos, sin = (_cuda(t) for t in rope_tables(hd, cap, 10000.0))
    seqd, posd = _cuda(seq), _cuda(pos)
    lib = N.load()
    out = []
    caches = []
    for form in ("two_call", "decode"):
        kc, vc, qq = kc0.clone(), vc0.clone(), q.clone()
        ws = _workspace(n, heads, hd, cap - 1)
        o = torch.full((n, heads, hd), float("nan"), device="cuda")
        if form == "decode":
            rc = lib.draco_attention_decode(qq.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            cos.data_ptr(), sin.data_ptr(), seqd.data_ptr(), posd.data_ptr(), cap - 1,
                                            o.data_ptr(), n, heads, kv_heads, hd, cap, slots, ws.data_ptr(),
                                            ws.numel(), None)
            assert rc == 0, N.last_error()
            assert torch.equal(qq, q)  # q is rotated in shared memory only
        else:
            rc = lib.draco_rope_kv_append(qq.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                          cos.data_ptr(), sin.data_ptr(), seqd.data_ptr(), posd.data_ptr(), n, heads,
                                          kv_heads, hd, cap, slots, None)
            assert rc == 0, N.last_error()
            rc = lib.draco_attention_cached(qq.data_ptr(), kc.data_ptr(), vc.data_ptr(), seqd.data_ptr(),
                                            posd.data_ptr(), cap - 1, o.data_ptr(), n, heads, kv_heads, hd, cap,
                                            slots, ws.data_ptr(), ws.numel(), None)
            assert rc == 0, N.last_error()
        torch.cuda.synchronize()
        assert int(ws[:16 + 4 * n * heads].count_nonzero()) == 0  # status and counters back at zero
        out.append(o)
        caches.append((kc, vc))
    assert torch.equal(out[0], out[1])
    assert torch.equal(caches[0][0], caches[1][0]) and torch.equal(caches[0][1], caches[1][1])
    ref = _attention_ref(D.apply_rope(q.cpu().numpy(), *D.build_rope_cache(hd, cap, 10000.0), pos),
                         caches[1][0].cpu().numpy(), caches[1][1].cpu().numpy(), seq, pos)
    got = out[1].cpu().numpy()
    for i in range(n):
        assert O_rel(got[i], ref[i]) < ATTN_TOL, i


def test_decode_form_is_repeatable_on_one_workspace():
    """The merge counters reset themselves: ten launches on one workspace give
    the same bits."""
    rng = np.random.default_rng(5)
    slots, kvh, heads, hd, cap = 4, 4, 8, 128, 300
    kc = torch.from_numpy(rng.standard_normal((slots, kvh, cap, hd)).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.standard_normal((slots, kvh, cap, hd)).astype(np.float32)).cuda()
    q, k, v = (torch.from_numpy(rng.standard_normal((4, h, hd)).astype(np.float32)).cuda() for h in (heads, kvh, kvh))
    cos, sin = (_cuda(t) for t in rope_tables(hd, cap, 10000.0))
    seqd, posd = _cuda(np.arange(4, dtype=np.int32)), _cuda(np.array([299, 100, 40, 7], dtype=np.int32))
    ws = _workspace(4, heads, hd, cap - 1)
    lib = N.load()
    outs = []
    for _ in range(10):
        o = torch.empty((4, heads, hd), device="cuda")
        rc = lib.draco_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                        cos.data_ptr(), sin.data_ptr(), seqd.data_ptr(), posd.data_ptr(), cap - 1,
                                        o.data_ptr(), 4, heads, kvh, hd, cap, slots, ws.data_ptr(), ws.numel(), None)
        assert rc == 0, N.last_error()
        outs.append(o)
    torch.cuda.synchronize()
    assert all(torch.equal(o, outs[0]) for o in outs)
    assert int(ws[:16 + 4 * 4 * heads].count_nonzero()) == 0
