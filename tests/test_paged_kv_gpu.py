"""The paged KV attention (b200q_rope_attention_decode_paged) against the
restatement of the reference's PagedKVStore and its attention
(oracle/paged_kv_ref.py, model_graph.cpp:1413-1576, 1686-1930).

* Q8 pages, 150 consecutive decode steps of 2 sequences over 64-position
  pages (three pages, two page boundaries, up to three attention chunks):
  value codes and scales bit-exact against the restated quantizer at every
  position, key codes bit-exact at position 0 (rotation by angle 0) and
  within one code elsewhere (the device rotates in fp32); every step's
  output within max |d| / max |ref| <= 1e-4 of the restated attention over
  the rows the device stored (theta = 1, so rotation angles are exact
  integers and the fp32 rotation adds only rounding).
* fp16 pages with a permuted page table against the contiguous-cache kernel
  on the same rows, one token and three consecutive tokens per sequence:
  outputs, activation codes and the appended rows bit-identical.
* A page missing from the table and a slot past the pool: those positions
  are masked as the reference masks a position without a page (score -1e9,
  no value), the call records STATUS_BAD_PAGE (NativeError -11 from
  check_device), and the output matches the restatement with those pages
  dropped; a missing page at the appended position masks that position.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HD = 128


def _rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _st():
    import torch

    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("H,KV", [(32, 8), (64, 8), (8, 8)])
def test_q8_steps_against_restatement(H, KV):
    import torch

    from cybel_b200 import _native
    from cybel_b200.kv_cache import PagedKVCache
    from oracle.paged_kv_ref import PagedKVStoreRef, q8_rows, rope

    B, P, steps, theta = 2, 64, 150, 1.0
    cache = PagedKVCache(layers=1, kv_heads=KV, max_seq=256, batch=B, page_size=P, q8=True)
    rng = np.random.default_rng(H + KV)
    qs, ks, vs, outs = [], [], [], []
    out = torch.empty((B, H, HD), device="cuda")
    for pos in range(steps):
        q = rng.standard_normal((B, H, HD)).astype(np.float32)
        k = rng.standard_normal((B, KV, HD)).astype(np.float32)
        v = (rng.standard_normal((B, KV, HD)) * (0.0 if pos == 7 else 1.0)).astype(np.float32)  # one all-zero row
        qt, kt, vt = (torch.from_numpy(a).cuda() for a in (q, k, v))
        cache.ensure(pos)
        cache.attention(0, qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), pos, H, theta, out.data_ptr(), None, 0, _st())
        torch.cuda.synchronize()
        qs.append(q), ks.append(k), vs.append(v), outs.append(out.cpu().numpy())
    _native.check_device(0)
    assert cache.pages_in_use == B * 3
    for b in range(B):
        for h in range(KV):
            kc, vc, ksc, vsc = cache.rows(0, b, h, 0, steps)
            want_v, want_vs = q8_rows(np.stack([vs[p][b, h] for p in range(steps)]))
            assert np.array_equal(vc, want_v) and np.array_equal(vsc, want_vs)
            k_rot = np.stack([rope(ks[p][b, h], p, theta) for p in range(steps)]).astype(np.float32)
            want_k, want_ks = q8_rows(k_rot)
            assert np.array_equal(kc[0], want_k[0]) and ksc[0] == want_ks[0]
            d = np.abs(kc.astype(np.int32) - want_k.astype(np.int32))
            assert d.max() <= 1 and (d == 0).mean() >= 0.999
            assert np.allclose(ksc, want_ks, rtol=1e-5, atol=0)
    # attention of every step over the rows the device stored
    for b in range(B):
        ref = PagedKVStoreRef(1, KV, HD, 256, P, q8=True)
        rows = [cache.rows(0, b, h, 0, steps) for h in range(KV)]
        for p in range(steps):
            ref.set_row(0, p, np.stack([r[0][p] for r in rows]), np.stack([r[1][p] for r in rows]),
                        np.stack([r[2][p] for r in rows]), np.stack([r[3][p] for r in rows]))
        for pos in range(steps):
            want = ref.attention(0, rope(qs[pos][b], pos, theta), pos + 1)
            assert _rel(outs[pos][b], want) <= 1e-4, (b, pos)


@pytest.mark.parametrize("n_tok", [1, 3])
@pytest.mark.parametrize("H,KV,act", [(32, 8, 2), (64, 8, 1), (16, 16, 0)])
def test_f16_pages_match_contiguous_cache(H, KV, act, n_tok):
    import torch

    from cybel_b200 import _native
    from cybel_b200.kv_cache import PagedKVCache

    B, P, max_ctx, pos, theta = 2, 64, 320, 300, 500000.0
    L = _native.lib()
    rng = np.random.default_rng(7 + H)
    contig_k = torch.from_numpy(rng.standard_normal((B, KV, max_ctx, HD)).astype(np.float16)).cuda()
    contig_v = torch.from_numpy(rng.standard_normal((B, KV, max_ctx, HD)).astype(np.float16)).cuda()
    cache = PagedKVCache(layers=1, kv_heads=KV, max_seq=max_ctx, batch=B, page_size=P, q8=False)
    perm = rng.permutation(cache.n_slots)
    for b in range(B):
        for pg in range(cache.pages_per_seq):
            slot = int(perm[b * cache.pages_per_seq + pg])
            cache.assign(0, b, pg, slot)
            cache.k[slot] = contig_k[b, :, pg * P:(pg + 1) * P]
            cache.v[slot] = contig_v[b, :, pg * P:(pg + 1) * P]
    cache.sync_table()
    assert cache.pages_in_use == cache.n_slots
    q = torch.from_numpy(rng.standard_normal((B, n_tok, H, HD)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((B, n_tok, KV, HD)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((B, n_tok, KV, HD)).astype(np.float32)).cuda()
    xb = int(L.b200q_xq_row_bytes(H * HD, act)) if act else 16
    outs, xqs = [], []
    for paged in (False, True):
        out = torch.empty((B, n_tok, H, HD), device="cuda")
        xq = torch.zeros((B, n_tok, xb), dtype=torch.uint8, device="cuda")
        xp = xq.data_ptr() if act else None
        if paged:
            cache.attention(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos, H, theta, out.data_ptr(), xp, act, _st(),
                            n_tokens=n_tok)
        elif n_tok == 1:
            _native.check(L.b200q_rope_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, KV, HD, pos,
                                                        theta, contig_k.data_ptr(), contig_v.data_ptr(), max_ctx,
                                                        out.data_ptr(), xp, act, _st()), "contiguous")
        else:
            _native.check(L.b200q_rope_attention_decode_tokens(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, n_tok, H,
                                                               KV, HD, pos, theta, contig_k.data_ptr(),
                                                               contig_v.data_ptr(), max_ctx, out.data_ptr(), xp, act,
                                                               0, 0, _st()), "contiguous tokens")
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
        xqs.append(xq.cpu().numpy())
    _native.check_device(0)
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(xqs[0], xqs[1])
    for b in range(B):
        for h in range(KV):
            kc, vc, _, _ = cache.rows(0, b, h, pos, pos + n_tok)
            assert np.array_equal(kc, contig_k[b, h, pos:pos + n_tok].cpu().numpy())
            assert np.array_equal(vc, contig_v[b, h, pos:pos + n_tok].cpu().numpy())


def test_missing_and_bad_pages_are_masked_and_reported():
    import torch

    from cybel_b200 import _native
    from cybel_b200.kv_cache import PagedKVCache
    from oracle.paged_kv_ref import PagedKVStoreRef, rope

    B, H, KV, P, pos, theta = 3, 32, 8, 64, 200, 1.0
    cache = PagedKVCache(layers=1, kv_heads=KV, max_seq=256, batch=B, page_size=P, q8=True)
    cache.ensure(0, pos)
    g = torch.Generator(device="cuda").manual_seed(9)
    cache.k.copy_(torch.randint(-127, 128, cache.k.shape, generator=g, device="cuda", dtype=torch.int32))
    cache.v.copy_(torch.randint(-127, 128, cache.v.shape, generator=g, device="cuda", dtype=torch.int32))
    cache.ks.uniform_(0.001, 0.02, generator=g)
    cache.vs.uniform_(0.001, 0.02, generator=g)
    rows = [[cache.rows(0, b, h, 0, pos) for h in range(KV)] for b in range(B)]  # before the edits below
    cache.table_host[0, 0, 1] = -1                   # sequence 0: page 1 not allocated
    cache.table_host[0, 1, 2] = cache.n_slots + 5     # sequence 1: page 2 past the pool
    cache.table_host[0, 2, pos // P] = -1             # sequence 2: no page at pos
    cache.table.copy_(torch.from_numpy(cache.table_host))
    rng = np.random.default_rng(3)
    q = rng.standard_normal((B, H, HD)).astype(np.float32)
    k = rng.standard_normal((B, KV, HD)).astype(np.float32)
    v = rng.standard_normal((B, KV, HD)).astype(np.float32)
    qt, kt, vt = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty((B, H, HD), device="cuda")
    _native.check_device(0)  # clear
    cache.attention(0, qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), pos, H, theta, out.data_ptr(), None, 0, _st())
    torch.cuda.synchronize()
    with pytest.raises(_native.NativeError) as e:
        _native.check_device(0)
    assert e.value.status == -11
    got = out.cpu().numpy()
    dropped = {0: 1, 1: 2, 2: pos // P}  # sequence 2 loses the page holding pos, so 192..200
    for b in range(B):
        ref = PagedKVStoreRef(1, KV, HD, 256, P, q8=True)
        for p in range(pos):
            ref.set_row(0, p, np.stack([r[0][p] for r in rows[b]]), np.stack([r[1][p] for r in rows[b]]),
                        np.stack([r[2][p] for r in rows[b]]), np.stack([r[3][p] for r in rows[b]]))
        if b < 2:  # the appended row, read back from the device
            ap = [cache.rows(0, b, h, pos, pos + 1) for h in range(KV)]
            ref.set_row(0, pos, np.stack([a[0][0] for a in ap]), np.stack([a[1][0] for a in ap]),
                        np.stack([a[2][0] for a in ap]), np.stack([a[3][0] for a in ap]))
        ref.drop_page(0, dropped[b])
        want = ref.attention(0, rope(q[b], pos, theta), pos + 1)
        assert _rel(got[b], want) <= 1e-4, b


def test_paged_entry_rejects_bad_arguments():
    import torch

    from cybel_b200 import _native

    L = _native.lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    f = torch.zeros(1 << 14, device="cuda")
    tbl = torch.zeros(4, dtype=torch.int32, device="cuda")
    p, fp, tp = buf.data_ptr(), f.data_ptr(), tbl.data_ptr()
    st = _st()
    args = dict(q=fp, k=fp, v=fp, batch=1, H=8, KV=8, hd=HD, pos=10, theta=1e4, mode=_native.KV_Q8, kp=p, vp=p,
                ks=fp, vs=fp, n_slots=1, page=64, table=tp, pps=1, out=fp, xq=None, act=0, qs=0, kvs=0)

    def call(**over):
        a = dict(args, **over)
        return L.b200q_rope_attention_decode_paged(a["q"], a["k"], a["v"], a["batch"], 1, a["H"], a["KV"], a["hd"],
                                                   a["pos"], a["theta"], a["mode"], a["kp"], a["vp"], a["ks"],
                                                   a["vs"], a["n_slots"], a["page"], a["table"], a["pps"], a["out"],
                                                   a["xq"], a["act"], a["qs"], a["kvs"], st)

    assert call(ks=None) == -1           # Q8 without scales
    assert call(mode=5) == -1            # unknown storage mode
    assert call(table=None) == -1
    assert call(pos=64) == -3            # past pages_per_seq * page_size
    assert call(hd=64) == -3
    assert call(kp=p + 2) == -4          # pools 16-byte aligned
    assert call(qs=8 * HD - 4) == -3     # q rows overlapping
    assert call(kvs=8 * HD + 2) == -4    # k / v rows not 16-byte aligned
    assert call(mode=_native.KV_F16, ks=None, vs=None, kp=p + 4) == -4  # fp16 pools too
    torch.cuda.synchronize()


@pytest.mark.parametrize("pos0", [90, 62])
@pytest.mark.parametrize("n_tok", [3, 5])
def test_q8_multi_token_pages_not_aligned_to_chunks(n_tok, pos0):
    """Several tokens per sequence in one call over Q8 pages of 48 positions
    (pages and 64-position attention chunks cross each other; from pos0 = 62
    the call's tokens span one or two chunks): each token attends causally
    over the cache and the tokens before it; the rows the
    call appends are the restated quantizer's codes (values bit-exact) and
    every token's output matches the restated attention over the stored
    rows, within 1e-4 of max |ref|."""
    import torch

    from cybel_b200 import _native
    from cybel_b200.kv_cache import PagedKVCache
    from oracle.paged_kv_ref import PagedKVStoreRef, q8_rows, rope

    B, H, KV, P, theta = 2, 16, 4, 48, 1.0
    # pos0 = 90: the call covers pages 1 and 2 inside chunk 1; pos0 = 62: its
    # tokens straddle the first 64-position chunk boundary (1 or 2 chunks each)
    cache = PagedKVCache(layers=1, kv_heads=KV, max_seq=192, batch=B, page_size=P, q8=True)
    rng = np.random.default_rng(40 + n_tok)
    out1 = torch.empty((B, H, HD), device="cuda")
    for pos in range(pos0):  # single-token steps fill the cache
        q = torch.from_numpy(rng.standard_normal((B, H, HD)).astype(np.float32)).cuda()
        k = torch.from_numpy(rng.standard_normal((B, KV, HD)).astype(np.float32)).cuda()
        v = torch.from_numpy(rng.standard_normal((B, KV, HD)).astype(np.float32)).cuda()
        cache.ensure(pos)
        cache.attention(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos, H, theta, out1.data_ptr(), None, 0, _st())
    q = rng.standard_normal((B, n_tok, H, HD)).astype(np.float32)
    k = rng.standard_normal((B, n_tok, KV, HD)).astype(np.float32)
    v = rng.standard_normal((B, n_tok, KV, HD)).astype(np.float32)
    qt, kt, vt = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty((B, n_tok, H, HD), device="cuda")
    cache.ensure(pos0, pos0 + n_tok - 1)
    cache.attention(0, qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), pos0, H, theta, out.data_ptr(), None, 0, _st(),
                    n_tokens=n_tok)
    torch.cuda.synchronize()
    _native.check_device(0)
    got = out.cpu().numpy()
    last = pos0 + n_tok
    for b in range(B):
        rows = [cache.rows(0, b, h, 0, last) for h in range(KV)]
        for h in range(KV):
            want_v, want_vs = q8_rows(v[b, :, h])
            assert np.array_equal(rows[h][1][pos0:], want_v) and np.array_equal(rows[h][3][pos0:], want_vs)
        ref = PagedKVStoreRef(1, KV, HD, 192, P, q8=True)
        for p in range(last):
            ref.set_row(0, p, np.stack([r[0][p] for r in rows]), np.stack([r[1][p] for r in rows]),
                        np.stack([r[2][p] for r in rows]), np.stack([r[3][p] for r in rows]))
        for t in range(n_tok):
            want = ref.attention(0, rope(q[b, t], pos0 + t, theta), pos0 + t + 1)
            assert _rel(got[b, t], want) <= 1e-4, (b, t)
