"""The paged KV cache on the host: the Q8 row quantizer of the restatement
(oracle/paged_kv_ref.py) pinned by known answers of the reference's formula
(model_graph.cpp:1552-1572), the ANVIL_KV_QUANT switch
(model_graph.cpp:468-513), and PagedKVCache's page bookkeeping (lazy page
assignment, pool exhaustion, reset, snapshot / restore) with host pools."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.paged_kv_ref import PagedKVStoreRef, q8_row, q8_rows


def test_q8_known_answers():
    # amax 127 -> scale 1, inv 1: codes are std::round(x), half away from zero
    codes, scale = q8_row(np.array([127.0, -63.5, 0.5, -0.5, 2.4999, 1.5, -2.5, 0.0], np.float32))
    assert scale == np.float32(1.0)
    assert codes.tolist() == [127, -64, 1, -1, 2, 2, -3, 0]
    # an all-zero row: scale 1 / 127, codes 0
    codes, scale = q8_row(np.zeros(128, np.float32))
    assert scale == np.float32(1.0) / np.float32(127.0)
    assert not codes.any()
    # amax 254 -> scale 2: 3 * 0.5 = 1.5 -> 2, -1 * 0.5 -> -1 (half away), the max maps to 127
    codes, scale = q8_row(np.array([254.0, 3.0, -1.0, -254.0], np.float32))
    assert scale == np.float32(2.0)
    assert codes.tolist() == [127, 2, -1, -127]


def test_q8_scale_is_fp32_amax_over_127():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 128)).astype(np.float32)
    codes, scales = q8_rows(x)
    amax = np.abs(x).max(axis=1)
    assert np.array_equal(scales, (amax / np.float32(127.0)).astype(np.float32))
    assert np.abs(codes).max() == 127
    # reconstruction within half a step
    assert np.all(np.abs(codes * scales[:, None] - x) <= 0.5 * scales[:, None] * (1 + 1e-6))


def test_attention_restatement_masks_missing_pages():
    rng = np.random.default_rng(1)
    st = PagedKVStoreRef(layers=1, kv_heads=2, head_dim=8, max_seq=32, page_size=8, q8=False)
    for p in range(20):
        st.write(0, p, rng.standard_normal((2, 8)), rng.standard_normal((2, 8)))
    q = rng.standard_normal((4, 8))
    full = st.attention(0, q, 20)
    # exact softmax over the stored rows
    k = np.stack([st.pages[(0, p // 8)]["k"][p % 8] for p in range(20)]).astype(np.float64)
    v = np.stack([st.pages[(0, p // 8)]["v"][p % 8] for p in range(20)]).astype(np.float64)
    for h in range(4):
        s = k[:, h // 2] @ q[h] / np.sqrt(8)
        e = np.exp(s - s.max())
        assert np.allclose(full[h], e @ v[:, h // 2] / e.sum())
    st.drop_page(0, 1)  # positions 8..15 now have no page
    part = st.attention(0, q, 20)
    keep = [p for p in range(20) if not 8 <= p < 16]
    for h in range(4):
        s = k[keep, h // 2] @ q[h] / np.sqrt(8)
        e = np.exp(s - s.max())
        assert np.allclose(part[h], e @ v[keep, h // 2] / e.sum())


@pytest.mark.parametrize("val,want", [(None, False), ("", False), ("q8", True), ("1", True), ("on", True),
                                      ("yes", True), ("0", False), ("false", False), ("off", False)])
def test_kv_quant_switch(val, want):
    from cybel_b200.kv_cache import q8_from_env

    assert q8_from_env({} if val is None else {"ANVIL_KV_QUANT": val}) is want


def test_page_bookkeeping_on_host():
    from cybel_b200.kv_cache import PagedKVCache

    c = PagedKVCache(layers=2, kv_heads=1, max_seq=40, batch=2, page_size=16, q8=True, n_slots=9, device="cpu")
    assert c.pages_per_seq == 3 and c.pages_in_use == 0
    assert (c.table_host == -1).all()
    c.ensure(0)
    assert c.pages_in_use == 4 and (c.table_host[:, :, 0] >= 0).all() and (c.table_host[:, :, 1:] == -1).all()
    c.ensure(5)  # same page: nothing new
    assert c.pages_in_use == 4
    with pytest.raises(MemoryError):
        c.ensure(16, 33)  # pages 1 and 2: 8 more, 5 free
    assert c.pages_in_use == 4  # nothing assigned by the failed call
    c.reset()
    c.ensure(0, 31)
    assert c.pages_in_use == 8
    slots = c.table_host[c.table_host >= 0]
    assert len(set(slots.tolist())) == 8 and slots.max() < 9
    snap = c.snapshot()
    c.k[0].fill_(7)
    with pytest.raises(MemoryError):
        c.ensure(32)  # 4 more pages, 1 free
    c.restore(snap)
    assert int(c.k[0].abs().max()) == 0 and c.pages_in_use == 8
    assert np.array_equal(c.table.numpy(), c.table_host)
    free = [s for s in range(9) if s not in set(c.table_host[c.table_host >= 0].tolist())][0]
    c.assign(1, 0, 2, free)  # caller-chosen placement takes the slot off the free list
    c.sync_table()
    assert c.pages_in_use == 9 and int(c.table[1, 0, 2]) == free
    with pytest.raises(MemoryError):
        c.ensure(32)
    # Replacing a page: the old slot returns to the pool unless another
    # entry still uses it (a page shared between two sequences).
    shared = int(c.table_host[0, 0, 0])
    c.assign(0, 1, 0, shared)  # sequence 1's own page 0 is freed
    assert c.pages_in_use == 8
    old = int(c.table_host[0, 0, 1])
    c.assign(0, 0, 1, shared)
    assert c.pages_in_use == 7 and old not in set(c.table_host[c.table_host >= 0].tolist())
    c.assign(0, 0, 1, old)  # shared stays in use by (0, 0, 0) and (0, 1, 0)
    assert c.pages_in_use == 8 and int(c.table_host[0, 1, 0]) == shared
