"""The decode GEMV's launch plan (b200q_gemv_plan), checked on the host for a
sweep of formats, activation modes and shapes, without a GPU:

* every plan the kernel may be launched with fits the kernel's launch bounds
  and the shared memory of an SM, covers every row, and keeps the staged
  activations inside the ring above the slots filled before them;
* every Llama-3-8B / 70B shape of the benchmark configurations has a plan, in
  both activation modes, from codes and from fp32 x.
"""

from __future__ import annotations

import ctypes
import itertools

import pytest

FIELDS = ("threads", "smem", "grid", "S", "WR", "G", "SW", "R", "NS", "stage_stride", "PD", "x_off", "x_bytes",
          "row_bytes", "rows_cta")
BLOCK = {2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210), 112: (256, 144), 114: (256, 210), 214: (256, 276)}
BLOCKS_PER_SLICE = {2: 64, 8: 64, 12: 16, 14: 4, 112: 16, 114: 4, 214: 4}
SMS = 148


def _plan(lib, qt, act, k, n, mr, fq):
    out = (ctypes.c_longlong * len(FIELDS))()
    rc = lib.b200q_gemv_plan(qt, act, k, n, mr, fq, SMS, out, len(FIELDS))
    return rc, dict(zip(FIELDS, list(out)))


def _check(qt, act, k, n, mr, p):
    elems, nbytes = BLOCK[qt]
    nb = k // elems
    rb = nb * nbytes
    max_warps = 16 if (act == 1 and mr == 1) else 12
    assert p["row_bytes"] == rb
    assert p["S"] == -(-nb // BLOCKS_PER_SLICE[qt])
    assert p["G"] * p["SW"] == p["WR"] and p["S"] * p["WR"] <= max_warps
    assert p["threads"] == (p["S"] * p["WR"] + 1) * 32
    assert p["grid"] == min(SMS, -(-n // 4))
    assert p["rows_cta"] * p["grid"] >= n
    assert p["R"] >= 1 and (qt not in (112, 114) or p["R"] % 4 == 0)
    # a stage holds the 16-byte-aligned window around its rows plus the
    # 4-byte over-read of the unaligned word loads
    assert p["stage_stride"] % 128 == 0 and p["stage_stride"] >= p["R"] * rb + 34
    assert p["NS"] >= 2
    ring = p["NS"] * p["stage_stride"]
    assert p["smem"] >= ring and p["smem"] <= 220 * 1024
    # staged activations at the ring's end, above every slot filled before them
    assert p["x_off"] % 128 == 0 and p["x_off"] + p["x_bytes"] <= ring
    assert 0 <= p["PD"] <= p["x_off"] // p["stage_stride"]


@pytest.mark.parametrize("qt", sorted(BLOCK))
@pytest.mark.parametrize("act", [1, 2])
def test_plans_respect_kernel_limits(qt, act):
    from cybel_b200 import _native

    lib = _native.lib()
    elems = BLOCK[qt][0]
    ks = sorted({elems, 2 * elems, 4 * elems, 1024, 2304 if elems == 32 else 2048, 4096, 8192, 14336, 28672})
    ns = [1, 3, 7, 66, 1024, 4096, 14336, 128256]
    planned = 0
    for k, n, mr, fq in itertools.product(ks, ns, (1, 2), (0, 1)):
        if k % elems:
            continue
        rc, p = _plan(lib, qt, act, k, n, mr, fq)
        if rc == -3:  # no plan: only when the row needs more k-slices than the CTA has warps
            nb = k // elems
            assert -(-nb // BLOCKS_PER_SLICE[qt]) > (16 if (act == 1 and mr == 1) else 12) or k >= 14336, (k, n, mr)
            continue
        assert rc == 0, (qt, act, k, n, mr, fq, rc)
        _check(qt, act, k, n, mr, p)
        planned += 1
    assert planned > 0


@pytest.mark.parametrize("act", [1, 2])
@pytest.mark.parametrize("fq", [0, 1])
def test_benchmark_shapes_have_plans(act, fq):
    from cybel_b200 import _native

    lib = _native.lib()
    shapes = [(12, 4096, 4096), (12, 4096, 1024), (12, 4096, 14336), (12, 14336, 4096), (12, 4096, 6144),
              (12, 4096, 28672), (12, 8192, 8192), (12, 8192, 1024), (12, 8192, 57344), (12, 28672, 8192),
              (12, 8192, 128256), (14, 4096, 128256), (8, 4096, 4096), (8, 4096, 1024), (8, 4096, 14336),
              (8, 14336, 4096), (2, 4096, 4096)]
    for qt, k, n in shapes:
        rc, p = _plan(lib, qt, act, k, n, 1, fq)
        assert rc == 0, (qt, k, n, rc)
        _check(qt, act, k, n, 1, p)


def test_plan_rejects_bad_arguments():
    from cybel_b200 import _native

    lib = _native.lib()
    out = (ctypes.c_longlong * len(FIELDS))()
    assert lib.b200q_gemv_plan(12, 3, 4096, 4096, 1, 0, SMS, out, len(FIELDS)) == -1  # F16 is the tile path
    assert lib.b200q_gemv_plan(12, 1, 4096, 4096, 1, 0, SMS, out, 3) == -1             # short output
    assert lib.b200q_gemv_plan(12, 1, 100, 4096, 1, 0, SMS, out, len(FIELDS)) == -3    # k not whole blocks
    assert lib.b200q_gemv_plan(99, 1, 4096, 4096, 1, 0, SMS, out, len(FIELDS)) == -2   # unknown qtype
