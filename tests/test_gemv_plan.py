"""The decode GEMV's launch plan (b200q_gemv_plan), checked on the host for a
sweep of formats, activation modes and shapes, without a GPU:

* every plan the kernel may be launched with fits the kernel's launch bounds
  and the shared memory of an SM, covers every row, keeps the staged
  activation codes in bytes of their own past the ring, and has a ring whose
  slot count is a multiple of the walker groups;
* the planner refuses exactly the shapes its rule refuses;
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


def _rows_per_iter(qt, act, mr):
    """Rows a consumer warp carries per iteration (kRowsPerIter in gemv.cuh)."""
    return 2 if mr == 1 else 1


def _max_warps(act, mr, n=0):
    """Consumer warps the planner allows (kGemvWarps in gemv.cuh; x16 single
    rows take 14 for matrices of >= 8192 rows)."""
    if act == 1 and mr == 1:
        return 16
    return 14 if (act == 2 and mr == 1 and n >= 8192) else 12


def _check(qt, act, k, n, mr, p):
    elems, nbytes = BLOCK[qt]
    nb = k // elems
    rb = nb * nbytes
    assert p["row_bytes"] == rb
    assert p["S"] == -(-nb // BLOCKS_PER_SLICE[qt])
    assert p["G"] * p["SW"] == p["WR"] and p["S"] * p["WR"] <= _max_warps(act, mr, n)
    assert p["threads"] == (p["S"] * p["WR"] + 1) * 32  # consumer warps and the producer warp
    assert p["grid"] == min(SMS, -(-n // 4))
    assert p["rows_cta"] * p["grid"] >= n
    assert p["R"] >= 1 and (qt not in (112, 114) or p["R"] % 4 == 0)
    # a stage holds the 16-byte-aligned window around its rows plus the
    # 4-byte over-read of the unaligned word loads
    assert p["stage_stride"] % 128 == 0 and p["stage_stride"] >= p["R"] * rb + 34
    # stage s and s + NS belong to the same walker group
    assert p["NS"] >= 2 and p["NS"] % p["G"] == 0
    ring = p["NS"] * p["stage_stride"]
    # the staged activation codes have their own bytes past the ring
    assert p["x_off"] == ring
    kp = k + 16 * (-(-k // 256))
    assert p["x_bytes"] == mr * (-(-(act * kp + (k // 32) * 8) // 16) * 16)
    assert p["smem"] >= ring + p["x_bytes"] + p["NS"] * 16 and p["smem"] <= 220 * 1024
    assert 0 <= p["PD"] <= p["NS"]


def _max_rows(qt, act):
    """Activation rows one launch carries (max_rows_per_launch in gemv.cu)."""
    q4k = qt in (12, 112)
    if act == 1:
        return 2 if q4k else 4
    return 1 if q4k else 2


def _launch_rows(qt, act):
    return [mr for mr in (1, 2, 4) if mr <= _max_rows(qt, act)]


def _no_plan_expected(qt, act, k, n, mr, fq):
    """The planner's refusals (make_plan in gemv.cu), restated: more k-slices
    than the kernel has consumer warps, one row (one 4-row group for R4) over the
    largest stage (96 KB), fewer than two stages left in the shared-memory
    budget (220 KB) beside the staged activation codes, or (fq) fp32 rows
    larger than the ring they are first copied into."""
    elems, nbytes = BLOCK[qt]
    nb = k // elems
    rb = nb * nbytes
    S = -(-nb // BLOCKS_PER_SLICE[qt])
    if S > _max_warps(act, mr, n):
        return True
    r4 = qt in (112, 114)
    U = _rows_per_iter(qt, act, mr)
    n_quads = -(-n // 4)
    grid = min(SMS, n_quads)
    rows_cta = 4 * (-(-n_quads // grid))
    R = U * max(1, (48 * 1024 + U * rb // 2) // (U * rb))
    R = min(R, max(U, -(-rows_cta // U) * U))
    if r4:
        R = -(-R // 4) * 4
    if R * rb + 48 > 96 * 1024:
        R = 4 if r4 else max(1, (96 * 1024 - 48) // rb)
        if R * rb + 48 > 96 * 1024:
            return True
    stride = -(-(R * rb + 48) // 128) * 128
    kp = k + 16 * (-(-k // 256))
    x_bytes = mr * (-(-(act * kp + (k // 32) * 8) // 16) * 16)
    budget = (220 if k >= 8192 else 200) * 1024  # ring budget by row length
    room = budget - x_bytes - (48 * 16 + 20 + 16 * 4 + rows_cta * mr * S * 4 + 64)
    NS = min(48, room // stride if room > 0 else 0)
    if NS < 2:
        return True
    walkers = max(1, _max_warps(act, mr, n) // S)
    SW = max(1, min(walkers, -(-R // U)))
    if act == 1 and k >= 8192:  # x8, long rows: SW divides the walkers
        while SW > 1 and walkers % SW:
            SW -= 1
    G = min(max(1, walkers // SW), NS)
    NS -= NS % G
    nx = -(-(mr * k * 4) // stride) if fq else 0
    return nx > NS


@pytest.mark.parametrize("qt", sorted(BLOCK))
@pytest.mark.parametrize("act", [1, 2])
def test_plans_respect_kernel_limits(qt, act):
    from cybel_b200 import _native

    lib = _native.lib()
    elems = BLOCK[qt][0]
    ks = sorted({elems, 2 * elems, 4 * elems, 1024, 2304 if elems == 32 else 2048, 4096, 8192, 14336, 28672, 57344})
    ns = [1, 3, 7, 66, 1024, 4096, 14336, 128256]
    planned = refused = 0
    for k, n, mr, fq in itertools.product(ks, ns, _launch_rows(qt, act), (0, 1)):
        if k % elems:
            continue
        rc, p = _plan(lib, qt, act, k, n, mr, fq)
        if rc == -3:
            assert _no_plan_expected(qt, act, k, n, mr, fq), (k, n, mr, fq)
            refused += 1
            continue
        assert rc == 0, (qt, act, k, n, mr, fq, rc)
        assert not _no_plan_expected(qt, act, k, n, mr, fq), (k, n, mr, fq)
        _check(qt, act, k, n, mr, p)
        planned += 1
    assert planned > 0


@pytest.mark.parametrize("qt", sorted(BLOCK))
@pytest.mark.parametrize("act", [1, 2])
def test_plan_refuses_row_counts_never_launched(qt, act):
    from cybel_b200 import _native

    lib = _native.lib()
    k = BLOCK[qt][0] * 8
    for mr in (0, 3, 5):
        assert _plan(lib, qt, act, k, 64, mr, 0)[0] == -1
    for mr in (1, 2, 4):
        rc = _plan(lib, qt, act, k, 64, mr, 0)[0]
        assert rc == (0 if mr <= _max_rows(qt, act) else -1), (mr, rc)


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
