"""Loader for libb200q.so (the sm_100a kernels behind the C ABI in
include/b200q.h).

There is no CPU fallback: if the library is missing or cannot be loaded,
``lib()`` raises. Build it with ``python -m cybel_b200.build``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libb200q.so"

ACT_X8 = 1
ACT_X16 = 2
ACT_F16 = 3  # tile path (tcgen05, fp16 operands), Q4_K, device entry points
WEIGHTS_STATIC = 1
TILE_FROM_2 = 2  # Q4_K batches of 2-7 rows on the tile kernel too

STATUS = {
    0: "ok",
    -1: "invalid argument",
    -2: "unsupported qtype",
    -3: "unsupported shape",
    -4: "pointer not 16-byte aligned",
    -5: "CUDA runtime error",
    -6: "device allocation failed",
    -7: "kernel pipeline wait timed out",
    -8: "no usable sm_100 device",
    -9: "scratch must grow during stream capture",
    -10: "request larger than the fixed no-alloc scratch",
    -11: "page table entry names no page or one outside the pool",
}

# Every symbol include/b200q.h declares: (name, argtypes, restype).
_vp = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_fp = ctypes.POINTER(ctypes.c_float)
SIGNATURES: dict[str, tuple[list, object]] = {}
for _q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q6k_lm", "q8_0", "q4_0"):
    SIGNATURES[f"simd_matvec_{_q}"] = ([_fp, _vp, _fp, _i, _i], None)
for _q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q8_0", "q4_0"):
    SIGNATURES[f"simd_matmul_{_q}"] = ([_fp, _vp, _fp, _i, _i, _i], None)
_ip = ctypes.POINTER(ctypes.c_int)
_vpp = ctypes.POINTER(ctypes.c_void_p)
_fpp = ctypes.POINTER(ctypes.POINTER(ctypes.c_float))
_f = ctypes.c_float
SIGNATURES.update(
    {
        "simd_repack_q4k_r4": ([_vp, _vp, _i, _i], _i),
        "simd_repack_q6k_r4": ([_vp, _vp, _i, _i], _i),
        "simd_repack_q6k_lm": ([_vp, _vp, _i, _i], _i),
        "simd_dequantize_row": ([_vp, _i, _i, _fp, _i], _i),
        "simd_fused_qkv_matvec_quant": ([_fp, _vp, _i, _fp, _i, _vp, _i, _fp, _i, _vp, _i, _fp, _i, _i], _i),
        "simd_fused_quad_matvec_quant": ([_fp, _vp, _i, _fp, _i, _vp, _i, _fp, _i, _vp, _i, _fp, _i, _vp, _i, _fp, _i, _i], _i),
        "simd_fused_expert_swiglu": ([_fp, _i, _vp, _i, _i, _vp, _i, _vp, _i, _i, _fp], None),
        "simd_fused_moe_ffn": ([_fp, _i, _ip, _fp, _i, _vpp, _i, _i, _vpp, _i, _vpp, _i, _i, _fp, _i], None),
        "b200q_repack": ([_i, _vp, _vp, _i, _i, _vp], _i),
        "b200q_dequantize_rows": ([_i, _vp, _vp, _i, _vp, _i, _i, _vp], _i),
        "b200q_fused_matvec": ([_i, _vp, _i, _i, _vpp, _ip, _vpp, _ip, _i, _vp], _i),
        "b200q_expert_swiglu": ([_i, _vp, _i, _vp, _i, _i, _vp, _i, _vp, _i, _i, _vp, _f, _f, _i, _vp], _i),
        "b200q_moe_ffn": ([_i, _vp, _i, _ip, _fp, _i, _vpp, _i, _i, _vpp, _i, _vpp, _i, _i, _vp, _i, _i, _vp], _i),
        "b200q_matmul": ([_i, _i, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
        "b200q_matmul_ex": ([_i, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp], _i),
        "b200q_matvec_isums": ([_i, _i, _vp, _vp, _vp, _vp, _i, _i, _vp], _i),
        "b200q_matvec_noalloc": ([_i, _i, _vp, _vp, _vp, _i, _i, _vp], _i),
        "b200q_matvec_quant": ([_vp, _i, _vp, _vp, _i, _i, _vp], _i),
        "b200q_matvec_dispatch": ([_vp, _vp, _i, _vp, _vp, _i, _i, _vp], _i),
        "b200q_add_rmsnorm": ([_vp, _vp, _vp, _vp, _i, _i, ctypes.c_float, _vp], _i),
        "b200q_rope_kv": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float, _vp, _vp, _i, _vp], _i),
        "b200q_attention_decode": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp], _i),
        "b200q_swiglu": ([_vp, _vp, _vp, ctypes.c_longlong, _vp], _i),
        "b200q_unshard_rows": ([_vp, _vp, _i, _i, _i, _vp], _i),
        "b200q_xq_row_bytes": ([_i, _i], ctypes.c_longlong),
        "b200q_add_rmsnorm_q": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, ctypes.c_float, _vp], _i),
        "b200q_attention_decode_q": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp], _i),
        "b200q_rope_attention_decode": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, _i, _vp, _vp, _i, _vp], _i),
        "b200q_rope_attention_decode_paged": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _vp, _vp, _vp, _i,
                                               _i, _vp, _i, _vp, _vp, _i, _ll, _ll, _vp], _i),
        "b200q_rope_attention_decode_tokens": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _i, _vp, _vp, _i,
                                                _ll, _ll, _vp], _i),
        "b200q_swiglu_q": ([_vp, _vp, _vp, _i, _i, _vp], _i),
        "b200q_swiglu_rows": ([_vp, _vp, _i, _i, _vp], _i),
        "b200q_matmul_xq": ([_i, _i, _vp, _vp, _vp, _i, _i, _i, ctypes.c_float, ctypes.c_float, _i, _vp], _i),
        "b200q_matmul_norm": ([_i, _i, _vp, _vp, _f, _vp, _vp, _i, _i, _f, _f, _i, _vp], _i),
        "b200q_matmul_swiglu": ([_i, _i, _vp, _vp, _vp, _vp, _i, _i, _f, _f, _i, _vp], _i),
        "b200q_gemv_plan": ([_i, _i, _i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_longlong), _i], _i),
        "b200q_ipc_alloc": ([ctypes.c_longlong, ctypes.POINTER(ctypes.c_void_p), _vp], _i),
        "b200q_ipc_open": ([_vp, ctypes.POINTER(ctypes.c_void_p)], _i),
        "b200q_ipc_close": ([_vp], _i),
        "b200q_ipc_free": ([_vp], _i),
        "b200q_allgather_peer": ([_vp, _i, _i, ctypes.POINTER(ctypes.c_void_p), ctypes.c_longlong, ctypes.c_longlong,
                                  _i, _i, _vp, _i, _vp, _i, _vp], _i),
        "b200q_quantize_rows": ([_i, _vp, _i, _i, _vp, _vp], _i),
        "b200q_set_act_mode": ([_i], _i),
        "b200q_get_act_mode": ([], _i),
        "b200q_last_error": ([], _i),
        "b200q_status_string": ([_i], ctypes.c_char_p),
        "b200q_device_status": ([_i], _i),
        "b200q_set_peer_wait_ns": ([ctypes.c_longlong], ctypes.c_longlong),
        "b200q_weight_cache_clear": ([], None),
        "b200q_weight_cache_evict": ([_vp], _i),
        "b200q_weight_cache_bytes": ([], ctypes.c_longlong),
        "b200q_set_pdl": ([_i], _i),
        "b200q_version": ([], ctypes.c_char_p),
    }
)

_LIB: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A libb200q entry point returned a non-zero status."""

    def __init__(self, status: int, what: str = ""):
        self.status = int(status)
        super().__init__(f"{what}: {STATUS.get(self.status, 'unknown status')} ({self.status})")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library with `python -m cybel_b200.build` "
                "(there is no CPU fallback)"
            )
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


def check(status: int, what: str) -> None:
    if int(status) != 0:
        raise NativeError(status, what)


STATUS_TIMEOUT = 1  # device status bit: a kernel's bounded wait gave up
STATUS_BAD_PAGE = 2  # device status bit: a paged cache's table named no page or one outside the pool
KV_F16, KV_Q8 = 0, 1  # paged KV storage modes


def check_device(device: int, what: str = "device status") -> None:
    """Raise NativeError(B200Q_ETIMEOUT) if a kernel on `device` recorded a
    wait that gave up since the last check, NativeError(B200Q_EPAGE) if a
    paged attention met a bad page-table entry (call after synchronizing the
    stream the work ran on); the status is cleared by the read."""
    v = int(lib().b200q_device_status(int(device)))
    if v < 0:
        raise NativeError(v, what)
    if v & STATUS_TIMEOUT:
        raise NativeError(-7, what)
    if v & STATUS_BAD_PAGE:
        raise NativeError(-11, what)
