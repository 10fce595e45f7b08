"""Which decode layout each weight gets when a stack is registered.

The reference engine decides, as it hands each quantized weight to its graph
(JSBuild/src/verso/Anvil/core/native/model_graph_wrapper.py:684-842,
``_get_quant_info``), whether to keep the canonical GGUF rows or to repack
them into a decode layout: Q4_K rows into the 4-row interleaved Q4_K_R4
layout, and the LM head (Q6_K) into Q6_K_R4 or the expanded Q6_K_LM layout
-- each under an optional byte budget. This module restates that policy with
the same environment switches, so a deployment configured for the reference
gets the same layouts here; the repacks themselves run on the device
(b200q_repack), and every layout has its own GEMV instance.

Switches (unset = the reference's default):

=============================  =========================================
ANVIL_Q4K_R4                   Q4_K linears -> Q4_K_R4 (default: only for
                               the granitehybrid architecture)
ANVIL_Q4K_R4_MAX_MB            byte budget of those repacks (0: none)
ANVIL_LM_HEAD_PACKED           repack the LM head (default on)
ANVIL_LM_HEAD_PACKED_MAX_MB    byte budget of the head repack (0: none)
ANVIL_LM_HEAD_Q4K_R4           a Q4_K head -> Q4_K_R4 (default: ANVIL_Q4K_R4)
ANVIL_LM_HEAD_Q6K_LM           a Q6_K head -> Q6_K_LM instead of Q6_K_R4
                               (default off)
=============================  =========================================

A value of 0 / false / off / no disables a switch; any other value enables it.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Mapping

from .formats import Q4_K, Q4_K_R4, Q6_K, Q6_K_LM, Q6_K_R4, row_bytes

_OFF = {"0", "false", "off", "no"}
MiB = 1024 * 1024


def _flag(env: Mapping[str, str], name: str, default: bool) -> bool:
    v = env.get(name)
    if v is None:
        return default
    return v.strip().lower() not in _OFF


def _budget(env: Mapping[str, str], name: str) -> int:
    v = env.get(name)
    if v is None:
        return 0
    try:
        return max(0, int(v or "0")) * MiB
    except ValueError:
        return 0


@dataclass
class RepackPolicy:
    q4k_r4: bool = False
    q4k_r4_budget: int = 0          # bytes; 0 = no limit
    lm_head_packed: bool = True
    lm_head_budget: int = 0         # bytes; 0 = no limit
    lm_head_q4k_r4: bool = False
    lm_head_q6k_lm: bool = False
    used: dict = field(default_factory=lambda: {"linear": 0, "head": 0})

    @classmethod
    def from_env(cls, architecture: str = "llama", env: Mapping[str, str] | None = None) -> "RepackPolicy":
        """The policy the reference derives from its environment
        (model_graph_wrapper.py:684-740) for a model of `architecture`."""
        env = os.environ if env is None else env
        q4k_r4 = _flag(env, "ANVIL_Q4K_R4", str(architecture) == "granitehybrid")
        return cls(
            q4k_r4=q4k_r4,
            q4k_r4_budget=_budget(env, "ANVIL_Q4K_R4_MAX_MB"),
            lm_head_packed=_flag(env, "ANVIL_LM_HEAD_PACKED", True),
            lm_head_budget=_budget(env, "ANVIL_LM_HEAD_PACKED_MAX_MB"),
            lm_head_q4k_r4=_flag(env, "ANVIL_LM_HEAD_Q4K_R4", q4k_r4),
            lm_head_q6k_lm=_flag(env, "ANVIL_LM_HEAD_Q6K_LM", False),
        )

    @classmethod
    def canonical(cls) -> "RepackPolicy":
        """Every weight keeps its canonical GGUF rows."""
        return cls(q4k_r4=False, lm_head_packed=False)

    def choose(self, qtype: int, k: int, n: int, lm_head: bool = False) -> int:
        """The layout (qtype) a weight of `qtype` with n rows of k gets, and the
        budget it consumes (model_graph_wrapper.py:796-842): the LM head first
        by the head switches (falling through to the linear rule when they
        leave it canonical), every Q4_K weight by ANVIL_Q4K_R4; a repack that
        would overrun its budget leaves the weight canonical."""
        if lm_head and self.lm_head_packed:
            target = qtype
            if qtype == Q6_K:
                target = Q6_K_LM if self.lm_head_q6k_lm else Q6_K_R4
            elif qtype == Q4_K and self.lm_head_q4k_r4:
                target = Q4_K_R4
            if target != qtype:
                nbytes = n * row_bytes(target, k)
                if self.lm_head_budget > 0 and self.used["head"] + nbytes > self.lm_head_budget:
                    return qtype
                self.used["head"] += nbytes
                return target
        if self.q4k_r4 and qtype == Q4_K:
            nbytes = n * row_bytes(Q4_K_R4, k)
            if self.q4k_r4_budget > 0 and self.used["linear"] + nbytes > self.q4k_r4_budget:
                return qtype
            self.used["linear"] += nbytes
            return Q4_K_R4
        return qtype


def apply(policy: RepackPolicy | None, matrix, lm_head: bool = False):
    """The device matrix in the layout the policy picks for it (a new
    DeviceMatrix repacked on the device by b200q_repack, or `matrix` itself)."""
    import torch

    from . import _native
    from .quantized_matmul import DeviceMatrix

    if policy is None:
        return matrix
    target = policy.choose(matrix.qtype, matrix.input_dim, matrix.output_dim, lm_head=lm_head)
    if target == matrix.qtype:
        return matrix
    k, n = matrix.input_dim, matrix.output_dim
    dst = torch.empty(n * row_bytes(target, k), dtype=torch.uint8, device=matrix.buffer.device)
    st = torch.cuda.current_stream(matrix.buffer.device).cuda_stream
    _native.check(_native.lib().b200q_repack(target, matrix.ptr, dst.data_ptr(), k, n, st), "repack")
    return DeviceMatrix(target, k, n, dst, name=matrix.name)
