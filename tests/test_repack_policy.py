"""The decode-layout policy on weight registration (repack_policy), restated
from the reference engine (model_graph_wrapper.py:684-842), checked on the
host: defaults per architecture, the ANVIL_* switches, and the byte budgets."""

from __future__ import annotations

from cybel_b200.formats import Q4_K, Q4_K_R4, Q6_K, Q6_K_LM, Q6_K_R4, Q8_0, row_bytes
from cybel_b200.repack_policy import MiB, RepackPolicy


def test_llama_defaults_pack_only_the_q6k_head():
    p = RepackPolicy.from_env("llama", env={})
    assert p.choose(Q4_K, 4096, 4096) == Q4_K
    assert p.choose(Q6_K, 4096, 128256, lm_head=True) == Q6_K_R4
    assert p.choose(Q4_K, 4096, 128256, lm_head=True) == Q4_K  # head Q4_K_R4 follows ANVIL_Q4K_R4
    assert p.choose(Q8_0, 4096, 4096) == Q8_0


def test_granitehybrid_defaults_pack_q4k():
    p = RepackPolicy.from_env("granitehybrid", env={})
    assert p.choose(Q4_K, 4096, 4096) == Q4_K_R4
    assert p.choose(Q4_K, 4096, 1000, lm_head=True) == Q4_K_R4


def test_switches():
    env = {"ANVIL_Q4K_R4": "1", "ANVIL_LM_HEAD_Q6K_LM": "yes", "ANVIL_LM_HEAD_Q4K_R4": "off"}
    p = RepackPolicy.from_env("llama", env=env)
    assert p.choose(Q4_K, 256, 8) == Q4_K_R4
    assert p.choose(Q6_K, 256, 8, lm_head=True) == Q6_K_LM
    # the head switch leaves a Q4_K head canonical, then the linear rule repacks it
    assert p.choose(Q4_K, 256, 8, lm_head=True) == Q4_K_R4
    for off in ("0", "false", "off", "no", "OFF"):
        q = RepackPolicy.from_env("granitehybrid", env={"ANVIL_Q4K_R4": off, "ANVIL_LM_HEAD_PACKED": off})
        assert q.choose(Q4_K, 256, 8) == Q4_K and q.choose(Q6_K, 256, 8, lm_head=True) == Q6_K
    assert RepackPolicy.canonical().choose(Q6_K, 256, 8, lm_head=True) == Q6_K


def test_budgets():
    k, n = 4096, 1024  # 2,359,296 bytes as Q4_K_R4
    size = n * row_bytes(Q4_K_R4, k)
    p = RepackPolicy.from_env("llama", env={"ANVIL_Q4K_R4": "1", "ANVIL_Q4K_R4_MAX_MB": "5"})
    assert p.choose(Q4_K, k, n) == Q4_K_R4  # 2.25 MiB used
    assert p.choose(Q4_K, k, n) == Q4_K_R4  # 4.5 MiB used
    assert p.choose(Q4_K, k, n) == Q4_K     # would exceed 5 MiB: canonical, nothing counted
    assert p.used["linear"] == 2 * size
    h = RepackPolicy.from_env("llama", env={"ANVIL_LM_HEAD_Q6K_LM": "1", "ANVIL_LM_HEAD_PACKED_MAX_MB": "1"})
    assert h.choose(Q6_K, 4096, 128256, lm_head=True) == Q6_K  # 141 MiB > 1 MiB
    assert h.used["head"] == 0
    assert RepackPolicy.from_env("llama", env={"ANVIL_Q4K_R4_MAX_MB": "x"}).q4k_r4_budget == 0
    assert MiB == 1 << 20
