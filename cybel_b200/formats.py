"""GGUF block formats consumed by the B200 kernels.

Type ids and block specs follow the engine's wrapper
(core/native/quantized_matmul_wrapper.py:28-42; quantized_matmul.cpp:39-44);
Q4_0 is ggml's type 2 (32 elements, fp16 scale + 16 nibble bytes), which the
reference does not implement.
"""

from __future__ import annotations

Q4_0 = 2
Q8_0 = 8
Q4_K = 12
Q6_K = 14
Q4_K_R4 = 112  # 4-row block-major regrouping of Q4_K (quantized_matmul.cpp:250-300)
Q6_K_R4 = 114  # 4-row block-major regrouping of Q6_K
Q6_K_LM = 214  # Q6_K expanded to int8 codes + int8 scales + fp32 d (quantized_matmul.cpp:302-365)

BLOCK_SPECS: dict[int, tuple[int, int]] = {
    Q4_0: (32, 18),
    Q8_0: (32, 34),
    Q4_K: (256, 144),
    Q6_K: (256, 210),
    Q4_K_R4: (256, 144),
    Q6_K_R4: (256, 210),
    Q6_K_LM: (256, 276),
}

QTYPE_NAMES = {
    Q4_0: "q4_0",
    Q8_0: "q8_0",
    Q4_K: "q4k",
    Q6_K: "q6k",
    Q4_K_R4: "q4k_r4",
    Q6_K_R4: "q6k_r4",
    Q6_K_LM: "q6k_lm",
}


def row_bytes(qtype: int, k: int) -> int:
    elems, nbytes = BLOCK_SPECS[qtype]
    if k % elems:
        raise ValueError(f"k={k} is not a multiple of the qtype {qtype} block ({elems})")
    return (k // elems) * nbytes


def weight_bytes(qtype: int, k: int, n: int) -> int:
    return row_bytes(qtype, k) * n
