"""CPU: the oracle's per-head QK-norm + partial split-half RoPE at the H3 attention layout
(56 heads x 128, rot_dim 96, eps 1e-5) against the reference's eager outputs
(``tests/golden/make_golden.py``, fixture ``qknorm_rope_h3``).

With the fp32 table the oracle equals comfy_kitchen's eager ``rms_rope_split_half`` bit for
bit. With the bf16 table the oracle (and the CUDA kernel) widen the table to fp32, as the
reference's CUDA kernel does (backends/cuda/ops/rms_rope.cu: ComputeType is float whenever
RMSNorm runs), while the eager and H3 CPU paths round every product to bf16; the two agree
within the north-star tolerance.
"""

import numpy as np

import oracle as O


def _rel(a, b):
    fa, fb = O.bf16_to_f32(a).astype(np.float64), O.bf16_to_f32(b).astype(np.float64)
    return np.linalg.norm(fa - fb) / np.linalg.norm(fb), float(np.abs(fa - fb).max())


def test_oracle_fp32_table_bit_exact(golden):
    g = golden("qknorm_rope_h3")
    qo, ko = O.rms_rope_split_half(g["q"], g["k"], g["table_f32"], g["wq"], g["wk"], 1e-5, 96)
    np.testing.assert_array_equal(qo, g["q_f32tab"])
    np.testing.assert_array_equal(ko, g["k_f32tab"])


def test_oracle_bf16_table_within_tolerance(golden):
    g = golden("qknorm_rope_h3")
    qo, ko = O.rms_rope_split_half(g["q"], g["k"], O.bf16_to_f32(g["table_bf16"]), g["wq"], g["wk"], 1e-5, 96)
    np.testing.assert_array_equal(g["q_bf16tab"], g["q_h3"])   # eager and H3 CPU paths agree
    for got, ref in ((qo, g["q_bf16tab"]), (ko, g["k_bf16tab"]), (qo, g["q_h3"]), (ko, g["k_h3"])):
        rel, mx = _rel(got, ref)
        assert rel <= 1e-2 and mx <= 2e-2
