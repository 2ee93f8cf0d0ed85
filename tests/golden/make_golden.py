"""Writes tests/golden/known_answers.json: the known-answer vectors of the
reference's own kernel tests, transcribed from its test sources.

The reference is Java and cannot run here, so its test inputs and expected
values are restated literally; expected values that the Java tests compute
with an expression are evaluated with the same binary32 semantics
(numpy.float32 for every float operation, (float)Math.f(double) as
float32(math.f(x))).  Citations are paths inside the reference project under
src/test/java/com/arturskowronski/llama3babylon/hat/.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os

import numpy as np

f32 = np.float32
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")


def fl(v) -> float:
    return float(f32(v))


def java_silu(x: np.float32) -> np.float32:
    # SiLU.java:38 / SiLUHatVsJavaTest.java:36-41: x / (1.0f + (float) Math.exp(-x))
    return f32(x / (f32(1.0) + f32(math.exp(float(-x)))))


def ramp(size: int, start: float) -> list[float]:
    # SiLUHatVsJavaTest.java:44-50: startVal + i * 0.01f (float ops)
    return [fl(f32(start) + f32(i) * f32(0.01)) for i in range(size)]


def cases() -> list[dict]:
    c = []
    c.append(dict(id="gemv_f32_4x3", kernel="gemv_f32", source="kernels/GEMVTest.java:18-52",
                  rows=4, cols=3, matrix=[float(i + 1) for i in range(12)], vector=[1.0, 1.0, 1.0],
                  expected=[6.0, 15.0, 24.0, 33.0], tol=1e-5))
    c.append(dict(id="gemv_f16_2x4", kernel="gemv_f16", source="kernels/F16ToFloatOpenCLCodegenTest.java:102-111,136-137",
                  rows=2, cols=4, matrix=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0], vector=[1.0] * 4,
                  expected=[10.0, 26.0], tol=0.01))
    c.append(dict(id="rmsnorm_simple", kernel="rmsnorm", source="kernels/RMSNormTest.java:24-50",
                  input=[1.0, 2.0, 3.0, 4.0], weight=[1.0] * 4,
                  property="mean_of_squares", expected_mean_of_squares=1.0, tol=1e-5))
    c.append(dict(id="rmsnorm_weights", kernel="rmsnorm", source="kernels/RMSNormTest.java:52-74",
                  input=[3.0, 4.0], weight=[0.5, 2.0],
                  expected=[fl(f32(3.0) / f32(math.sqrt(12.5)) * f32(0.5)),
                            fl(f32(4.0) / f32(math.sqrt(12.5)) * f32(2.0))], tol=1e-5))
    cos1, sin1 = fl(math.cos(1.0)), fl(math.sin(1.0))
    cos001, sin001 = fl(math.cos(0.01)), fl(math.sin(0.01))
    c.append(dict(id="rope_2x4_pos1", kernel="rope", source="kernels/RoPETest.java:14-60",
                  num_heads=2, head_dim=4, pos=1, theta=10000.0, input=[1.0, 0.0] * 4,
                  expected=[cos1, sin1, cos001, sin001] * 2, tol=1e-5))
    c.append(dict(id="silu_3", kernel="silu", source="kernels/SiLUTest.java:24-42",
                  input=[-1.0, 0.0, 1.0],
                  expected=[fl(f32(-1.0) / (f32(1.0) + f32(math.exp(1.0)))), 0.0,
                            fl(f32(1.0) / (f32(1.0) + f32(math.exp(-1.0))))], tol=1e-6))
    for size, start in ((3, -1.0), (64, -2.0), (2048, -5.0), (8192, -10.0)):
        xs = ramp(size, start)
        c.append(dict(id=f"silu_ramp_{size}", kernel="silu", source="kernels/SiLUHatVsJavaTest.java:44-122",
                      input=xs, expected=[fl(java_silu(f32(x))) for x in xs], tol=1e-5))
    c.append(dict(id="softmax_values", kernel="softmax", source="kernels/SoftmaxTest.java:43-61",
                  input=[1.0, 2.0, 3.0, 4.0, 5.0],
                  expected=[0.01165, 0.03168, 0.08612, 0.23412, 0.63640], tol=1e-3))
    c.append(dict(id="softmax_sums_to_one", kernel="softmax", source="kernels/SoftmaxTest.java:23-41",
                  input=[1.0, 2.0, 3.0, 4.0, 5.0], property="sum", expected_sum=1.0, tol=1e-4))
    c.append(dict(id="softmax_monotonic", kernel="softmax", source="kernels/SoftmaxTest.java:63-81",
                  input=[1.0, 2.0, 3.0, 4.0], property="increasing"))
    c.append(dict(id="softmax_stable", kernel="softmax", source="kernels/SoftmaxTest.java:122-143",
                  input=[1000.0, 1001.0, 1002.0], property="finite_sum", expected_sum=1.0, tol=1e-4))
    c.append(dict(id="softmax_row", kernel="softmax_row", source="kernels/SoftmaxTest.java:83-120",
                  input=[0.0, 0.0, 0.0, 1.0, 2.0, 3.0, 4.0, 0.0, 0.0, 0.0], row_offset=3, row_size=4,
                  property="row_sum_untouched_rest", expected_sum=1.0, tol=1e-4))
    hd, sl = 64, 4
    c.append(dict(id="attention_uniform", kernel="attention", source="kernels/AttentionTest.java:15-60",
                  head_dim=hd, seq_len=sl, query=[0.1] * hd, keys=[0.01] * (sl * hd),
                  values=[float(i) for _ in range(sl) for i in range(hd)],
                  expected_scores=[0.008] * sl, expected_probs=[0.25] * sl,
                  expected_out=[float(i) for i in range(hd)], tol=1e-5))
    c.append(dict(id="f16_exact", kernel="f16_to_f32", source="F16WeightsTest.java:87-100",
                  values=[0.0, 1.0, -1.0, 0.5, 2.0, 65504.0],
                  bits=[int(np.float16(v).view(np.uint16)) for v in (0.0, 1.0, -1.0, 0.5, 2.0, 65504.0)], tol=0.0))
    for name, vals, idx, line in (("positive", [1.0, 3.0, 2.0, 0.5], 1, "10-14"),
                                  ("negative", [-5.0, -1.0, -3.0, -2.0], 1, "16-20"),
                                  ("mixed", [-1.0, 0.0, 5.0, -3.0, 2.0], 2, "22-26"),
                                  ("last", [0.0, 0.0, 0.0, 1.0], 3, "28-32"),
                                  ("single", [42.0], 0, "34-38")):
        c.append(dict(id=f"argmax_{name}", kernel="argmax", source=f"LlamaInferenceTest.java:{line}",
                      values=vals, expected_index=idx))
    return c


def main() -> None:
    data = {"about": "Known-answer vectors of the reference's kernel tests (see make_golden.py).",
            "cases": cases()}
    with open(OUT, "w") as f:
        json.dump(data, f, separators=(",", ":"))
    print(OUT, len(data["cases"]), "cases")


if __name__ == "__main__":
    main()
