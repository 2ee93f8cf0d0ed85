"""Tolerances and error measures used by every parity test.

Floating-point gate (per kernel): max relative error <= 1e-3 against the
oracle's fp32 result, measured element-wise with a floor:

    rel = max_i |g_i - r_i| / max(|r_i|, 1e-2 * max_j |r_j|)

Entries smaller than 1% of the largest entry are dominated by the
reference's own sequential fp32 rounding (its dot products accumulate in
column order), so they are held to an absolute bound of 1e-5 * max|r|
instead.  Every failure message also carries the strict figure, the same
quotient with a floor of 1e-6 * max|r| (so near-zero entries count in full),
and the normwise error max|g - r| / max|r|; `parity_report` returns all
three for tests that log them.
End to end: logits max-abs <= 1e-2; greedy tokens identical wherever the
oracle's top-2 logit margin exceeds 1e-2.  Long decodes (hundreds of
positions through every layer) are gated end to end plus a normwise bound
of 1e-4 on the logits, with the relative figures reported.
"""
import numpy as np

KERNEL_REL_TOL = 1e-3
LOGITS_ABS_TOL = 1e-2
NORMWISE_E2E_TOL = 1e-4  # end-to-end logits: max|g - r| / max|r|
MARGIN = 1e-2
GATE_FLOOR = 1e-2    # floor of the gated relative error, as a fraction of max|r|
STRICT_FLOOR = 1e-6  # floor of the strict (reported) relative error


def max_rel_err(g, r, floor: float = GATE_FLOOR) -> float:
    g = np.asarray(g, np.float64).ravel()
    r = np.asarray(r, np.float64).ravel()
    if r.size == 0:
        return 0.0
    big = np.abs(r).max()
    den = np.maximum(np.abs(r), floor * big)
    den[den == 0] = 1.0
    return float((np.abs(g - r) / den).max())


def normwise_err(g, r) -> float:
    g = np.asarray(g, np.float64).ravel()
    r = np.asarray(r, np.float64).ravel()
    if r.size == 0:
        return 0.0
    big = np.abs(r).max()
    return float(np.abs(g - r).max() / (big if big else 1.0))


def parity_report(g, r) -> dict:
    """The gated figure, the strict figure and the normwise error of g vs r."""
    return {"rel_gate": max_rel_err(g, r, GATE_FLOOR), "rel_strict": max_rel_err(g, r, STRICT_FLOOR),
            "normwise": normwise_err(g, r)}


def describe(g, r) -> str:
    d = parity_report(g, r)
    return (f"max rel err {d['rel_gate']:.3e} (floor {GATE_FLOOR:g}*max|r|); strict {d['rel_strict']:.3e} "
            f"(floor {STRICT_FLOOR:g}*max|r|); normwise {d['normwise']:.3e}")


def assert_kernel_close(g, r, tol: float = KERNEL_REL_TOL):
    e = max_rel_err(g, r)
    assert e <= tol, f"{describe(g, r)}; gate {tol}"


def top2_margin(logits) -> float:
    s = np.sort(np.asarray(logits, np.float64))
    return float(s[-1] - s[-2])
