"""Comparison helpers shared by the parity tests."""

from __future__ import annotations

import numpy as np

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def bf16_tol(values, ulps: float = 2.0, floor: float = 2e-2) -> float:
    """Absolute tolerance for BF16 results: ``ulps`` BF16 ulps of the largest
    magnitude (2**-7 relative per ulp at the top of a binade), never below ``floor``."""
    m = float(np.max(np.abs(values))) if np.size(values) else 0.0
    if m == 0.0:
        return floor
    ulp = 2.0 ** (np.floor(np.log2(m)) - 7)
    return max(floor, ulps * ulp)


def beam_mismatches(tok_a, sc_a, tok_b, sc_b, tol: float) -> list[str]:
    """Differences between two GRBeam results that are NOT near-ties.

    Per request, beams are compared as sets of token sequences.  A sequence
    found in only one result is accepted when its score lies within ``tol`` of
    that result's boundary (its lowest finite score): the two runs then
    disagree only about which of several near-equal candidates fills the last
    slots.  Sequences found in both must agree in score within ``tol``.
    Scores must be sorted in descending order.
    """
    problems = []
    tok_a, tok_b = np.asarray(tok_a), np.asarray(tok_b)
    sc_a, sc_b = np.asarray(sc_a, np.float64), np.asarray(sc_b, np.float64)
    for r in range(tok_a.shape[0]):
        for name, sc in (("a", sc_a[r]), ("b", sc_b[r])):
            fin = sc[np.isfinite(sc)]
            if np.any(np.diff(fin) > 1e-6):
                problems.append(f"request {r}: scores of {name} not sorted")
        A = {tuple(s): v for s, v in zip(tok_a[r].tolist(), sc_a[r]) if np.isfinite(v)}
        B = {tuple(s): v for s, v in zip(tok_b[r].tolist(), sc_b[r]) if np.isfinite(v)}
        la = min(A.values()) if A else -np.inf
        lb = min(B.values()) if B else -np.inf
        for seq in A.keys() & B.keys():
            if abs(A[seq] - B[seq]) > tol:
                problems.append(f"request {r}: beam {seq} score {A[seq]:.5f} vs {B[seq]:.5f}")
        for seq in A.keys() - B.keys():
            if A[seq] - la > tol:
                problems.append(f"request {r}: beam {seq} ({A[seq]:.5f}) only in a, boundary {la:.5f}")
        for seq in B.keys() - A.keys():
            if B[seq] - lb > tol:
                problems.append(f"request {r}: beam {seq} ({B[seq]:.5f}) only in b, boundary {lb:.5f}")
        if np.isfinite(sc_a[r]).sum() != np.isfinite(sc_b[r]).sum():
            problems.append(f"request {r}: different number of valid beams")
    return problems


def assert_close_rel(actual, desired, rel: float = 1e-2, peak: float = 5e-2, what: str = "") -> None:
    """BF16-path closeness: relative L2 error <= ``rel`` and every element within
    ``peak`` x max|desired|.  Rounding noise from a different accumulation order
    propagates through layers, so elementwise ulp bounds are too strict here."""
    a = np.asarray(actual, np.float64)
    d = np.asarray(desired, np.float64)
    assert a.shape == d.shape, f"{what}: shape {a.shape} vs {d.shape}"
    assert np.array_equal(np.isfinite(a), np.isfinite(d)), f"{what}: finiteness differs"
    fin = np.isfinite(d)
    a, d = a[fin], d[fin]
    scale = float(np.linalg.norm(d)) or 1.0
    err = float(np.linalg.norm(a - d)) / scale
    assert err <= rel, f"{what}: relative L2 error {err:.3e} > {rel}"
    top = float(np.max(np.abs(d))) if d.size else 0.0
    worst = float(np.max(np.abs(a - d))) if d.size else 0.0
    assert worst <= peak * max(top, 1e-30), f"{what}: max abs error {worst:.3e} > {peak} x {top:.3e}"


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) or 1.0))


def assert_bf16_as_accurate(ours, ref_bf16, exact, slack: float = 1.5, floor: float = 5e-3, what: str = "") -> None:
    """End-to-end BF16 check: ours must be as close to the exact (fp32) answer as
    the reference's own BF16 path is (within ``slack`` x, plus ``floor``)."""
    e_ours = rel_l2(ours, exact)
    e_ref = rel_l2(ref_bf16, exact)
    assert e_ours <= slack * e_ref + floor, f"{what}: error vs fp32 {e_ours:.3e}, reference bf16 {e_ref:.3e}"
