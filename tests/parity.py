"""Shared parity rules for the model-level GPU tests (test infrastructure).

Bars (the workload's tolerances): logits cosine >= 0.999 and normwise
max_rel_err <= 2e-2 against the fp32-dequant oracle at every step; ids
bit-exact given identical logits. An id the GPU picks must equal the
oracle's argmax whenever that argmax is determined, i.e. whenever the
oracle's top-2 gap exceeds twice the logit error measured at that step: an
error of at most E per logit cannot reorder two logits more than 2E apart.
Only inside that near-tie band may the ids differ.
"""
import numpy as np

from oracle import oracle as O

COS_MIN = 0.999
REL_MAX = 2e-2


def check_logits(got, ref, rel_max: float = REL_MAX) -> float:
    """Cosine and normwise relative error of every row; returns the largest
    absolute logit error seen."""
    worst = 0.0
    for g, r in zip(np.atleast_2d(got), np.atleast_2d(ref)):
        assert O.cosine(g, r) >= COS_MIN, O.cosine(g, r)
        assert O.max_rel_err(g, r) <= rel_max, O.max_rel_err(g, r)
        worst = max(worst, float(np.max(np.abs(np.asarray(g, np.float64) - np.asarray(r, np.float64)))))
    return worst


def top2_gap(r) -> float:
    s = np.sort(np.asarray(r, np.float64).ravel())
    return float(s[-1] - s[-2])


def check_id(tok: int, ref, err: float) -> bool:
    """tok must be the oracle's argmax unless the oracle's top-2 gap is
    within 2 * err; returns True when the id was determined (and matched)."""
    ref = np.asarray(ref).ravel()
    if top2_gap(ref) > 2.0 * err:
        assert int(tok) == int(np.argmax(ref)), (int(tok), int(np.argmax(ref)), top2_gap(ref), err)
        return True
    return False
