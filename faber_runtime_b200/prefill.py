"""Logits comparison harness — compare_gpu_logits (src/prefill.rs:387-440).

The reference gates GPU prompt-end logits on: top-1 over non-EOG ids equal,
every element within |gpu - golden| <= atol + rtol*|golden| (1e-5/1e-5 for
its own pinned row), and a finite gate. The same verdict fields are kept
here; the tolerance is a parameter because the synthetic Q4_K workloads
state theirs as max-abs <= 1e-3 x RMS(golden).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

Q2_ATOL = 1e-5
Q2_RTOL = 1e-5


def top1_non_eog(logits: np.ndarray, eog=()) -> int:
    """Argmax over non-EOG ids, lowest id on ties, -inf/NaN never win
    (src/cpu_oracle.rs:979-995)."""
    lg = np.asarray(logits, np.float32).copy()
    bad = ~(lg > -np.inf)
    lg[bad] = -np.inf
    for e in eog:
        if 0 <= e < lg.size:
            lg[e] = -np.inf
    if not np.any(lg > -np.inf):
        return 0
    return int(np.argmax(lg))


@dataclass
class PrefillComparison:
    gpu_top1: int
    golden_top1: int
    top1_matches: bool
    max_delta: float
    numeric_matches: bool
    all_finite: bool
    failing_thresholds: list = field(default_factory=list)
    ok: bool = False

    def divergence_field(self) -> str:
        if self.ok:
            return "none"
        return (f"position 0 (prompt end): GPU top-1 {self.gpu_top1} vs golden {self.golden_top1}; "
                f"failing [{', '.join(self.failing_thresholds)}]; max delta {self.max_delta:.3e}")


def compare_gpu_logits(gpu_logits, golden_logits, eog=(0, 2), atol: float = Q2_ATOL,
                       rtol: float = Q2_RTOL, rms_tol: float | None = None) -> PrefillComparison:
    """Verdict of the reference's Q2 comparison. ``rms_tol`` switches the
    numeric row to max|gpu - golden| <= rms_tol * RMS(golden)."""
    g = np.asarray(gpu_logits, np.float32)
    o = np.asarray(golden_logits, np.float32)
    if g.shape != o.shape or g.ndim != 1:
        raise ValueError("comparison needs equal-length logits vectors")
    gpu_top1, golden_top1 = top1_non_eog(g, eog), top1_non_eog(o, eog)
    finite = bool(np.all(np.isfinite(g)) and np.all(np.isfinite(o)))
    both = np.isfinite(g) & np.isfinite(o)
    delta = np.abs(g[both].astype(np.float64) - o[both].astype(np.float64))
    max_delta = float(delta.max()) if delta.size else 0.0
    if rms_tol is not None:
        rms = float(np.sqrt(np.mean(o[both].astype(np.float64) ** 2))) if both.any() else 0.0
        numeric = finite and max_delta <= rms_tol * rms
    else:
        bound = atol + rtol * np.abs(o[both].astype(np.float64))
        numeric = finite and bool(np.all(delta <= bound))
    failing = []
    if gpu_top1 != golden_top1:
        failing.append("top-1")
    if not numeric:
        failing.append("band")
    if not finite:
        failing.append("finite")
    return PrefillComparison(gpu_top1, golden_top1, gpu_top1 == golden_top1, max_delta, numeric,
                             finite, failing, not failing)
