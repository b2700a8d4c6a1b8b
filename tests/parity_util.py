"""Parity checks shared by the GPU tests, with the numbers they measured printed.

The north-star tolerance for floating-point outputs is max |err| <= 2e-3 x
RMS(reference). The decoder's logits and KV caches are fp16 storage values (the
reference rounds every linear output to its storage dtype, decoder_llm.py:16,
31, 88), so two correct implementations whose fp32 sums differ in the last bits
can land on neighbouring fp16 values when the exact result sits near a rounding
midpoint: a one-ulp difference, which for |value| >= 4 is above 2e-3 x RMS at
the C3 logit scale. `fp16_close` therefore accepts an element when it is within
2e-3 x RMS OR exactly one fp16 ulp of the reference value away, counts the
elements that needed the ulp clause and bounds that count; every call prints
max|err| / RMS, the ulp-clause count and, when given, the noise floor (the
spread between two oracles that differ only in fp32 summation order).

Greedy tokens are bit-exact (apps/decoder_llm_main.cpp:122-166): a mismatch is
accepted only where the reference's own top-2 logits are within one fp16 ulp
of each other (a storage-rounding tie) or, when the GPU's logits are given,
within twice the measured max|err| of those logits (the step's logits passed
the tolerance check, and a difference that small can reorder two logits that
close); such steps are counted and printed.
"""

import numpy as np


def fp16_ulp(values) -> np.ndarray:
    """One fp16 ulp at each |value| (the spacing to the next larger fp16)."""
    v = np.abs(np.asarray(values, np.float32)).astype(np.float16)
    return np.spacing(v).astype(np.float64)


def fp16_close(got, ref, what, floor=None, max_ulp_fraction=1e-3, stats=None):
    """max|err| <= 2e-3 x RMS(ref) per element, or a one-ulp storage-rounding
    difference (at most `max_ulp_fraction` of the elements). Returns the
    measured numbers (also printed)."""
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    rms = float(np.sqrt(np.mean(ref ** 2)))
    tol = 2e-3 * rms
    err = np.abs(got - ref)
    strict = err <= tol
    ulp = err <= fp16_ulp(ref) * (1.0 + 1e-6)
    ok = strict | ulp
    n_ulp = int(np.count_nonzero(~strict & ulp))
    worst = int(np.argmax(np.where(ok, 0.0, err)))
    ratio_strict = float(np.max(np.where(strict, err, 0.0))) / rms if rms > 0 else 0.0
    result = {"what": what, "max_err": float(err.max()), "rms": rms, "max_err_over_rms": float(err.max()) / rms,
              "max_err_over_rms_within_tol": ratio_strict, "ulp_clause": n_ulp, "elements": int(ref.size),
              "noise_floor": floor}
    print(f"[parity] {what}: max|err|/RMS {result['max_err_over_rms']:.2e} "
          f"(tol 2e-3; {ratio_strict:.2e} over the elements inside it), "
          f"one-ulp storage-rounding elements {n_ulp}/{ref.size}"
          + (f", oracle noise floor {floor:.2e} ({floor / rms:.2e} x RMS)" if floor is not None else ""))
    assert ok.all(), (f"{what}: element {worst} err {err[worst]:.3e} above 2e-3 x RMS = {tol:.3e} "
                      f"and above one fp16 ulp {fp16_ulp(ref[worst:worst + 1])[0]:.3e} (ref {ref[worst]:.4f})")
    assert n_ulp <= max(4, int(max_ulp_fraction * ref.size)), f"{what}: {n_ulp} one-ulp differences"
    if stats is not None:
        stats.append(result)
    return result


class TokenCheck:
    """Greedy tokens bit-exact against the oracle, except at fp16 ties of the
    oracle's own top-2 logits (counted)."""

    def __init__(self, what):
        self.what = what
        self.steps = 0
        self.near_ties = 0
        self.tie_mismatches = 0

    def check(self, got_token, ref_token, ref_logits, got_logits=None):
        self.steps += 1
        ref_logits = np.asarray(ref_logits, np.float32).reshape(-1)
        top2 = np.sort(ref_logits)[-2:]
        allowance = float(fp16_ulp(top2[1:])[0]) * (1.0 + 1e-6)
        if got_logits is not None:
            err = np.abs(np.asarray(got_logits, np.float64).reshape(-1) - ref_logits)
            allowance = max(allowance, 2.0 * float(err.max()))
        tie = float(top2[1] - top2[0]) <= allowance
        self.near_ties += int(tie)
        if int(got_token) != int(ref_token):
            assert tie, (f"{self.what}: token {got_token} != oracle {ref_token} "
                         f"(top-2 margin {top2[1] - top2[0]:.4g} > allowance {allowance:.4g})")
            self.tie_mismatches += 1

    def report(self):
        print(f"[parity] {self.what}: {self.steps} greedy tokens, {self.steps - self.tie_mismatches} equal, "
              f"{self.near_ties} oracle top-2 margins within the tie allowance, {self.tie_mismatches} of them differ")
        return {"steps": self.steps, "near_ties": self.near_ties, "tie_mismatches": self.tie_mismatches}
