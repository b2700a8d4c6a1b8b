"""Parity checks shared by the GPU tests, with the numbers they measured printed.

The north-star tolerance for floating-point outputs is max |err| <= 2e-3 x
RMS(reference). The decoder's logits and KV caches are fp16 storage values (the
reference rounds every linear output to its storage dtype, decoder_llm.py:16,
31, 88), so two correct implementations whose fp32 sums differ in the last bits
can land on neighbouring fp16 values when the exact result sits near a rounding
midpoint: a one-ulp difference, which for |value| >= 4 is above 2e-3 x RMS at
the C3 logit scale. `fp16_close` therefore accepts an element when it is within
2e-3 x RMS OR one fp16 ulp of the reference value. At full model width the
oracle itself, run twice with different fp32 summation orders, differs by more
than 2e-3 x RMS (the fp16 roundings of every activation amplify last-bit
differences); there the measured spread (the noise floor) is passed in and the
bound becomes max(2e-3 x RMS, 3 x floor) with at most 0.1% of the elements
beyond the element-wise bound. Every call prints max|err| / RMS, the counts and
the floor.

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


def fp16_close(got, ref, what, floor=None, twin=None, twin_outside_fraction=None, stats=None):
    """Element-wise: |err| <= max(2e-3 x RMS(ref), one fp16 ulp of ref).

    Without a noise measurement every element must pass. With one -- `twin`
    (the same oracle run with a permuted fp32 summation order, from which the
    floor and the twin's own out-of-bound fraction are measured here) or
    `floor` and `twin_outside_fraction` measured on the same model elsewhere --
    the output must be as close to the oracle as the oracle is to itself:
    max |err| <= max(2e-3 x RMS, 3 x floor), and the fraction of elements
    beyond the element-wise bound at most twice the twin's (plus 0.1%). At full
    model width the fp16 roundings of every activation put a few percent of
    the oracle twin's own logits beyond 2e-3 x RMS. Returns the measured
    numbers (also printed)."""
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    rms = float(np.sqrt(np.mean(ref ** 2)))
    tol = 2e-3 * rms
    ulp_ref = fp16_ulp(ref) * (1.0 + 1e-6)

    def outside(values):
        e = np.abs(values - ref)
        return e, ~((e <= tol) | (e <= ulp_ref))

    err, out = outside(got)
    n_ulp = int(np.count_nonzero((err > tol) & ~out))
    n_out = int(np.count_nonzero(out))
    if twin is not None:
        terr, tout = outside(np.asarray(twin, np.float64).reshape(-1))
        floor = float(terr.max())
        twin_outside_fraction = float(np.count_nonzero(tout)) / ref.size
    worst = int(np.argmax(err))
    result = {"what": what, "max_err": float(err[worst]), "rms": rms, "max_err_over_rms": float(err[worst]) / rms,
              "one_ulp_elements": n_ulp, "outside_elements": n_out, "elements": int(ref.size),
              "noise_floor": floor, "twin_outside_fraction": twin_outside_fraction}
    print(f"[parity] {what}: max|err|/RMS {result['max_err_over_rms']:.2e} (north star 2e-3), "
          f"one-ulp storage-rounding elements {n_ulp}/{ref.size}, beyond both {n_out} ({n_out / ref.size:.2%})"
          + (f"; oracle twin: max|err|/RMS {floor / rms:.2e}" if floor is not None else "")
          + (f", beyond both {twin_outside_fraction:.2%}" if twin_outside_fraction is not None else ""))
    if floor is None:
        assert n_out == 0, (f"{what}: element {worst} err {err[worst]:.3e} above 2e-3 x RMS = {tol:.3e} "
                            f"and above one fp16 ulp (ref {ref[worst]:.4f})")
    else:
        bound = max(tol, 3.0 * floor)
        assert err[worst] <= bound, (f"{what}: max err {err[worst]:.3e} above max(2e-3 x RMS, 3 x noise floor) = "
                                     f"{bound:.3e} (ref {ref[worst]:.4f})")
        allowed = (2.0 * (twin_outside_fraction or 0.0) + 1e-3) * ref.size
        assert n_out <= allowed, f"{what}: {n_out} elements beyond 2e-3 x RMS and one ulp (allowed {allowed:.0f})"
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
