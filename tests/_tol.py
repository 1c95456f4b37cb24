"""Tolerance rules of the parity tests (stated once, used everywhere).

* Integer, byte and index results: bit-exact.
* IEEE-exact fp32 operations (add, sub, mul, div, min, max, the fp32->bf16
  cast): bit-exact.
* fp32 results of multi-step math: relative tolerance 1e-4.
* bf16 results against the fp32 oracle: relative tolerance 1e-2.

The stated tolerances are enforced on the output's own scale by
assert_output_close: |got - ref| <= rtol * max(|ref|, rms(ref)) element-wise.
That is the tolerance a caller reads off the output (a TF32 product, or an
attention output a few percent off, fails it); the condition-number forms
below (|A||B| for a product, P|V| for attention) are kept beside it as a
second, looser check that names the source of an error.

"Relative" is measured against max(|ref|, floor * rms(ref)) element-wise, so
that entries whose exact value is near zero (cancellation in a sum, a dot
product or a rotation) are judged on the scale of the tensor rather than on
their own vanishing magnitude.  Sums are judged against the sum of absolute
values of their terms, the natural condition number of summation.
"""
import numpy as np


def rel_err(got, ref, floor=1e-3):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), floor * np.sqrt(np.mean(ref * ref)) if ref.size else 0.0)
    scale = np.where(scale == 0, 1.0, scale)
    return float(np.max(np.abs(got - ref) / scale)) if ref.size else 0.0


def assert_rel(got, ref, rtol, floor=1e-3, what=""):
    e = rel_err(got, ref, floor)
    assert e <= rtol, f"{what}: max relative error {e:.3e} > {rtol:.1e}"


def output_err(got, ref):
    """max |got - ref| / max(|ref|, rms(ref)) over the finite entries of ref."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    ok = np.isfinite(ref)
    if not ok.any():
        return 0.0
    g, r = got[ok], ref[ok]
    rms = float(np.sqrt(np.mean(r * r)))
    scale = np.maximum(np.abs(r), rms)
    scale = np.where(scale == 0, 1.0, scale)
    return float(np.max(np.abs(g - r) / scale))


def assert_output_close(got, ref, rtol, what="", elementwise_rtol=None):
    """The stated tolerance on the output's own scale: the norm-wise relative
    error ||got - ref|| / ||ref|| <= rtol, and element-wise
    |got - ref| <= e_rtol * max(|ref|, rms(ref)) with e_rtol = rtol unless
    given.  Prints the observed errors so a run with -s records them.

    Attention passes elementwise_rtol = 2 * rtol: its P is rounded to bf16
    before P.V (the tensor core's operand format), which alone puts single
    entries near 1e-2 of rms(O) while the norm-wise error stays near 2e-3
    (tests/test_tolerance_rules.py simulates it on the CPU)."""
    e = output_err(got, ref)
    g = np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    ok = np.isfinite(r)
    nrm = float(np.linalg.norm(g[ok] - r[ok]) / max(np.linalg.norm(r[ok]), 1e-300)) if ok.any() else 0.0
    erel = rtol if elementwise_rtol is None else elementwise_rtol
    print(f"[tol] {what}: max error {e:.3e} of max(|ref|, rms(ref)) (bound {erel:.0e}), "
          f"norm-wise {nrm:.3e} (bound {rtol:.0e})")
    assert nrm <= rtol, f"{what}: norm-wise relative error {nrm:.3e} > {rtol:.1e}"
    assert e <= erel, f"{what}: max error {e:.3e} x max(|ref|, rms(ref)) > {erel:.1e}"


def assert_sum_close(got, ref, abs_terms, rtol, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    lim = rtol * np.maximum(np.asarray(abs_terms, np.float64), 1e-30)
    bad = np.abs(got - ref) > lim
    assert not bad.any(), f"{what}: {int(bad.sum())} sums outside {rtol:.1e} x sum|x|"


def assert_dot_close(got, ref, a, b, rtol, what=""):
    """Matrix products: |got - ref| <= rtol * (|A| @ |B|) element-wise (the
    condition of each dot product), with a, b the fp32 operands (batched or not)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.abs(np.asarray(a, np.float64)) @ np.abs(np.asarray(b, np.float64))
    scale = np.maximum(scale, 1e-30)
    e = float(np.max(np.abs(got - ref) / scale)) if ref.size else 0.0
    assert e <= rtol, f"{what}: max error {e:.3e} x (|A||B|) > {rtol:.1e}"


def attention_scale(q, k, v, scale):
    """Per-element condition of O = softmax(Q K^T * scale) V: P @ |V| (P >= 0),
    in float64, for use with assert_scaled."""
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    s = np.einsum("hid,hjd->hij", q, k) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return p @ np.abs(v)


def assert_scaled(got, ref, scale, rtol, what=""):
    """|got - ref| <= rtol * scale element-wise (scale from a condition formula)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    e = float(np.max(np.abs(got - ref) / np.maximum(scale, 1e-30))) if ref.size else 0.0
    assert e <= rtol, f"{what}: max scaled error {e:.3e} > {rtol:.1e}"
