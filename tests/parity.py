"""Tolerances of the parity contract (stated once, used by every parity test).

elementwise : per element, |gpu - ref| <= 1e-6 * |ref| where |ref| > 1e-30, else <= 1e-30
              (bit-exact for graphs of + - * / relu, which round identically)
reduction   : norm-wise ||gpu - ref||_2 <= 1e-6 * ||ref||_2 ; max bit-exact
gemm        : relative Frobenius ||gpu - ref||_F <= 1e-5 * ||ref||_F
transcendental elementwise (exp, tanh, sigmoid in the expression): the reference's float
              libm (glibc expf/tanhf) and the GPU's correctly rounded double-evaluated
              exp/tanh can differ by an ulp, which a later cancelling subtraction turns
              into large relative error of a small result.  Per element:
              |gpu - ref| <= 1e-6 * |ref| + 8 * 2^-24 * m, with m the element's
              magnitude bound (oracle.magnitude: |.| on every operand, + for every +/-),
              the standard floating-point rounding-error scale of the expression.
identity    : reference values obtained through op identities (exp = sigmoid(x)/sigmoid(-x),
              tanh = 2 sigmoid(2x) - 1) carry the identity's own rounding; the oracle is
              held to 2e-5 relative + 1e-6 absolute against them.
"""

import numpy as np

ELEMENTWISE_RTOL = 1e-6
ELEMENTWISE_ATOL = 1e-30
REDUCTION_NORM_RTOL = 1e-6
GEMM_FROB_RTOL = 1e-5
IDENTITY_RTOL = 2e-5
IDENTITY_ATOL = 1e-6


def assert_elementwise(got, ref, rtol=ELEMENTWISE_RTOL, atol=ELEMENTWISE_ATOL):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_ref = np.isnan(ref)
    assert np.array_equal(nan_ref, np.isnan(got)), "NaN pattern differs"
    inf_ref = np.isinf(ref)
    assert np.array_equal(got[inf_ref], ref[inf_ref]), "inf values differ"
    m = ~(nan_ref | inf_ref)
    g, r = got[m].astype(np.float64), ref[m].astype(np.float64)
    big = np.abs(r) > atol
    err = np.abs(g - r)
    assert np.all(err[big] <= rtol * np.abs(r[big])), f"max rel err {np.max(err[big] / np.abs(r[big])) if big.any() else 0}"
    assert np.all(err[~big] <= atol), "abs err on tiny values"


TRANSCENDENTAL_ULPS = 8.0


def assert_elementwise_scaled(got, ref, mag, rtol=ELEMENTWISE_RTOL, ulps=TRANSCENDENTAL_ULPS):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    mag = np.asarray(mag, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_ref = np.isnan(ref)
    assert np.array_equal(nan_ref, np.isnan(got)), "NaN pattern differs"
    inf_ref = np.isinf(ref)
    assert np.array_equal(got[inf_ref], ref[inf_ref]), "inf values differ"
    m = ~(nan_ref | inf_ref)
    g, r = got[m].astype(np.float64), ref[m].astype(np.float64)
    bound = rtol * np.abs(r) + ulps * 2.0 ** -24 * np.broadcast_to(mag, got.shape)[m]
    err = np.abs(g - r)
    bad = err > bound
    assert not bad.any(), f"{int(bad.sum())} elements exceed the bound; worst excess {np.max(err - bound):.3e}"


def assert_bitexact(got, ref):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    gi, ri = got.view(np.uint32), ref.view(np.uint32)
    bad = gi != ri
    # NaN payloads may differ; all NaNs are equivalent
    bad &= ~(np.isnan(got) & np.isnan(ref))
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} elements differ; first {got[bad][:4]} vs {ref[bad][:4]}"


def norm_rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    den = np.linalg.norm(ref.ravel())
    return np.linalg.norm((got - ref).ravel()) / (den if den > 0 else 1.0)


def assert_norm(got, ref, rtol):
    assert np.asarray(got).shape == np.asarray(ref).shape, (np.asarray(got).shape, np.asarray(ref).shape)
    e = norm_rel(got, ref)
    assert e <= rtol, f"norm-wise relative error {e:.3e} > {rtol:.1e}"
