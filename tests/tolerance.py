"""The output tolerance of every expert-FFN parity test (GPU output against the dequantised reference).

Two conditions, both required:
  * the north star's: max |y - ref| / max |ref| <= RTOL (1e-2), the maximum error relative to the
    largest reference value;
  * elementwise: |y - ref| <= RTOL * |ref| + ATOL_RMS * rms(ref) for every element, with
    ATOL_RMS = 1e-2, so no element may be off by more than 1% of itself plus 1% of the output's RMS.
    The absolute term covers outputs near zero, where a relative bound alone is meaningless. The GPU
    rounds y to bf16 (at most 2^-9 of |y|) and, on the tensor-core path, each dequantised weight and
    the SwiGLU output to f16 (2^-11 each), so its error sits well inside both terms.
"""
import numpy as np

RTOL = 1e-2
ATOL_RMS = 1e-2


def check_close(got, ref, rtol: float = RTOL, atol_rms: float = ATOL_RMS):
    """Returns (global relative error, worst elementwise ratio err / bound); the test passes when both
    are <= 1 after dividing the first by rtol."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = np.abs(got - ref)
    glob = float(err.max() / max(np.abs(ref).max(), 1e-30))
    bound = rtol * np.abs(ref) + atol_rms * float(np.sqrt(np.mean(ref * ref)))
    worst = float((err / np.maximum(bound, 1e-30)).max())
    return glob, worst


def assert_close(got, ref, rtol: float = RTOL, atol_rms: float = ATOL_RMS, what: str = ""):
    glob, worst = check_close(got, ref, rtol, atol_rms)
    assert glob <= rtol and worst <= 1.0, (f"{what}: max|err|/max|ref| = {glob:.3e} (limit {rtol}), "
                                           f"worst elementwise err/bound = {worst:.3f} (limit 1)")
