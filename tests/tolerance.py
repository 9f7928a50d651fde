"""The parity bar for low-precision runs, in one place.

Forward output and dQ/dK/dV must lie within max-abs 2e-2 (bf16) / 5e-3 (fp16) of a float32
reference run on the same inputs. A value whose own magnitude is large (the root node's dK sums
L x num_samples contributions) cannot be stored that accurately in the output dtype: one bf16
ulp at |x| = 64 is 0.5. For such entries the bar adds at most ``ulps`` units in the last place
of the output dtype at |ref|:

    |got - ref| <= atol + ulps * ulp_dtype(|ref|)

with ulp_bf16(x) = 2^(floor(log2 x) - 7) and ulp_fp16(x) = 2^(floor(log2 x) - 10). Below
|ref| = 2.56 (bf16) / 10 (fp16) the ulp term is smaller than atol, so there the bar is the
plain max-abs tolerance.
"""

from __future__ import annotations

import numpy as np

ATOL = {"bf16": 2e-2, "f16": 5e-3}
MANTISSA_BITS = {"bf16": 7, "f16": 10, "f32": 23}


def ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """One unit in the last place of ``dtype`` at |x| (normal range)."""
    a = np.maximum(np.abs(np.asarray(x, np.float64)), np.finfo(np.float32).tiny)
    return np.exp2(np.floor(np.log2(a)) - MANTISSA_BITS[dtype])


def assert_within(got, ref, dtype: str, name: str = "", ulps: int = 2, atol: float | None = None):
    """Assert |got - ref| <= atol + ulps * ulp_dtype(ref) elementwise; report the worst entry."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, f"{name}: shape {got.shape} vs {ref.shape}"
    a = ATOL[dtype] if atol is None else atol
    bound = a + ulps * ulp(ref, dtype)
    err = np.abs(got - ref)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{name}: {int(bad.sum())} of {err.size} entries beyond atol {a} + {ulps} ulp; worst at "
            f"{tuple(int(x) for x in i)}: got {got[i]:.6g}, ref {ref[i]:.6g}, |err| {err[i]:.3g} "
            f"> {bound[i]:.3g} (max |err| {err.max():.3g})")
