"""Test helpers: mirror synthetic weights into the oracle's layout."""
import numpy as np

from oracle.littlebit import RtBranch


def oracle_branches(branches):
    np_ = lambda t: None if t is None else t.numpy()
    return [RtBranch(np_(b["v_sign"]), np_(b["v2"]), b["mid"].numpy(), b["u_sign"].numpy(),
                     b["u1"].numpy(), int(b["rank"])) for b in branches]


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


# Tolerance of the per-layer parity tests against the fp64 restatement of
# LittleBitLinear._compute_forward: rtol 1e-3 (the parity bar), plus an
# absolute floor of 1e-4 x max|y| for outputs that cancel to near zero.
def assert_linear_close(y, ref, rtol=1e-3, atol_frac=1e-4):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    np.testing.assert_allclose(y, ref, rtol=rtol, atol=atol_frac * np.abs(ref).max())
