"""The operator's parity bar: |x - ref| <= atol + rtol*|ref| elementwise with
rtol = 2e-3, atol = 1e-2 (bf16 inputs, fp32 accumulation), for outputs, final
states and every gradient."""

import numpy as np

RTOL, ATOL = 2e-3, 1e-2


def to_np(x):
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().float().cpu().numpy().astype(np.float64)
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, np.float64)


def assert_close(actual, expected, name="", rtol=RTOL, atol=ATOL):
    a, e = to_np(actual), to_np(expected)
    assert a.shape == e.shape, f"{name}: shape {a.shape} vs {e.shape}"
    assert np.isfinite(a).all(), f"{name}: non-finite values"
    err = np.abs(a - e)
    bad = err > atol + rtol * np.abs(e)
    assert not bad.any(), (
        f"{name}: {int(bad.sum())}/{bad.size} out of tolerance (rtol={rtol}, atol={atol}); "
        f"max abs err {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}, "
        f"max |ref| {np.abs(e).max():.3e}")


def max_err(actual, expected):
    return float(np.abs(to_np(actual) - to_np(expected)).max())


def gate_param_masses(g_raw, dt_bias, dg_raw, H):
    """Summed magnitudes of the terms that the A_log and dt_bias gradients add
    up: dA_log[h] = sum_{t,c} dy*yg and ddt_bias[h,c] = sum_t dg_raw, with
    |dy*yg| = |dg_raw| * softplus(x) / sigmoid(x), x = g + dt_bias.  A bound on
    a sum of N rounded terms scales with this mass, not with the sum itself."""
    g = to_np(g_raw)
    K = g.shape[-1]
    x = g + (to_np(dt_bias).reshape(H, K) if dt_bias is not None else 0.0)
    sp = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
    sg = 1.0 / (1.0 + np.exp(-x))
    d = np.abs(to_np(dg_raw))
    mA = (d * sp / sg).reshape(-1, H, K).sum((0, 2))
    mdt = d.reshape(-1, H * K).sum(0)
    return mA, mdt


def assert_close_reduced(actual, expected, mass, name="", rtol=RTOL, atol=ATOL):
    """Parity for a gradient that is a sum of many terms: |x - ref| <= atol + rtol * sum|terms|."""
    a, e, m = to_np(actual), to_np(expected), to_np(mass)
    err = np.abs(a - e)
    bad = err > atol + rtol * m
    assert not bad.any(), (f"{name}: {int(bad.sum())}/{bad.size} out of tolerance; max abs err "
                           f"{err.max():.3e}, bound {float((atol + rtol * m).min()):.3e}")
