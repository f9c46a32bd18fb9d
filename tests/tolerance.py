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
