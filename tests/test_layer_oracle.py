"""Pin the layer oracle (short conv + SiLU, gated RMSNorm) to fla's own kernels:
every ``tests/golden/layer_*.npz`` (written by ``make_golden_layer.py``) must be
reproduced by ``oracle.layer_oracle``.  Both sides compute in >= fp32, so the
bound is tight: |x - ref| <= 1e-5 + 1e-4*|ref|.
"""

import numpy as np
import pytest

from golden_io import case_names, load_case
from oracle import layer_oracle as lo


def check(name, actual, expected, rtol=1e-4, atol=1e-5):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape, (name, actual.shape, expected.shape)
    err = np.abs(actual - expected)
    bad = err > atol + rtol * np.abs(expected)
    assert not bad.any(), f"{name}: {bad.sum()} / {bad.size} out of tolerance; max abs err {err.max():.3e}"


@pytest.mark.parametrize("name", case_names("conv"))
def test_short_conv_matches_fla(name):
    meta, t, _ = load_case(name)
    cu = meta["cu_seqlens"]
    y, fs, z = lo.short_conv_fwd(t["x"], t["weight"], t.get("bias"), t.get("h0"), cu)
    check("y", y, t["y"])
    check("final_state", fs, t["final_state"])
    dx, dw, db, dh0 = lo.short_conv_bwd(t["x"], t["weight"], z, t["dy"], t.get("h0"), cu)
    check("dx", dx, t["dx"])
    check("dweight", dw, t["dweight"], atol=1e-4)
    if meta["bias"]:
        check("dbias", db, t["dbias"], atol=1e-4)
    if meta["h0"]:
        check("dh0", dh0, t["dh0"])


@pytest.mark.parametrize("name", case_names("norm_gate"))
def test_norm_gate_matches_fla(name):
    meta, t, _ = load_case(name)
    y, rstd = lo.norm_gate_fwd(t["x"], t["gate"], t["weight"], meta["eps"])
    check("y", y, t["y"])
    dx, dg, dw = lo.norm_gate_bwd(t["x"], t["gate"], t["weight"], rstd, t["dy"])
    check("dx", dx, t["dx"])
    check("dgate", dg, t["dgate"])
    check("dweight", dw, t["dweight"], atol=1e-4)


def test_gates_bwd_matches_finite_difference():
    rng = np.random.default_rng(0)
    br, wr = rng.normal(size=(5, 7)), rng.normal(size=(5, 9))
    db, dw = rng.normal(size=br.shape), rng.normal(size=wr.shape)
    gb, gw = lo.gates_bwd(br, wr, db, dw, 2.0)
    h = 1e-6
    fb = (lo.gates_fwd(br + h, wr, 2.0)[0] - lo.gates_fwd(br - h, wr, 2.0)[0]) / (2 * h)
    fw = (lo.gates_fwd(br, wr + h)[1] - lo.gates_fwd(br, wr - h)[1]) / (2 * h)
    np.testing.assert_allclose(gb, db * fb, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(gw, dw * fw, rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("name", case_names("layer"))
def test_layer_composite_matches_reference_layer(name):
    """The fp64 composite (projections -> prep -> operator oracle -> gated norm
    -> output projection, and its hand-written backward) against the
    reference's own GatedDeltaNet2 run in fp32."""
    meta, t, _ = load_case(name)
    params = {k[2:]: v for k, v in t.items() if k.startswith("p:")}
    cfg = dict(num_heads=meta["num_heads"], head_dim=meta["head_dim"], conv_size=meta["conv_size"],
               allow_neg_eigval=meta["allow_neg_eigval"], norm_eps=meta["norm_eps"],
               num_v_heads=meta.get("num_v_heads"))
    out, G = lo.layer_forward_backward(params, t["x"], t["dout"], cfg)
    check("out", out, t["out"], rtol=1e-3, atol=1e-5)
    check("dx", G["x"], t["dx"], rtol=1e-3, atol=1e-5)
    for n in params:
        ref = t["g:" + n]
        scale = float(np.abs(ref).max())
        check("d" + n, G[n], ref, rtol=1e-3, atol=1e-4 * scale)


@pytest.mark.parametrize("name", case_names("layer"))
def test_layer_state_dict_matches_reference(gdn2, name):
    """A reference GatedDeltaNet2 state dict loads into the B200 layer unchanged."""
    meta, t, _ = load_case(name)
    ref = {k[2:]: v.shape for k, v in t.items() if k.startswith("p:")}
    m = gdn2.GatedDeltaNet2(hidden_size=meta["hidden"], head_dim=meta["head_dim"], num_heads=meta["num_heads"],
                            num_v_heads=meta.get("num_v_heads"), conv_bias=meta["conv_bias"],
                            allow_neg_eigval=meta["allow_neg_eigval"])
    ours = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert ours == {k: tuple(s) for k, s in ref.items()}
