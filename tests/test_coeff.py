"""SpectralBias coefficient block (model/attn_bias.py:306-324, 419-478).

CPU: the oracle's restatement against the reference's own outputs
(tests/golden/coeff_*.npz, written by gen_golden.py from SpectralBias.forward).
GPU: the fused kernel (scope_spectral_coeffs) against the fixtures.  The two
bf16 linears accumulate in a different order on the tensor cores than on the
CPU, so a hidden activation or an MLP output may round to the neighbouring
bf16 value: y is checked against the bound such roundings allow
(sum_j |W2_oj| step(h_j) + step(y_o)), and everything after the MLP is
checked tightly against the oracle evaluated on the kernel's own y, and
against the fixtures on the rows whose y came out identical."""
import os

import numpy as np
import pytest
import torch

from oracle import coeff_oracle as CO
from tests.golden import cases as C

HERE = os.path.dirname(os.path.abspath(__file__))
OUTS = ("coeff_cos", "coeff_sin", "slope", "b0", "delta_star", "pi", "budget_logits", "delta_main", "width")
# absolute tolerances on the outputs that follow the MLP (float32 arithmetic,
# transcendental functions within a few ulp of each other)
TOL = dict(coeff_cos=2e-5, coeff_sin=2e-5, slope=1e-7, b0=4e-5, delta_star=None, pi=2e-6, budget_logits=0.0,
           delta_main=None, width=1e-4)


def _load(name):
    z = np.load(os.path.join(HERE, "golden", f"coeff_{name}.npz"))
    case = C.COEFF_CASES[name]
    x = C.coeff_inputs(case)
    assert str(z["in_hash"]) == C.input_hash(*(x[n] for n in sorted(x))), "fixture inputs drifted"
    return case, x, z


def _knobs(case, z):
    T = case["T"]
    return dict(M=case["M"], omegas=torch.from_numpy(z["omegas"]), log_omegas=torch.from_numpy(z["log_omegas"]),
                delta_cap=float(min(max(int(z["delta_star_max"]), 0), T - 1)),
                logw_min=float(z["logw_min"]), logw_max=float(z["logw_max"]), use_slope=case["use_slope"],
                subtract_b0=case["subtract_b0"], c_scale=float(z["c_scale"]), width_min=float(z["width_min"]),
                width_max=float(z["width_max"]), eps=float(z["eps"]))


def _weights(case, x):
    w = {n: torch.from_numpy(x[n]) for n in ("w1", "b1", "w2", "b2")}
    if case["share"]:
        w = {n: t[0] for n, t in w.items()}
    return w


def _close(name, got, want, tol, rel=False):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    if rel:
        err = err / np.maximum(np.abs(want), 1e-30)
    assert err.max() <= tol, (name, float(err.max()), tol)


@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_oracle_matches_reference_fixture(name):
    case, x, z = _load(name)
    w = _weights(case, x)
    y = CO.mlp(torch.from_numpy(x["q"]).to(torch.bfloat16), w["w1"], w["b1"], w["w2"], w["b2"])
    assert torch.equal(y.float(), torch.from_numpy(z["y"])), "MLP restatement differs from the reference"
    kn = _knobs(case, z)
    kn.pop("omegas"), kn.pop("log_omegas")
    r = CO.heads(torch.from_numpy(z["y"]), omegas=z["omegas"], log_omegas=z["log_omegas"], **kn)
    for n in OUTS:
        np.testing.assert_allclose(r[n].numpy(), z[n], rtol=1e-6, atol=1e-7, err_msg=n)


def _bf16_step(v):
    """Spacing of bf16 values at |v| (the distance to the next bf16 magnitude)."""
    a = np.maximum(np.abs(v), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def _y_bound(q, w, y_ref):
    """How far y may move when hidden activations round to a neighbouring
    bf16 value: sum_j |W2_oj| step(h_j), plus one step of y itself."""
    h = CO.hidden(q, w["w1"], w["b1"]).float().numpy()
    w2 = np.abs(w["w2"].float().numpy())
    st = _bf16_step(h)
    if w2.ndim == 2:
        b = st @ w2.T
    else:   # per head: h [1,H,T,hid], w2 [H,n_out,hid]
        b = np.einsum("bhtk,hok->bhto", st, w2)
    return b + _bf16_step(y_ref)


def _check_against(case, z, out, y_k, rows_equal=None):
    """Kernel outputs vs the oracle on the kernel's own y (all rows)."""
    kn = _knobs(case, z)
    kn.pop("omegas"), kn.pop("log_omegas")
    r = CO.heads(torch.from_numpy(y_k), omegas=z["omegas"], log_omegas=z["log_omegas"], **kn)
    cap = kn["delta_cap"]
    for n in OUTS:
        got = getattr(out, n).cpu().numpy()
        if n in ("delta_star", "delta_main"):
            _close(n, got, r[n].numpy(), 4e-7 * max(cap, 1.0))
        else:
            _close(n, got, r[n].numpy(), TOL[n])
    if rows_equal is not None and rows_equal.any():
        for n in ("coeff_cos", "coeff_sin", "pi", "width"):
            got = getattr(out, n).cpu().numpy()[0][rows_equal]
            _close(n + " vs reference", got, z[n][0][rows_equal], TOL[n])


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_kernel_matches_reference_fixture(name):
    from scope_b200 import device_errors, spectral_coefficients
    case, x, z = _load(name)
    H, T = case["H"], case["T"]
    q = torch.from_numpy(x["q"]).to("cuda", torch.bfloat16)
    if name == "c_perhead":   # the layout the reference passes: a head-major view of [1,T,H,D]
        q = q.transpose(1, 2).contiguous().transpose(1, 2)
    w = _weights(case, x)
    device_errors("cuda")
    out = spectral_coefficients(q, **w, **_knobs(case, z), return_mlp=True)
    torch.cuda.synchronize()
    assert device_errors("cuda") == 0
    y_k = out.mlp_out.float().cpu().numpy()
    y_r = z["y"]
    diff = np.abs(y_k - y_r)
    bound = _y_bound(torch.from_numpy(x["q"]).to(torch.bfloat16), w, y_r)
    assert (diff <= bound + 1e-12).all(), float((diff / bound).max())
    same = (diff == 0).all(axis=-1)[0]            # [H,T] rows whose MLP output is identical
    assert same.mean() >= 0.5, same.mean()
    _check_against(case, z, out, y_k, rows_equal=same)


@pytest.mark.gpu
def test_c3_size_properties():
    """C3's shape (16 heads, T = 2^17, K = 16, M = 8): size-independent
    properties on every row, and the oracle on a sample of rows."""
    from scope_b200 import SpectralCoefficients, device_errors
    H, T = 16, 131072
    sc = SpectralCoefficients(head_dim=64, num_heads=H, L_train=T, K=16, M=8, seed=3)
    g = torch.Generator().manual_seed(4)
    w2 = (torch.randn(sc.w2.shape, generator=g) * 0.08)
    b2 = sc.b2 + torch.randn(sc.b2.shape, generator=g) * 0.5
    b1 = torch.randn(sc.b1.shape, generator=g) * 0.1
    sc.load_weights(sc.w1[0], b1[0], w2[0], b2[0])
    q = torch.randn(1, T, H, 64, generator=g).to("cuda", torch.bfloat16).transpose(1, 2)
    device_errors("cuda")
    res, y = sc(q, return_mlp=True)
    torch.cuda.synchronize()
    assert device_errors("cuda") == 0
    cc, cs, slope, b0, ds, pi, bl, dm, wd = res[:9]
    for t in res[:9]:
        assert torch.isfinite(t).all()
    assert (pi.sum(-1) - 1).abs().max().item() < 2e-6
    assert (b0 - cc.sum(-1)).abs().max().item() < 1e-4
    assert cc.abs().max().item() <= 1 + 1e-5 and cs.abs().max().item() <= 1 + 1e-5
    cap = float(sc.delta_star_max_active)
    assert ds.min().item() >= 0 and ds.max().item() <= cap
    assert slope.abs().max().item() <= sc.c_scale
    # sampled rows against the oracle evaluated on the kernel's own y
    rows = torch.randint(0, T, (256,), generator=g)
    yk = y[0][:, rows].float().cpu()
    r = CO.heads(yk, M=8, omegas=sc.omegas.cpu(), log_omegas=sc.log_omegas.cpu(), delta_cap=cap,
                 logw_min=sc.logw_min, logw_max=sc.logw_max, use_slope=True, subtract_b0=True, c_scale=sc.c_scale,
                 width_min=sc.width_min, width_max=sc.width_max, eps=sc.eps)
    for n, t in zip(OUTS, res[:9]):
        got = t[0][:, rows].cpu().numpy()
        if n in ("delta_star", "delta_main"):
            _close(n, got, r[n].numpy(), 4e-7 * cap)
        else:
            _close(n, got, r[n].numpy(), TOL[n])
    # the MLP on the same rows, within one bf16 step of the CPU linears
    w = {k: getattr(sc, k)[0] for k in ("w1", "b1", "w2", "b2")}
    qr = q[:, :, rows].cpu()
    yr = CO.mlp(qr, w["w1"], w["b1"], w["w2"], w["b2"]).float().numpy()
    assert (np.abs(yk.numpy()[None] - yr) <= _y_bound(qr, w, yr) + 1e-12).all()


GRAD_NAMES = ("dq", "dw1", "db1", "dw2", "db2")


def _oracle_backward(case, z, x, q_bf16):
    """Autograd through the oracle (MLP + heads) from the fixture's upstream gradients."""
    w = {n: torch.from_numpy(x[n]).clone().requires_grad_(True) for n in ("w1", "b1", "w2", "b2")}
    ww = {n: (t[0] if case["share"] else t) for n, t in w.items()}
    q = q_bf16.clone().requires_grad_(True)
    y = CO.mlp(q, ww["w1"], ww["b1"], ww["w2"], ww["b2"]).float()
    kn = _knobs(case, z)
    kn.pop("omegas"), kn.pop("log_omegas")
    r = CO.heads(y, omegas=z["omegas"], log_omegas=z["log_omegas"], **kn)
    ups = C.coeff_upstream(case)
    outs = [r[n] for n in OUTS]
    live = [i for i in range(len(OUTS)) if outs[i].requires_grad]
    torch.autograd.backward([outs[i] for i in live], [torch.from_numpy(ups[i]) for i in live])
    return {"dq": q.grad.float(), "dw1": w["w1"].grad, "db1": w["b1"].grad, "dw2": w["w2"].grad,
            "db2": w["b2"].grad}


@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_oracle_backward_matches_reference_fixture(name):
    case, x, z = _load(name)
    g = _oracle_backward(case, z, x, torch.from_numpy(x["q"]).to(torch.bfloat16))
    for n in GRAD_NAMES:
        want = z[n]
        err = np.abs(g[n].numpy() - want).max()
        assert err <= 1e-3 * max(np.abs(want).max(), 1e-6), (n, float(err))


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_backward_kernel_dy_matches_oracle(name):
    """dL/dy from the kernel against autograd through the oracle's heads, both
    evaluated on the kernel's own MLP output."""
    from scope_b200 import device_errors, spectral_coefficients
    from scope_b200.coeff import coeff_dy
    case, x, z = _load(name)
    q = torch.from_numpy(x["q"]).to("cuda", torch.bfloat16)
    kn = _knobs(case, z)
    out = spectral_coefficients(q, **_weights(case, x), **kn, return_mlp=True)
    ups = [torch.from_numpy(u) for u in C.coeff_upstream(case)]
    ups_live = [u if (n not in ("slope",) or case["use_slope"]) and (n != "b0" or case["subtract_b0"]) else None
                for n, u in zip(OUTS, ups)]
    kw = {k: v for k, v in kn.items()}
    dy = coeff_dy(out.mlp_out, [None if u is None else u.cuda() for u in ups_live], **kw)
    torch.cuda.synchronize()
    assert device_errors("cuda") == 0
    yk = out.mlp_out.float().cpu().requires_grad_(True)
    kn.pop("omegas"), kn.pop("log_omegas")
    r = CO.heads(yk, omegas=z["omegas"], log_omegas=z["log_omegas"], **kn)
    live = [i for i, u in enumerate(ups_live) if u is not None and r[OUTS[i]].requires_grad]
    torch.autograd.backward([r[OUTS[i]] for i in live], [ups_live[i] for i in live])
    want = yk.grad.numpy()
    err = np.abs(dy.cpu().numpy() - want).max()
    assert err <= 1e-4 * np.abs(want).max() + 1e-6, (float(err), float(np.abs(want).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_backward_matches_reference_fixture(name):
    """Gradients of q and of the MLP weights through the autograd path (the dy
    kernel, then the reference's MLP ops) against the reference's own."""
    from scope_b200 import spectral_coefficients
    case, x, z = _load(name)
    q = torch.from_numpy(x["q"]).to("cuda", torch.bfloat16).requires_grad_(True)
    w = {n: t.cuda().requires_grad_(True) for n, t in _weights(case, x).items()}
    out = spectral_coefficients(q, **w, **_knobs(case, z))
    ups = [torch.from_numpy(u).cuda() for u in C.coeff_upstream(case)]
    outs = [getattr(out, n) for n in OUTS]
    torch.autograd.backward(outs, ups)
    got = {"dq": q.grad.float(), "dw1": w["w1"].grad, "db1": w["b1"].grad, "dw2": w["w2"].grad, "db2": w["b2"].grad}
    for n in GRAD_NAMES:
        want = z[n][0] if (case["share"] and n != "dq") else z[n]
        g = got[n].float().cpu().numpy()
        err = np.abs(g - want).max()
        assert err <= 3e-2 * max(np.abs(want).max(), 1e-6), (n, float(err), float(np.abs(want).max()))


@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_oracle_regularisers_match_reference_fixture(name):
    case, x, z = _load(name)
    kn = _knobs(case, z)
    kn.pop("omegas"), kn.pop("log_omegas")
    r = CO.heads(torch.from_numpy(z["y"]), omegas=z["omegas"], log_omegas=z["log_omegas"], **kn)
    reg = CO.reg_loss(r, omegas=z["omegas"], T=case["T"], M=case["M"], delta_cap=kn["delta_cap"], eps=kn["eps"])
    assert abs(reg.item() - float(z["t_reg"])) <= 1e-5 * abs(float(z["t_reg"])), (reg.item(), float(z["t_reg"]))


def _train_block(case, z, x):
    from scope_b200 import SpectralCoefficients
    sc = SpectralCoefficients(head_dim=64, num_heads=case["H"], L_train=case["L_train"], K=case["K"], M=case["M"],
                              share_across_heads=case["share"], use_slope=case["use_slope"],
                              subtract_b0=case["subtract_b0"], delta_star_max=case["delta_star_max"])
    w = {n: t.cuda().float().requires_grad_(True) for n, t in _weights(case, x).items()}
    sc.load_weights(w["w1"], w["b1"], w["w2"], w["b2"])
    sc.omegas = torch.from_numpy(z["omegas"]).cuda()
    sc.log_omegas = torch.from_numpy(z["log_omegas"]).cuda()
    return sc.train(), w


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(C.COEFF_CASES))
def test_training_regularisers_match_reference_fixture(name):
    """reg_loss in training mode and the gradients of reg_loss alone (the
    regularisers' share of the full gradient is ~1e-5 of it) against the
    reference's."""
    case, x, z = _load(name)
    sc, w = _train_block(case, z, x)
    q = torch.from_numpy(x["q"]).to("cuda", torch.bfloat16).requires_grad_(True)
    res = sc(q)
    reg = res[11]
    want = float(z["t_reg"])
    assert abs(reg.item() - want) <= 2e-3 * abs(want), (reg.item(), want)
    reg.backward()
    got = {"dq": q.grad.float(), "dw1": w["w1"].grad, "db1": w["b1"].grad, "dw2": w["w2"].grad, "db2": w["b2"].grad}
    for n in GRAD_NAMES:
        ref = z["r_" + n][0] if (case["share"] and n != "dq") else z["r_" + n]
        g = got[n].float().cpu().numpy()
        err = np.abs(g - ref).max()
        assert err <= 5e-2 * max(np.abs(ref).max(), 1e-12), (n, float(err), float(np.abs(ref).max()))
