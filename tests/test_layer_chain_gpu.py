"""One SCOPE attention layer chained through this package the way
CausalSelfAttention.forward chains the reference's pieces
(scoped_medium.py:340-476, qk_aug mode): q -> the coefficient block
(coefficients, slope, delta*, pi, budget logits) -> the pointer block mask
built from delta* and the budget logits -> block-sparse attention with the
spectral bias -> out, then the backward to q, k, v, the coefficients and the
slope.  Each stage is checked against its oracle evaluated on the previous
stage's GPU outputs, so a mismatch in shapes, strides or semantics between
the stages shows up here."""
import math

import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO
from oracle import coeff_oracle as CO
from oracle import mask_oracle as MO

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_layer_chain_matches_oracles():
    from scope_b200 import (PointerBlockMaskBuilder, SpectralCoefficients, SpectralScoreMod, device_errors,
                            flex_attention)
    H, T, bs, K, M = 2, 1024, 128, 8, 4
    g = torch.Generator().manual_seed(21)
    # the layout the reference passes: head-major views of [1, T, H, 64]
    q, k, v, do = (torch.randn(1, T, H, 64, generator=g).to(DEV, torch.bfloat16).transpose(1, 2)
                   for _ in range(4))
    docs = torch.zeros(T, dtype=torch.int32)
    docs[T // 2 + 37:] = 1
    sc = SpectralCoefficients(head_dim=64, num_heads=H, L_train=T, K=K, M=M, seed=5)
    n_out = 5 * M + 1
    b2 = sc.b2[0] + torch.randn(n_out, generator=g) * 0.5
    b2[:M] = torch.linspace(-2.0, 2.0, M)
    sc.load_weights(sc.w1[0], torch.randn(128, generator=g) * 0.1, torch.randn(n_out, 128, generator=g) * 0.08, b2)
    device_errors(DEV)

    # 1. coefficient block
    res, y = sc(q, return_mlp=True)
    cc, cs, slope, b0, ds, pi, bl, dm, wd, cos_t, sin_t, reg = res
    cap = float(min(sc.delta_star_max, T - 1))
    r = CO.heads(y.float().cpu(), M=M, omegas=sc.omegas.cpu(), log_omegas=sc.log_omegas.cpu(), delta_cap=cap,
                 logw_min=sc.logw_min, logw_max=sc.logw_max, use_slope=True, subtract_b0=True, c_scale=sc.c_scale,
                 width_min=sc.width_min, width_max=sc.width_max, eps=sc.eps)
    assert (cc.cpu() - r["coeff_cos"]).abs().max().item() < 2e-5
    assert (ds.cpu() - r["delta_star"]).abs().max().item() < 4e-7 * cap
    assert reg.item() == 0.0

    # 2. pointer block mask from delta* and the budget logits (the representative rows t_rep)
    knobs = dict(local_blocks=2, half_blocks=2, global_blocks_max=1, budget_blocks=4, budget_is_total=False,
                 budget_temp=0.5)
    builder = PointerBlockMaskBuilder(num_heads=H, M=M, pointer_local_blocks=2, pointer_half_blocks=2,
                                      pointer_global_blocks=1, pointer_budget_blocks=4,
                                      pointer_budget_is_total=False, pointer_budget_temp=0.5)
    bm = builder.build_pointer_blockmask(docs=docs.to(DEV), delta_star=ds, pi=pi, budget_logits=bl, block_size=bs)
    ref = MO.build_pointer_blockmask(docs=docs.numpy(), block_size=bs, M=M,
                                     budget_rep=bl[0, :, bs - 1::bs].cpu().numpy(),
                                     delta_rep=ds[0, :, bs - 1::bs].cpu().numpy(), **knobs)
    np.testing.assert_array_equal(bm.kv_num_blocks[0].cpu().numpy(), ref["kv_num"])
    np.testing.assert_array_equal(bm.kv_indices[0].cpu().numpy(), ref["kv_packed"])

    # 3. attention with the spectral bias (qk_aug), forward and backward
    ql, kl, vl = (t.detach().requires_grad_(True) for t in (q, k, v))
    ccl, csl, sll = (t[0].detach().requires_grad_(True) for t in (cc, cs, slope))
    sm = SpectralScoreMod(coeff_cos=ccl, coeff_sin=csl, cos_tab=cos_t, sin_tab=sin_t, beta=0.5, slope=sll,
                          impl="qk_aug")
    out = flex_attention(ql, kl, vl, bm, score_mod=sm, scale=0.12)
    out.backward(do)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    # the oracle on the augmented inputs cast to q's dtype, as the reference casts
    # them (scoped_medium.py:380-423), then the chain rule to the coefficients
    mask = AO.dense_mask(ref["kv_num"], ref["kv_packed"], T, bs, docs=docs.numpy())
    c0 = lambda t: t[0].cpu()
    qa, ka, va = AO.qk_aug_inputs(c0(q), c0(k), c0(v), c0(cc), c0(cs), cos_t.cpu(), sin_t.cpu(), beta=0.5,
                                  scale=0.12, slope=c0(slope))
    dof = c0(do).float()
    pad = torch.zeros(H, T, va.shape[-1] - 64)
    o = AO.plain_grads(qa.float(), ka.float(), va.float(), torch.cat([dof, pad], -1), mask, scale=0.12)
    s = math.sqrt(0.5 / 0.12)
    dqa = o["dq"][..., 64:]
    ct = cos_t.cpu().to(torch.float64).transpose(0, 1)[None]
    st = sin_t.cpu().to(torch.float64).transpose(0, 1)[None]
    o["dcoeff_cos"] = s * (dqa[..., :K] * ct + dqa[..., K:2 * K] * st)
    o["dcoeff_sin"] = s * (dqa[..., :K] * st - dqa[..., K:2 * K] * ct)
    o["dslope"] = -s * dqa[..., 2 * K]
    for n in ("out", "dq", "dk", "dv"):
        o[n] = o[n][..., :64]
    for name, got, want in (("out", out[0], o["out"]), ("dq", ql.grad[0], o["dq"]), ("dk", kl.grad[0], o["dk"]),
                            ("dv", vl.grad[0], o["dv"])):
        err = (got.double().cpu() - want).abs().max().item()
        assert err < 2e-2, (name, err)
    for name, got, want in (("dcoeff_cos", ccl.grad, o["dcoeff_cos"]), ("dcoeff_sin", csl.grad, o["dcoeff_sin"]),
                            ("dslope", sll.grad, o["dslope"])):
        scale_ = want.abs().max().item()
        err = (got.double().cpu() - want).abs().max().item()
        assert err < 2e-2 * max(1.0, scale_), (name, err, scale_)
