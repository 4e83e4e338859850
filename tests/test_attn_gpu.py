"""CUDA attention (forward and backward) vs the float64 oracle and the
reference-generated fixtures.  Tolerances follow the spec: max-abs 1e-4 for
float32 inputs, 2e-2 for bf16 inputs, against the reference's math."""
import math
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import attn_oracle as AO
from oracle import mask_oracle as MO
from scope_b200 import SpectralScoreMod, build_mask, flex_attention, trig_tables

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _load(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


def _mask_from_lists(kv_num, kv_idx, T, bs, docs):
    """A ScopeBlockMask for given kv lists, built by the CUDA builder from
    equivalent knobs is not always possible; build one directly instead."""
    from scope_b200.mask import ScopeBlockMask, block_info
    H, QB = kv_num.shape
    words = (QB + 31) // 32
    bm = np.zeros((H, QB, words), dtype=np.uint32)
    for h in range(H):
        for q in range(QB):
            for kb in kv_idx[h, q, :kv_num[h, q]]:
                bm[h, kb, q // 32] |= np.uint32(1 << (q % 32))
    d = None if docs is None else torch.from_numpy(np.asarray(docs)).to(DEV, torch.int32)
    return ScopeBlockMask(torch.from_numpy(np.ascontiguousarray(kv_num)).to(DEV, torch.int32)[None],
                          torch.from_numpy(np.ascontiguousarray(kv_idx)).to(DEV, torch.int32)[None],
                          torch.from_numpy(bm.view(np.int32)).to(DEV), block_info(d, T, bs, device=DEV),
                          (bs, bs), (T, T), docs=d)


def _run(case, fx, dtype, *, impl, grads, layout="thd"):
    x = C.attn_inputs(case)
    T, bs, K = case["T"], case["bs"], case["K"]
    docs = C.attn_docs(case)
    bm = _mask_from_lists(fx["kv_num"], fx["kv_indices"], T, bs, docs)
    cos_t, sin_t = AO.trig_tables(x["omegas"], T)

    def dev(t, dt=dtype):
        if layout == "thd" and t.dim() == 3 and t.shape[-1] == 64:
            # the reference passes [B,H,T,D] views of [B,T,H,D] storage
            y = t.transpose(0, 1).contiguous().to(DEV, dt).transpose(0, 1)
        else:
            y = t.to(DEV, dt)
        return y.requires_grad_(grads)

    q, k, v = dev(x["q"]), dev(x["k"]), dev(x["v"])
    f32 = lambda t: t.to(DEV, torch.float32).requires_grad_(grads)  # noqa: E731
    cc, cs = f32(x["coeff_cos"]), f32(x["coeff_sin"])
    b0 = f32(x["b0"]) if case["b0"] else None
    sl = f32(x["slope"]) if case["slope"] else None
    dm, wd = f32(x["delta_main"]), f32(x["width"])
    sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=cos_t.to(DEV), sin_tab=sin_t.to(DEV), beta=0.5,
                          b0=b0, slope=sl, delta_main=dm, width=wd, gate=case["gate"], impl=impl)
    out, lse = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12, return_lse=True)
    res = {"out": out[0], "lse": lse[0]}
    if grads:
        g = torch.Generator().manual_seed(99)
        do = torch.randn(q.shape, generator=g)
        out.backward(do.to(DEV, dtype)[None])
        res.update(dq=q.grad, dk=k.grad, dv=v.grad, dcoeff_cos=cc.grad, dcoeff_sin=cs.grad, do=do)
        if b0 is not None:
            res["db0"] = b0.grad
        if sl is not None:
            res["dslope"] = sl.grad
        if case["gate"] != "none":
            res["ddelta_main"], res["dwidth"] = dm.grad, wd.grad
    return res, x, cos_t, sin_t, docs


def _oracle(case, fx, x, cos_t, sin_t, docs, do, impl, dtype):
    """The reference's math in float64 on the inputs the kernel saw (q, k, v
    and dO rounded to the run dtype; in qk_aug mode the augmented dims are
    formed and cast to that dtype exactly as scoped_medium.py:380-421 does)."""
    T, bs = case["T"], case["bs"]
    mask = AO.dense_mask(fx["kv_num"], fx["kv_indices"], T, bs, docs=docs)
    rd = lambda t: t.to(dtype).to(torch.float32)  # noqa: E731
    q, k, v, do = rd(x["q"]), rd(x["k"]), rd(x["v"]), rd(do)
    if impl == "score_mod":
        return AO.score_mod_grads(q, k, v, do, mask, scale=0.12, beta=0.5,
                                  coeff_cos=x["coeff_cos"], coeff_sin=x["coeff_sin"], cos_tab=cos_t, sin_tab=sin_t,
                                  b0=x["b0"] if case["b0"] else None, slope=x["slope"] if case["slope"] else None,
                                  delta_main=x["delta_main"] if case["gate"] != "none" else None,
                                  width=x["width"] if case["gate"] != "none" else None, gate=case["gate"])
    K = case["K"]
    slope = x["slope"] if case["slope"] else None
    qa, ka, va = AO.qk_aug_inputs(q.to(dtype), k.to(dtype), v.to(dtype), x["coeff_cos"], x["coeff_sin"], cos_t, sin_t,
                                  beta=0.5, scale=0.12, slope=slope)
    ref = AO.plain_grads(qa.float(), ka.float(), va.float(), torch.cat([do, torch.zeros(do.shape[0], T, va.shape[-1] - 64)], -1),
                         mask, scale=0.12)
    s = math.sqrt(0.5 / 0.12)
    dqa = ref["dq"][..., 64:]
    c = cos_t.to(torch.float64).transpose(0, 1)[None]
    sn = sin_t.to(torch.float64).transpose(0, 1)[None]
    ref["dcoeff_cos"] = s * (dqa[..., :K] * c + dqa[..., K:2 * K] * sn)
    ref["dcoeff_sin"] = s * (dqa[..., :K] * sn - dqa[..., K:2 * K] * c)
    if slope is not None:
        ref["dslope"] = -s * dqa[..., 2 * K]
    return ref


def _maxabs(a, b):
    return (a.detach().double().cpu() - b.detach().double().cpu()).abs().max().item()


@pytest.mark.parametrize("name", list(C.ATTN_CASES))
def test_fp32_forward_matches_reference_fixture(name):
    case = C.ATTN_CASES[name]
    fx = _load(f"attn_{name}.npz")
    res, *_ = _run(case, fx, torch.float32, impl=case["impl"], grads=False)
    got = res["out"][:, torch.from_numpy(fx["rows"]).to(DEV)].cpu().numpy()
    np.testing.assert_allclose(got, fx["out_rows"], atol=1e-4, rtol=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", list(C.ATTN_CASES))
def test_forward_backward_matches_oracle(name, dtype):
    case = C.ATTN_CASES[name]
    fx = _load(f"attn_{name}.npz")
    res, x, cos_t, sin_t, docs = _run(case, fx, dtype, impl=case["impl"], grads=True)
    ref = _oracle(case, fx, x, cos_t, sin_t, docs, res["do"], case["impl"], dtype)
    tol = TOL[dtype]
    assert _maxabs(res["out"], ref["out"][..., :64]) < tol
    assert _maxabs(res["lse"], ref["lse"]) < tol
    for n in ("dq", "dk", "dv"):
        assert _maxabs(res[n], ref[n][..., :64]) < tol, n
    # gradients of the captured bias tensors: the bound is relative to each
    # tensor's own scale (dslope sums dS * delta over hundreds of positions)
    for n in ("dcoeff_cos", "dcoeff_sin", "db0", "dslope", "ddelta_main", "dwidth"):
        if n in res:
            scale = max(1.0, ref[n].abs().max().item())
            assert _maxabs(res[n], ref[n]) < tol * scale, (n, _maxabs(res[n], ref[n]), scale)


def test_bias_off_and_causal_only():
    """No spectral bias and no documents: plain block-sparse causal attention."""
    case = C.ATTN_CASES["a_scoremod_plain"]
    fx = _load("attn_a_scoremod_plain.npz")
    x = C.attn_inputs(case)
    T, bs = case["T"], case["bs"]
    bm = _mask_from_lists(fx["kv_num"], fx["kv_indices"], T, bs, None)
    q, k, v = (x[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v"))
    out = flex_attention(q[None], k[None], v[None], bm, scale=0.12)
    do = torch.randn_like(out)
    out.backward(do)
    mask = AO.dense_mask(fx["kv_num"], fx["kv_indices"], T, bs, docs=None)
    ref = AO.plain_grads(x["q"], x["k"], x["v"], do[0].cpu(), mask, scale=0.12)
    assert _maxabs(out[0], ref["out"]) < 1e-4
    for n, t in (("dq", q), ("dk", k), ("dv", v)):
        assert _maxabs(t.grad, ref[n]) < 1e-4, n


def test_trig_tables_match_reference_formula():
    w = AO.reference_omegas(8, 4096, 1_000_000)
    c, s = trig_tables(w.to(DEV), 5000)
    rc, rs = AO.trig_tables(w, 5000)
    # cos/sin of the same float32 argument; bf16 rounding may split on rare ties
    assert (c.cpu().float() - rc.float()).abs().max().item() <= 2 ** -8
    assert (c.cpu() != rc).float().mean().item() < 1e-3
    assert (s.cpu() != rs).float().mean().item() < 1e-3


def test_builder_then_attention_end_to_end_config1_shape():
    """Config-1 path end to end at its own size: selection + build on the
    GPU, then fp32 attention with the spectral bias, against the oracle."""
    from scope_b200.synth import CONFIGS, make_inputs
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device="cpu", seed=3)
    H, T, bs = cfg.H, cfg.T, cfg.block_size
    QB = T // bs
    bm = build_mask(H=H, T=T, block_size=bs, M=cfg.M, device=DEV, docs=inp["docs"].to(DEV),
                    sel_logits=inp["logits"].to(DEV), sel_gumbel=inp["gumbel"].to(DEV), sel_tau=cfg.select_tau,
                    budget_rep=inp["budget_rep"].to(DEV), local_blocks=cfg.local_eff, half_blocks=cfg.half_blocks,
                    global_blocks=cfg.global_blocks, budget_blocks=cfg.budget_blocks,
                    budget_is_total=cfg.budget_is_total, budget_temp=cfg.budget_temp)
    cen = MO.select_pointer_blocks(inp["logits"].numpy(), inp["gumbel"].numpy(), M=cfg.M, tau=cfg.select_tau)
    ref_m = MO.build_pointer_blockmask(docs=inp["docs"].numpy(), block_size=bs, M=cfg.M, centres=cen,
                                       budget_rep=inp["budget_rep"].numpy(), local_blocks=cfg.local_eff,
                                       half_blocks=cfg.half_blocks, global_blocks_max=cfg.global_blocks,
                                       budget_blocks=cfg.budget_blocks, budget_is_total=cfg.budget_is_total,
                                       budget_temp=cfg.budget_temp)
    np.testing.assert_array_equal(bm.kv_num_blocks[0].cpu().numpy(), ref_m["kv_num"])
    cos_t, sin_t = AO.trig_tables(inp["omegas"], T)
    q, k, v = (inp[n].to(DEV) for n in ("q", "k", "v"))
    sm = SpectralScoreMod(coeff_cos=inp["coeff_cos"].to(DEV), coeff_sin=inp["coeff_sin"].to(DEV),
                          cos_tab=cos_t.to(DEV), sin_tab=sin_t.to(DEV), beta=0.5, impl="score_mod")
    out = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12)
    mask = AO.dense_mask(ref_m["kv_num"], ref_m["kv_packed"], T, bs, docs=None)
    ro, _ = AO.score_mod_attention(inp["q"], inp["k"], inp["v"], mask, scale=0.12, beta=0.5,
                                   coeff_cos=inp["coeff_cos"], coeff_sin=inp["coeff_sin"], cos_tab=cos_t,
                                   sin_tab=sin_t)
    assert _maxabs(out[0], ro) < 1e-4
