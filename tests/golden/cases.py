"""Golden-fixture case definitions (inputs only; no reference import).

``gen_golden.py`` runs the reference on these inputs and stores its outputs
under ``tests/golden/*.npz``; the tests rebuild the same inputs from the same
seeds with the functions here and compare.  Inputs are regenerated rather
than stored to keep the fixtures small; each fixture records a hash of its
inputs so a drift in the generators is caught.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np

# ---------------------------------------------------------------------------
# mask builder cases (model/attn_bias.py:623-874)
# ---------------------------------------------------------------------------
# knobs: constructor knobs of SpectralBias plus call arguments
MASK_CASES = {
    # config-1 shaped: selection of 2 peaks, 1 half block, budget 2 extra
    "m_c1": dict(H=4, T=2048, bs=128, M=2, local=2, half=1, glob=1, budget=2, total=False, temp=1.0,
                 mode="pi", source="select", sel_tau=1.0, docs="single", seed=11),
    # several documents, reset segments, Gumbel peak masking, total budget
    "m_docs_reset_gumbel": dict(H=3, T=64 * 40, bs=64, M=4, local=3, half=2, glob=2, glob_active=1,
                                budget=20, total=True, temp=0.5, mode="pi", source="delta",
                                gumbel_k=2, gumbel_tau=0.7, gumbel_seed=7, docs="multi", reset_len=640,
                                seed=12),
    # fixed radius mode with a schedule cap below the max half-width
    "m_fixed": dict(H=2, T=128 * 24, bs=128, M=3, local=4, half=3, half_active=2, glob=1, budget=0,
                    total=True, temp=1.0, mode="fixed", source="delta", docs="multi", seed=13),
    # pointer mask disabled by the schedule (centres forced to qb, radii 0)
    "m_disabled": dict(H=2, T=128 * 20, bs=128, M=2, local=2, half=2, glob=1, budget=6, total=True,
                       temp=1.0, mode="pi", source="delta", ptr_enabled=False, docs="single", seed=14),
    # qblock_rep="mean" representative, no doc clamp
    "m_mean_noclamp": dict(H=2, T=64 * 32, bs=64, M=3, local=2, half=2, glob=0, budget=9, total=True,
                           temp=2.0, mode="pi", source="delta", rep="mean", doc_clamp=False, docs="multi",
                           seed=15),
    # no half blocks: centres only (configs 2 and 5)
    "m_centres_only": dict(H=4, T=128 * 64, bs=128, M=4, local=8, half=0, glob=1, budget=0, total=False,
                           temp=0.5, mode="pi", source="select", sel_tau=0.5, docs="single", seed=16),
    # MAX_KV >= QB: the packed list is truncated to QB columns
    "m_truncate": dict(H=2, T=128 * 6, bs=128, M=3, local=4, half=2, glob=1, budget=12, total=True,
                       temp=1.0, mode="pi", source="delta", docs="multi", seed=17),
    # config-3 shaped at reduced size
    "m_c3_small": dict(H=2, T=128 * 256, bs=128, M=8, local=8, half=4, glob=1, budget=8, total=False,
                       temp=0.5, mode="pi", source="select", sel_tau=0.5, docs="single", seed=18),
    # config-3 shaped at full size (outputs stored as hashes and counts)
    "m_c3_full": dict(H=16, T=131072, bs=128, M=8, local=8, half=4, glob=1, budget=8, total=False,
                      temp=0.5, mode="pi", source="select", sel_tau=0.5, docs="single", seed=19,
                      large=True),
}


def mask_docs(case):
    T = case["T"]
    if case.get("docs", "single") == "single":
        return np.zeros(T, dtype=np.int64)
    rng = np.random.default_rng(case["seed"] + 1000)
    # a handful of document boundaries, some inside blocks, some on block edges
    nb = max(2, T // 700)
    cuts = np.sort(rng.choice(np.arange(1, T), size=nb, replace=False))
    cuts[0] = (cuts[0] // case["bs"]) * case["bs"] or case["bs"]
    d = np.zeros(T, dtype=np.int64)
    d[cuts] = 1
    return np.cumsum(d)


def selection_inputs(case):
    """Pointer logits ~ N(0,1) [H,QB,QB] and Gumbel g for the selection."""
    H, QB = case["H"], case["T"] // case["bs"]
    rng = np.random.default_rng(case["seed"])
    logits = rng.standard_normal((H, QB, QB), dtype=np.float32)
    u = rng.random((H, QB, QB), dtype=np.float32)
    g = (-np.log(-np.log(u + np.float32(1e-9)) + np.float32(1e-9))).astype(np.float32)
    return logits, g


def delta_budget_inputs(case):
    """Full [1,H,T,M] Δ* and budget logits (float32) as SpectralBias.forward
    would produce (model/attn_bias.py:440,431)."""
    H, T, M = case["H"], case["T"], case["M"]
    rng = np.random.default_rng(case["seed"] + 7)
    delta = (rng.random((1, H, T, M), dtype=np.float32) * np.float32(T * 0.9)).astype(np.float32)
    budget = rng.standard_normal((1, H, T, M), dtype=np.float32)
    return delta, budget


def budget_only(case):
    H, T, M = case["H"], case["T"], case["M"]
    rng = np.random.default_rng(case["seed"] + 7)
    return rng.standard_normal((1, H, T, M), dtype=np.float32)


def input_hash(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def arr_hash(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int32)).tobytes()).hexdigest()


# ---------------------------------------------------------------------------
# attention cases (scoped_medium.py:380-466)
# ---------------------------------------------------------------------------
ATTN_CASES = {
    # score_mod with every term on (b0, slope, softplus gate), several documents
    "a_scoremod_full": dict(H=2, T=768, bs=128, K=8, impl="score_mod", gate="softplus", b0=True,
                            slope=True, docs="multi", mask="m_docs_like", seed=21),
    # config-1 shaped score_mod: no gate, no b0, no slope, single document
    "a_scoremod_plain": dict(H=2, T=768, bs=128, K=8, impl="score_mod", gate="none", b0=False,
                             slope=False, docs="single", mask="m_c1_like", seed=22),
    # relu gate
    "a_scoremod_relu": dict(H=2, T=768, bs=128, K=4, impl="score_mod", gate="relu", b0=True,
                            slope=False, docs="multi", mask="m_docs_like", seed=24),
    # qk_aug (the reference default) with the slope column
    "a_qkaug": dict(H=2, T=768, bs=128, K=8, impl="qk_aug", gate="none", b0=False, slope=True,
                    docs="multi", mask="m_docs_like", seed=23),
}
ATTN_ROWS = 96          # rows of `out` stored per head (evenly spaced), all of lse


def attn_inputs(case):
    """q,k,v [H,T,64] float32, coeff_cos/sin [H,T,K], b0/slope/delta_main/width
    [H,T], omegas [K] (reference logspace with L_train=T, L_max=1e6)."""
    import torch
    H, T, K = case["H"], case["T"], case["K"]
    g = torch.Generator().manual_seed(case["seed"])
    q = torch.randn(H, T, 64, generator=g)
    k = torch.randn(H, T, 64, generator=g)
    v = torch.randn(H, T, 64, generator=g)
    W = torch.randn(64, 2 * K, generator=g) * 0.02
    c = q @ W
    cc, cs = c[..., :K].contiguous(), c[..., K:].contiguous()
    b0 = cc.sum(-1)
    slope = 0.01 * torch.tanh(torch.randn(H, T, generator=g))
    delta_main = torch.rand(H, T, generator=g) * T * 0.5
    width = 32.0 + 224.0 * torch.rand(H, T, generator=g)
    w_min, w_max = 2 * math.pi / 1_000_000, 2 * math.pi / T
    omegas = torch.logspace(math.log10(w_min), math.log10(w_max), K, dtype=torch.float32)
    return dict(q=q, k=k, v=v, coeff_cos=cc, coeff_sin=cs, b0=b0, slope=slope,
                delta_main=delta_main, width=width, omegas=omegas)


def attn_docs(case):
    T = case["T"]
    if case["docs"] == "single":
        return np.zeros(T, dtype=np.int64)
    d = np.zeros(T, dtype=np.int64)
    d[[200, 384, 517]] = 1          # one boundary inside a block, one on an edge
    return np.cumsum(d)


def attn_mask_knobs(case):
    """Builder knobs for the attention case's mask (reference semantics)."""
    if case["mask"] == "m_c1_like":
        return dict(M=2, local=2, half=1, glob=1, budget=2, total=False, temp=1.0)
    return dict(M=2, local=2, half=1, glob=1, budget=4, total=True, temp=0.5)


# ---------------------------------------------------------------------------
# teacher block-mass cases (scoped_medium.py:1760-1819): the reference's own
# code run on float32 inputs (the formula pinned tightly) and on bf16 inputs
# (its training dtype: scores rounded to bf16 by the bf16 matmuls)
# ---------------------------------------------------------------------------
TEACHER_CASES = {
    "t_slope_multi_f32": dict(H=2, T=1024, K=8, slope=True, spectral=True, docs="multi", dtype="float32", seed=31),
    "t_slope_multi_bf16": dict(H=2, T=1024, K=8, slope=True, spectral=True, docs="multi", dtype="bfloat16",
                               seed=31),
    "t_fourier_single_f32": dict(H=2, T=768, K=4, slope=False, spectral=True, docs="single", dtype="float32",
                                 seed=32),
    "t_plain_multi_f32": dict(H=1, T=768, K=4, slope=False, spectral=False, docs="multi", dtype="float32", seed=33),
}


# ---------------------------------------------------------------------------
# SpectralBias coefficient block cases (model/attn_bias.py:306-324, 419-478)
# ---------------------------------------------------------------------------
COEFF_CASES = {
    # the configs' K=16, M=8 with weights shared by the heads, slope and b0 on
    "c_shared": dict(H=2, T=256, K=16, M=8, share=True, use_slope=True, subtract_b0=True,
                     L_train=256, delta_star_max=None, seed=31),
    # one weight set per head, no slope / b0, a schedule cap on delta*
    "c_perhead": dict(H=3, T=128, K=8, M=4, share=False, use_slope=False, subtract_b0=False,
                      L_train=512, delta_star_max=100, seed=32),
    # the reference's constructor defaults K=6, M=2
    "c_k6m2": dict(H=1, T=384, K=6, M=2, share=True, use_slope=True, subtract_b0=True,
                   L_train=1024, delta_star_max=None, seed=33),
}


def coeff_inputs(case):
    """q [1,H,T,64] and the MLP weights as bf16-representable float32 arrays
    (w1 [Hw,128,64], b1 [Hw,128], w2 [Hw,n_out,128], b2 [Hw,n_out]; Hw = 1 when
    shared).  The delta* logits get a negative bias so delta* spreads over the
    cap instead of saturating."""
    import torch
    g = torch.Generator().manual_seed(case["seed"])
    H, T, M = case["H"], case["T"], case["M"]
    Hw = 1 if case["share"] else H
    n_out = 5 * M + (1 if case["use_slope"] else 0)
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(1, H, T, 64, generator=g))
    w1 = bf(torch.randn(Hw, 128, 64, generator=g) * 0.125)
    b1 = bf(torch.randn(Hw, 128, generator=g) * 0.1)
    w2 = bf(torch.randn(Hw, n_out, 128, generator=g) * 0.08)
    b2 = torch.randn(Hw, n_out, generator=g) * 0.5
    b2[:, :M] += torch.linspace(-3.0, 1.0, M)
    b2 = bf(b2)
    return {"q": q.numpy(), "w1": w1.numpy(), "b1": b1.numpy(), "w2": w2.numpy(), "b2": b2.numpy()}


def coeff_upstream(case):
    """Seeded upstream gradients of the block's nine outputs (coeff_cos,
    coeff_sin, slope, b0, delta_star, pi, budget_logits, delta_main, width)."""
    import torch
    g = torch.Generator().manual_seed(case["seed"] + 100)
    H, T, K, M = case["H"], case["T"], case["K"], case["M"]
    shapes = ((1, H, T, K), (1, H, T, K), (1, H, T), (1, H, T), (1, H, T, M), (1, H, T, M), (1, H, T, M),
              (1, H, T), (1, H, T))
    scales = (1.0, 1.0, 10.0, 0.5, 1e-3, 0.5, 0.2, 1e-3, 1e-2)
    return [(torch.randn(*sh, generator=g) * sc).numpy() for sh, sc in zip(shapes, scales)]
