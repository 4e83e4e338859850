"""The CPU oracle against fixtures produced by the reference itself.

Mask fixtures come from SpectralBias.build_pointer_blockmask
(model/attn_bias.py:623-874); attention fixtures from torch.compile'd CPU
flex_attention called as scoped_medium.py:380-466 calls it.
"""
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import attn_oracle as AO
from oracle import mask_oracle as MO

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


def oracle_for_mask_case(case, fx=None):
    H, T, bs, M = case["H"], case["T"], case["bs"], case["M"]
    QB = T // bs
    docs = C.mask_docs(case)
    kw = dict(docs=docs, block_size=bs, M=M, local_blocks=case["local"], half_blocks=case["half"],
              half_active=case.get("half_active"), ptr_enabled=case.get("ptr_enabled", True),
              global_blocks_max=case["glob"], global_active=case.get("glob_active"),
              radius_mode=case["mode"], budget_blocks=case["budget"], budget_is_total=case["total"],
              budget_temp=case["temp"], doc_clamp=case.get("doc_clamp", True),
              reset_active=bool(case.get("reset_len", 0)), reset_len=case.get("reset_len", 0))
    if case.get("gumbel_k"):
        kw.update(gumbel_k=case["gumbel_k"], gumbel_tau=case["gumbel_tau"], gumbel_g=fx["gumbel_g"])
    t_rep = (np.arange(QB) + 1) * bs - 1
    if case["source"] == "select":
        logits, g = C.selection_inputs(case)
        centres = MO.select_pointer_blocks(logits, g, M=M, tau=case["sel_tau"])
        budget_rep = C.budget_only(case)[0][:, t_rep]
        return MO.build_pointer_blockmask(centres=centres, budget_rep=budget_rep, **kw), (logits, g)
    delta_rep, budget_rep = fx["delta_rep"], fx["budget_rep"]
    return MO.build_pointer_blockmask(delta_rep=delta_rep, budget_rep=budget_rep, **kw), None


@pytest.mark.parametrize("name", [n for n, c in C.MASK_CASES.items() if not c.get("large")])
def test_mask_oracle_matches_reference(name):
    case = C.MASK_CASES[name]
    fx = _load(f"mask_{name}.npz")
    if case["source"] == "select":
        logits, g = C.selection_inputs(case)
        assert C.input_hash(logits, g, C.budget_only(case), C.mask_docs(case)) == str(fx["in_hash"])
    else:
        d, b = C.delta_budget_inputs(case)
        assert C.input_hash(d, b, C.mask_docs(case)) == str(fx["in_hash"])
    out, _ = oracle_for_mask_case(case, fx)
    # no row of these fixtures sits on an ulp tie of the float32 radius allocation
    assert np.all(out["margin"] > 1e-6)
    np.testing.assert_array_equal(out["kv_num"], fx["kv_num"])
    if "kv_indices" in fx:
        np.testing.assert_array_equal(out["kv_indices"], fx["kv_indices"])
        np.testing.assert_array_equal(out["q_indices"], fx["q_indices"])
    else:
        w = fx["kv_indices_prefix"].shape[-1]
        np.testing.assert_array_equal(out["kv_indices"][..., :w], fx["kv_indices_prefix"])
    assert C.arr_hash(out["kv_indices"]) == str(fx["kv_indices_hash"])
    np.testing.assert_array_equal(out["q_num"], fx["q_num"])
    assert C.arr_hash(out["q_indices"]) == str(fx["q_indices_hash"])


@pytest.mark.slow
def test_mask_oracle_matches_reference_config3_full():
    name = "m_c3_full"
    case = C.MASK_CASES[name]
    fx = _load(f"mask_{name}.npz")
    out, (logits, g) = oracle_for_mask_case(case, fx)
    assert C.input_hash(logits, g, C.budget_only(case), C.mask_docs(case)) == str(fx["in_hash"])
    # a few of the 16k rows sit within an ulp or two of a rounding decision;
    # the hashes below show the oracle still decides them as the reference did
    assert (out["margin"] < 1e-6).sum() < 8
    np.testing.assert_array_equal(out["kv_num"], fx["kv_num"])
    assert C.arr_hash(out["kv_indices"]) == str(fx["kv_indices_hash"])
    np.testing.assert_array_equal(out["q_num"], fx["q_num"])
    assert C.arr_hash(out["q_indices"]) == str(fx["q_indices_hash"])


def _attn_oracle(case, fx):
    x = C.attn_inputs(case)
    T, bs = case["T"], case["bs"]
    docs = C.attn_docs(case)
    mask = AO.dense_mask(fx["kv_num"], fx["kv_indices"], T, bs, docs=docs)
    cos_t, sin_t = AO.trig_tables(x["omegas"], T)
    if case["impl"] == "score_mod":
        out, lse = AO.score_mod_attention(
            x["q"], x["k"], x["v"], mask, scale=0.12, beta=0.5, coeff_cos=x["coeff_cos"],
            coeff_sin=x["coeff_sin"], cos_tab=cos_t, sin_tab=sin_t,
            b0=x["b0"] if case["b0"] else None, slope=x["slope"] if case["slope"] else None,
            delta_main=x["delta_main"], width=x["width"], gate=case["gate"])
    else:
        qa, ka, va = AO.qk_aug_inputs(x["q"], x["k"], x["v"], x["coeff_cos"], x["coeff_sin"], cos_t, sin_t,
                                      beta=0.5, scale=0.12, slope=x["slope"] if case["slope"] else None)
        out, lse = AO.attention(qa, ka, va, mask, scale=0.12)
        out = out[..., :64]
    return out, lse


@pytest.mark.parametrize("name", list(C.ATTN_CASES))
def test_attention_oracle_matches_reference_flex(name):
    case = C.ATTN_CASES[name]
    fx = _load(f"attn_{name}.npz")
    x = C.attn_inputs(case)
    assert C.input_hash(*(x[n].numpy() for n in sorted(x))) == str(fx["in_hash"])
    out, _ = _attn_oracle(case, fx)
    got = out[:, torch.from_numpy(fx["rows"])].numpy()
    # fp32 flex vs the float64 restatement
    np.testing.assert_allclose(got, fx["out_rows"], atol=2e-5, rtol=0)


def test_attention_mask_fixture_matches_builder_oracle():
    """The masks used by the attention fixtures are themselves builder outputs."""
    for name, case in C.ATTN_CASES.items():
        fx = _load(f"attn_{name}.npz")
        kn = C.attn_mask_knobs(case)
        out = MO.build_pointer_blockmask(
            docs=C.attn_docs(case), block_size=case["bs"], M=kn["M"], delta_rep=fx["delta_rep"],
            budget_rep=fx["budget_rep"], local_blocks=kn["local"], half_blocks=kn["half"],
            global_blocks_max=kn["glob"], budget_blocks=kn["budget"], budget_is_total=kn["total"],
            budget_temp=kn["temp"])
        np.testing.assert_array_equal(out["kv_num"], fx["kv_num"])
        np.testing.assert_array_equal(out["kv_indices"], fx["kv_indices"])


def test_qk_aug_equals_score_mod_up_to_rounding():
    """qk_aug and score_mod (gate off, b0 off) are the same bias by the
    cos(a-b) identity (scoped_medium.py:380-402); in float64 without the
    bf16 casts they agree closely at these positions."""
    case = dict(C.ATTN_CASES["a_scoremod_plain"])
    fx = _load("attn_a_scoremod_plain.npz")
    x = C.attn_inputs(case)
    T, bs = case["T"], case["bs"]
    mask = AO.dense_mask(fx["kv_num"], fx["kv_indices"], T, bs, docs=C.attn_docs(case))
    cos_t, sin_t = AO.trig_tables(x["omegas"], T)
    a, _ = AO.score_mod_attention(x["q"], x["k"], x["v"], mask, scale=0.12, beta=0.5,
                                  coeff_cos=x["coeff_cos"], coeff_sin=x["coeff_sin"], cos_tab=cos_t, sin_tab=sin_t)
    g = AO.qk_aug_grads(x["q"], x["k"], x["v"], torch.zeros_like(x["q"]), mask, scale=0.12, beta=0.5,
                        coeff_cos=x["coeff_cos"], coeff_sin=x["coeff_sin"], cos_tab=cos_t, sin_tab=sin_t)
    assert (a - g["out"]).abs().max().item() < 5e-3


def test_block_sparse_forward_matches_dense_oracle():
    """The full-length block-sparse CPU forward (the timed CPU baseline) is the
    same function as the dense oracle on a small case."""
    from oracle import attn_oracle as AO
    g = torch.Generator().manual_seed(3)
    H, T, bs = 2, 1024, 128
    QB = T // bs
    q, k = torch.randn(H, T, 96, generator=g), torch.randn(H, T, 96, generator=g)
    v = torch.randn(H, T, 64, generator=g)
    docs = torch.zeros(T, dtype=torch.int32)
    docs[300:] = 1
    docs[700:] = 2
    kvn = torch.zeros(H, QB, dtype=torch.int32)
    kvi = torch.zeros(H, QB, QB, dtype=torch.int32)
    for h in range(H):
        for qb in range(QB):
            bl = sorted({qb, max(0, qb - 1), 0, (qb * (h + 1)) // 3})
            kvn[h, qb] = len(bl)
            kvi[h, qb, :len(bl)] = torch.tensor(bl)
    out, pairs = AO.block_sparse_forward(q, k, v, kvn, kvi, docs, scale=0.12, block_size=bs)
    ref, _ = AO.attention(q, k, v, AO.dense_mask(kvn, kvi, T, bs, docs=docs), scale=0.12)
    assert pairs == int(kvn.sum())
    assert (out.double() - ref).abs().max().item() < 1e-5


@pytest.mark.parametrize("name", ["t_slope_multi_f32", "t_fourier_single_f32", "t_plain_multi_f32",
                                  "t_slope_multi_bf16"])
def test_teacher_mass_oracle_matches_reference(name):
    """The float64 teacher block mass against the reference's teacher block
    (scoped_medium.py:1761-1819) run on the same inputs: float32 inputs within
    2e-4 (its float32 sums), bf16 inputs within 0.05 (its bf16 matmuls round
    every score to bf16 before the softmax; measured 0.011)."""
    f = _load(f"teacher_{name}.npz")
    qp = torch.from_numpy(f["q_pos"]) if "q_pos" in f.files else None
    kp = torch.from_numpy(f["k_pos"]) if "k_pos" in f.files else None
    m = AO.teacher_block_mass(torch.from_numpy(f["q"]), torch.from_numpy(f["k"]), torch.from_numpy(f["docs"]),
                              scale=float(f["scale"]), q_pos=qp, k_pos=kp).numpy()
    bound = 0.05 if name.endswith("bf16") else 2e-4
    assert np.abs(m - f["mass"]).max() < bound
    # every query row's probabilities sum to one
    assert np.abs(m.sum(-1) - 128.0).max() < 1e-9
