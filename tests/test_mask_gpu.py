"""CUDA pointer block-mask builder vs the reference (golden fixtures) and the
CPU oracle.  Integer outputs must match bit for bit."""
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import mask_oracle as MO
from scope_b200 import PointerBlockMaskBuilder, build_mask

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def _load(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


def _gpu_mask_for_case(case, fx, layout="flex_padded", debug=False, stats=False):
    H, T, bs, M = case["H"], case["T"], case["bs"], case["M"]
    QB = T // bs
    docs = torch.from_numpy(C.mask_docs(case)).to(DEV)
    kw = dict(H=H, T=T, block_size=bs, M=M, device=DEV, docs=docs, local_blocks=case["local"],
              half_blocks=case["half"], half_active=case.get("half_active"), ptr_enabled=case.get("ptr_enabled", True),
              global_blocks=case["glob"], global_active=case.get("glob_active"), radius_mode=case["mode"],
              budget_blocks=case["budget"], budget_is_total=case["total"], budget_temp=case["temp"],
              doc_clamp=case.get("doc_clamp", True), reset_active=bool(case.get("reset_len", 0)),
              reset_len=case.get("reset_len", 0), layout=layout, debug=debug, stats=stats)
    if case.get("gumbel_k"):
        kw.update(peak_gumbel=torch.from_numpy(fx["gumbel_g"]).to(DEV), gumbel_k=case["gumbel_k"],
                  gumbel_tau=case["gumbel_tau"])
    t_rep = (np.arange(QB) + 1) * bs - 1
    if case["source"] == "select":
        logits, g = C.selection_inputs(case)
        brep = C.budget_only(case)[0][:, t_rep]
        return build_mask(sel_logits=torch.from_numpy(logits).to(DEV), sel_gumbel=torch.from_numpy(g).to(DEV),
                          sel_tau=case["sel_tau"], budget_rep=torch.from_numpy(np.ascontiguousarray(brep)).to(DEV),
                          **kw)
    return build_mask(delta_rep=torch.from_numpy(fx["delta_rep"]).to(DEV),
                      budget_rep=torch.from_numpy(fx["budget_rep"]).to(DEV), **kw)


@pytest.mark.parametrize("name", [n for n, c in C.MASK_CASES.items() if not c.get("large")])
def test_builder_matches_reference_fixture(name):
    case = C.MASK_CASES[name]
    fx = _load(f"mask_{name}.npz")
    bm = _gpu_mask_for_case(case, fx)
    kv_num = bm.kv_num_blocks[0].cpu().numpy()
    kv_idx = bm.kv_indices[0].cpu().numpy()
    np.testing.assert_array_equal(kv_num, fx["kv_num"])
    if "kv_indices" in fx:
        np.testing.assert_array_equal(kv_idx, fx["kv_indices"])
    assert C.arr_hash(kv_idx) == str(fx["kv_indices_hash"])
    q_num, q_idx = bm.q_lists(True)
    np.testing.assert_array_equal(q_num[0].cpu().numpy(), fx["q_num"])
    assert C.arr_hash(q_idx[0].cpu().numpy()) == str(fx["q_indices_hash"])


def test_builder_matches_reference_config3_full_size():
    name = "m_c3_full"
    case = C.MASK_CASES[name]
    fx = _load(f"mask_{name}.npz")
    bm = _gpu_mask_for_case(case, fx)
    np.testing.assert_array_equal(bm.kv_num_blocks[0].cpu().numpy(), fx["kv_num"])
    assert C.arr_hash(bm.kv_indices[0].cpu().numpy()) == str(fx["kv_indices_hash"])
    q_num, q_idx = bm.q_lists(True)
    np.testing.assert_array_equal(q_num[0].cpu().numpy(), fx["q_num"])
    assert C.arr_hash(q_idx[0].cpu().numpy()) == str(fx["q_indices_hash"])


def test_builder_class_reference_signature():
    """PointerBlockMaskBuilder.build_pointer_blockmask takes the reference's
    [1,H,T,M] tensors (model/attn_bias.py:623-649) and matches the fixture."""
    name = "m_mean_noclamp"
    case = C.MASK_CASES[name]
    fx = _load(f"mask_{name}.npz")
    delta, budget = C.delta_budget_inputs(case)
    b = PointerBlockMaskBuilder(num_heads=case["H"], M=case["M"], pointer_local_blocks=case["local"],
                                pointer_half_blocks=case["half"], pointer_global_blocks=case["glob"],
                                pointer_budget_blocks=case["budget"], pointer_budget_is_total=case["total"],
                                pointer_budget_temp=case["temp"], pointer_qblock_rep="mean",
                                pointer_doc_clamp=False)
    bm = b.build_pointer_blockmask(docs=torch.from_numpy(C.mask_docs(case)).to(DEV),
                                   delta_star=torch.from_numpy(delta).to(DEV), pi=torch.zeros_like(torch.from_numpy(delta)).to(DEV),
                                   budget_logits=torch.from_numpy(budget).to(DEV), block_size=case["bs"],
                                   layout="flex_padded")
    np.testing.assert_array_equal(bm.kv_num_blocks[0].cpu().numpy(), fx["kv_num"])
    np.testing.assert_array_equal(bm.kv_indices[0].cpu().numpy(), fx["kv_indices"])


def _random_case(rng):
    bs = int(rng.choice([64, 128]))
    QB = int(rng.integers(3, 70))
    M = int(rng.integers(1, 17))
    return dict(H=int(rng.integers(1, 4)), T=QB * bs, bs=bs, M=M, local=int(rng.integers(1, 12)),
                half=int(rng.integers(0, 5)), glob=int(rng.integers(0, 4)), budget=int(rng.integers(0, 40)),
                total=bool(rng.integers(0, 2)), temp=float(rng.choice([0.5, 1.0, 2.0, 0.25])),
                mode=str(rng.choice(["pi", "pi", "fixed"])), ptr_enabled=bool(rng.random() > 0.1),
                doc_clamp=bool(rng.random() > 0.2), reset_len=int(rng.choice([0, 0, 300, 1000])),
                docs=str(rng.choice(["single", "multi"])), seed=int(rng.integers(0, 1 << 30)))


@pytest.mark.parametrize("seed", range(40))
def test_builder_matches_oracle_random(seed):
    rng = np.random.default_rng(1234 + seed)
    case = _random_case(rng)
    H, T, bs, M = case["H"], case["T"], case["bs"], case["M"]
    QB = T // bs
    docs = C.mask_docs(case)
    use_sel = bool(rng.integers(0, 2))
    # the reference's schedule setter caps the active half width at the max
    half_active = int(rng.integers(0, case["half"] + 1)) if case["half"] else None
    glob_active = int(rng.integers(0, case["glob"] + 1)) if case["glob"] else None
    budget_rep = rng.standard_normal((H, QB, M)).astype(np.float32) * 2
    gk = int(rng.integers(0, M + 1)) if rng.random() < 0.4 else 0
    g_peak = MO.gumbel_from_uniform(rng.random((H, QB, M)).astype(np.float32))
    common = dict(docs=docs, block_size=bs, M=M, budget_rep=budget_rep, local_blocks=case["local"],
                  half_blocks=case["half"], half_active=half_active, ptr_enabled=case["ptr_enabled"],
                  global_blocks_max=case["glob"], global_active=glob_active, radius_mode=case["mode"],
                  budget_blocks=case["budget"], budget_is_total=case["total"], budget_temp=case["temp"],
                  gumbel_k=gk, gumbel_tau=0.7, gumbel_g=g_peak if gk else None,
                  doc_clamp=case["doc_clamp"], reset_active=bool(case["reset_len"]), reset_len=case["reset_len"])
    gkw = dict(H=H, T=T, block_size=bs, M=M, device=DEV, docs=torch.from_numpy(docs).to(DEV),
               budget_rep=torch.from_numpy(budget_rep).to(DEV), local_blocks=case["local"], half_blocks=case["half"],
               half_active=half_active, ptr_enabled=case["ptr_enabled"], global_blocks=case["glob"],
               global_active=glob_active, radius_mode=case["mode"], budget_blocks=case["budget"],
               budget_is_total=case["total"], budget_temp=case["temp"], doc_clamp=case["doc_clamp"],
               reset_active=bool(case["reset_len"]), reset_len=case["reset_len"], debug=True, stats=True,
               peak_gumbel=torch.from_numpy(g_peak).to(DEV) if gk else None, gumbel_k=gk, gumbel_tau=0.7)
    if use_sel:
        logits = rng.standard_normal((H, QB, QB)).astype(np.float32)
        g = MO.gumbel_from_uniform(rng.random((H, QB, QB)).astype(np.float32))
        tau = float(rng.choice([0.5, 1.0]))
        cen = MO.select_pointer_blocks(logits, g, M=M, tau=tau)
        ref = MO.build_pointer_blockmask(centres=cen, **common)
        bm = build_mask(sel_logits=torch.from_numpy(logits).to(DEV), sel_gumbel=torch.from_numpy(g).to(DEV),
                        sel_tau=tau, **gkw)
    else:
        delta = (rng.random((H, QB, M)) * T * 1.1 - T * 0.05).astype(np.float32)
        ref = MO.build_pointer_blockmask(delta_rep=delta, **common)
        bm = build_mask(delta_rep=torch.from_numpy(delta).to(DEV), **gkw)
    ok_rows = ref["margin"] > 1e-6
    r_gpu = bm.r_m.cpu().numpy()
    np.testing.assert_array_equal(r_gpu[ok_rows], ref["r_m"][ok_rows])
    np.testing.assert_array_equal(bm.centres.cpu().numpy(), ref["centres"])
    # the integer stages given the kernel's own radii: bit-exact on every row
    L = min(max(1, case["local"]), QB)
    p = case["half"]
    G = min(case["glob"], QB)
    ga = G if glob_active is None else min(max(glob_active, 0), G)
    kvb = MO.window_pieces(ref["centres"], r_gpu, ref["dsp"], ref["dsl"], QB=QB, local_blocks=L, half_blocks=p,
                           global_max=G, global_active=ga)
    num, packed = MO.dedup_pack(kvb, QB)
    np.testing.assert_array_equal(bm.kv_num_blocks[0].cpu().numpy(), num)
    np.testing.assert_array_equal(bm.kv_indices[0].cpu().numpy(), packed)
    q_num, q_idx = MO.transpose_ordered(num, MO.flex_padded(packed, QB))
    gq_num, gq_idx = bm.q_lists(True)
    np.testing.assert_array_equal(gq_num[0].cpu().numpy(), q_num)
    np.testing.assert_array_equal(gq_idx[0].cpu().numpy(), q_idx)
    kvh, prh, exh, zero = MO.pointer_stats(num, r_gpu, max_kv=kvb.shape[-1], half_blocks=p, M=M)
    st = bm.pointer_stats()
    np.testing.assert_array_equal(st["kv_unique_hist"].cpu().numpy(), kvh)
    np.testing.assert_array_equal(st["ptr_radius_hist"].cpu().numpy(), prh)
    np.testing.assert_array_equal(st["ptr_extra_sum_hist"].cpu().numpy(), exh)
    assert int(st["radius0_count"]) == zero


def test_compact_and_padded_layouts_agree():
    case = C.MASK_CASES["m_c3_small"]
    fx = _load("mask_m_c3_small.npz")
    a = _gpu_mask_for_case(case, fx, layout="compact")
    b = _gpu_mask_for_case(case, fx, layout="flex_padded")
    W = a.kv_indices.shape[-1]
    assert torch.equal(a.kv_num_blocks, b.kv_num_blocks)
    assert torch.equal(a.kv_indices, b.kv_indices[..., :W])
    assert torch.equal(a.q_bitmap, b.q_bitmap)


def test_block_info_matches_oracle():
    from scope_b200 import block_info
    rng = np.random.default_rng(5)
    for bs in (64, 128, 256):
        T = bs * 37
        d = np.cumsum(rng.random(T) < 0.004)
        for clamp, rlen in ((True, 0), (False, 0), (True, 700)):
            got = block_info(torch.from_numpy(d).to(DEV), T, bs, device=DEV, doc_clamp=clamp,
                             reset_active=rlen > 0, reset_len=rlen).cpu().numpy()
            dsp, dsl = MO.doc_start_blocks(d, bs, doc_clamp=clamp, reset_active=rlen > 0, reset_len=rlen)
            mn, mx = MO.doc_block_ranges(d, bs)
            np.testing.assert_array_equal(got[0], dsp)
            np.testing.assert_array_equal(got[1], dsl)
            np.testing.assert_array_equal(got[2], mn)
            np.testing.assert_array_equal(got[3], mx)


@pytest.mark.parametrize("M,ties", [(8, False), (16, False), (8, True)])
def test_selection_long_rows_matches_oracle(M, ties):
    """Rows of up to 2,600 candidate blocks (C5 reaches 4,096): the selection
    streams them 1,024 at a time against a running top-M.  Continuous scores
    take that path; heavily tied scores (logits on a 0.5 grid, no noise) send
    rows to the exact fallback.  Centres must equal the oracle's on every row."""
    rng = np.random.default_rng(77 + M + int(ties))
    H, QB, bs = 2, 2600, 128
    if ties:
        logits = (np.round(rng.standard_normal((H, QB, QB)) * 2) / 2).astype(np.float32)
        g = np.zeros((H, QB, QB), np.float32)
    else:
        logits = rng.standard_normal((H, QB, QB)).astype(np.float32)
        g = MO.gumbel_from_uniform(rng.random((H, QB, QB)).astype(np.float32))
    tau = 0.5
    ref = MO.select_pointer_blocks(logits, g, M=M, tau=tau)
    bm = build_mask(H=H, T=QB * bs, block_size=bs, M=M, device=DEV,
                    sel_logits=torch.from_numpy(logits).to(DEV), sel_gumbel=torch.from_numpy(g).to(DEV), sel_tau=tau,
                    budget_rep=torch.from_numpy(rng.standard_normal((H, QB, M)).astype(np.float32)).to(DEV),
                    local_blocks=4, half_blocks=2, global_blocks=1, budget_blocks=4, debug=True)
    np.testing.assert_array_equal(bm.centres.cpu().numpy(), ref)
