"""Attention parity at the sizes the benchmark runs: configurations C3
(H = 16, T = 2^17, K = 16, the bench's own seeded inputs and mask), C2
(H = 16, T = 2^16, K = 8, several documents) and C5 (T = 2^20, block size
256, the 2 heads one GPU holds at 8 GPUs).  The tensor-core kernels run the
whole layer; the float64 oracle (oracle.attn_oracle.SampledRows) evaluates
the same call on sampled block rows: forward out / lse, dq and the
coefficient gradients of sampled query blocks (the first, the last, one with
the longest kv list, document boundaries), dk / dv of sampled kv blocks
(the global block 0, whose q list spans the whole sequence and is cut into
chunks that meet in the fp32 slot buffer, and others).  bf16 tolerance:
2e-2 max-abs (coefficient gradients: relative to their scale)."""
import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO
from scope_b200 import SpectralScoreMod, device_errors, flex_attention, trig_tables
from scope_b200.synth import BETA, CONFIGS, SCALE, build_config_mask, make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def _docs(T, cuts):
    d = torch.zeros(T, dtype=torch.int32)
    d[torch.tensor(cuts)] = 1
    return d.cumsum(0).to(torch.int32)


def _run_layer(cfg, x, heads):
    bm = build_config_mask(cfg, x)
    leaves = {n: x[n].detach().requires_grad_(True) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")}
    ct, st = trig_tables(x["omegas"], cfg.T)
    sm = SpectralScoreMod(coeff_cos=leaves["coeff_cos"], coeff_sin=leaves["coeff_sin"], cos_tab=ct, sin_tab=st,
                          beta=BETA, impl="qk_aug")
    device_errors(DEV)
    out, lse = flex_attention(leaves["q"][None], leaves["k"][None], leaves["v"][None], bm, score_mod=sm,
                              scale=SCALE, return_lse=True)
    out.backward(x["do"][None])
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    res = {"out": out[0].detach(), "lse": lse[0].detach(), "dq": leaves["q"].grad, "dk": leaves["k"].grad,
           "dv": leaves["v"].grad, "dcoeff_cos": leaves["coeff_cos"].grad, "dcoeff_sin": leaves["coeff_sin"].grad}
    oracle = AO.SampledRows(x["q"].cpu(), x["k"].cpu(), x["v"].cpu(), x["do"].cpu(),
                            bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), x["docs"].cpu(),
                            block_size=cfg.block_size, scale=SCALE, beta=BETA, coeff_cos=x["coeff_cos"].cpu(),
                            coeff_sin=x["coeff_sin"].cpu(), cos_tab=ct.cpu(), sin_tab=st.cpu())
    return bm, res, oracle


def _check_q_blocks(res, oracle, picks, bs):
    for h, qb in picks:
        want = oracle.q_block(h, qb)
        sl = slice(qb * bs, (qb + 1) * bs)
        for n in ("out", "lse", "dq"):
            got = res[n][h, sl].double().cpu()
            err = (got - want[n]).abs().max().item()
            assert err < TOL, (n, h, qb, err)
        for n in ("dcoeff_cos", "dcoeff_sin"):
            got = res[n][h, sl].double().cpu()
            sc = max(1.0, want[n].abs().max().item())
            err = (got - want[n]).abs().max().item()
            assert err < TOL * sc, (n, h, qb, err, sc)


def _check_kv_blocks(res, oracle, picks, bs, min_q=0):
    for h, kb in picks:
        want = oracle.kv_block(h, kb)
        assert want["q_blocks"] >= min_q or kb != 0
        sl = slice(kb * bs, (kb + 1) * bs)
        for n in ("dk", "dv"):
            got = res[n][h, sl].double().cpu()
            err = (got - want[n]).abs().max().item()
            assert err < TOL, (n, h, kb, want["q_blocks"], err)


def _longest(bm, h):
    return int(bm.kv_num_blocks[0, h].argmax().item())


def _busiest_kv(bm, h, skip=(0,)):
    qn = bm.q_num_blocks[0, h].clone()
    for s in skip:
        qn[s] = -1
    return int(qn.argmax().item())


def test_c3_full_size_sampled_rows_match_oracle():
    cfg = CONFIGS["c3"]
    x = make_inputs(cfg, device=DEV, seed=0)
    bm, res, oracle = _run_layer(cfg, x, cfg.H)
    QB = cfg.QB
    assert int(bm.q_num_blocks[0, 0, 0]) > 64           # block 0's list is split into chunks
    _check_q_blocks(res, oracle, [(0, 0), (3, QB - 1), (7, _longest(bm, 7)), (15, 613), (11, 512)], 128)
    _check_kv_blocks(res, oracle, [(0, 0), (5, QB - 1), (9, _busiest_kv(bm, 9)), (14, 300)], 128, min_q=QB)


def test_c2_full_size_with_documents_sampled_rows_match_oracle():
    cfg = CONFIGS["c2"]
    T = cfg.T
    cuts = [T // 3 + 77, T // 2, T // 2 + 128 * 5, 2 * T // 3 + 5]
    x = make_inputs(cfg, device=DEV, seed=1, docs=_docs(T, cuts))
    bm, res, oracle = _run_layer(cfg, x, cfg.H)
    QB = cfg.QB
    straddle = [c // 128 for c in cuts]
    picks = [(0, 0), (15, QB - 1), (4, _longest(bm, 4))] + [(h, qb) for h, qb in zip((1, 6, 9, 13), straddle)]
    _check_q_blocks(res, oracle, picks, 128)
    kvp = [(0, 0), (8, straddle[0]), (12, straddle[2] + 1), (3, _busiest_kv(bm, 3))]
    _check_kv_blocks(res, oracle, kvp, 128)


def test_c5_full_length_backward_sampled_rows_match_oracle():
    """C5 (T = 2^20, block size 256; 2 heads): the oracle runs on the
    builder's 256-row lists directly, independent of the refinement the
    kernels use."""
    cfg = CONFIGS["c5"]
    x = make_inputs(cfg, device=DEV, seed=0, heads=slice(0, 2))
    bm, res, oracle = _run_layer(cfg, x, 2)
    QB = cfg.QB
    _check_q_blocks(res, oracle, [(0, 0), (1, QB - 1), (0, _longest(bm, 0)), (1, 1777)], 256)
    _check_kv_blocks(res, oracle, [(0, 2000), (1, QB - 1), (1, _busiest_kv(bm, 1))], 256)
