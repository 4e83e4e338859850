"""Block size 256 (config C5's mask granularity): the builder works at 256,
the attention kernels run the mask on 128-row tiles (scope_mask_refine).
Checked against the float64 oracle on the dense mask of the 256-block lists,
forward and backward, and the refined lists against a direct restatement."""
import math

import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO
from scope_b200 import SpectralScoreMod, build_mask, device_errors, flex_attention, trig_tables
from scope_b200.synth import gumbel_noise, radius_prior_logits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(T=4096, H=2, K=16, seed=5, multi_doc=True):
    g = torch.Generator().manual_seed(seed)
    QB = T // 256
    docs = torch.zeros(T, dtype=torch.int32)
    if multi_doc:
        d = torch.zeros(T, dtype=torch.int32)
        d[torch.tensor([T // 3 + 77, T // 2 + 5])] = 1
        docs = d.cumsum(0).to(torch.int32)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    logits = radius_prior_logits(H, QB, generator=gd, device=DEV, mu_blocks=2)
    gum = gumbel_noise((H, QB, QB), generator=gd, device=DEV)
    brep = torch.randn(H, QB, 4, generator=g).to(DEV)
    bm = build_mask(H=H, T=T, block_size=256, M=4, device=DEV, docs=docs.to(DEV), sel_logits=logits, sel_gumbel=gum,
                    sel_tau=0.5, budget_rep=brep, local_blocks=4, half_blocks=1, global_blocks=1, budget_blocks=4,
                    budget_is_total=False, budget_temp=0.5)
    x = {n: torch.randn(T, H, 64, generator=g).transpose(0, 1) for n in ("q", "k", "v", "do")}
    W = torch.randn(64, 2 * K, generator=g) * 0.02
    c = x["q"] @ W
    x["cc"], x["cs"] = c[..., :K].contiguous(), c[..., K:].contiguous()
    x["omegas"] = torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32)
    return bm, x, docs


def test_refine_lists_and_bitmap():
    bm, _, _ = _case()
    fine = bm.kernel_tiles(128)
    H, QB = bm.num_heads, bm.num_q_blocks
    kvn, kvi = bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy()
    fn, fi = fine.kv_num_blocks[0].cpu().numpy(), fine.kv_indices[0].cpu().numpy()
    bits = fine.q_bitmap.cpu().numpy().view(np.uint32)
    for h in range(H):
        for qf in range(2 * QB):
            want = [2 * kb + t for kb in kvi[h, qf // 2, :kvn[h, qf // 2]] for t in (0, 1) if 2 * kb + t <= qf]
            assert list(fi[h, qf, :fn[h, qf]]) == want, (h, qf)
            for kf in range(2 * QB):
                assert bool(bits[h, kf, qf >> 5] >> (qf & 31) & 1) == (kf in want)
    assert device_errors(DEV) == 0


def _grads(bm, x, K=16):
    q, k, v = (x[n].transpose(0, 1).contiguous().to(DEV, torch.bfloat16).transpose(0, 1).requires_grad_(True)
               for n in ("q", "k", "v"))
    T = q.shape[1]
    ct, st = trig_tables(x["omegas"].to(DEV), T)
    cc, cs = x["cc"].to(DEV).requires_grad_(True), x["cs"].to(DEV).requires_grad_(True)
    sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, impl="qk_aug")
    out = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12)
    out.backward(x["do"].to(DEV, torch.bfloat16)[None])
    return {"out": out[0], "dq": q.grad, "dk": k.grad, "dv": v.grad, "dcoeff_cos": cc.grad, "dcoeff_sin": cs.grad}


def test_bs256_forward_backward_match_oracle():
    bm, x, docs = _case()
    K = x["cc"].shape[-1]
    device_errors(DEV)
    res = _grads(bm, x)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    T = x["q"].shape[1]
    mask = AO.dense_mask(bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), T, 256,
                         docs=docs.numpy())
    q, k, v = (x[n].to(torch.bfloat16) for n in ("q", "k", "v"))
    ct, st = AO.trig_tables(x["omegas"], T)
    qa, ka, va = AO.qk_aug_inputs(q, k, v, x["cc"], x["cs"], ct, st, beta=0.5, scale=0.12)
    do = x["do"].to(torch.bfloat16).float()
    pad = torch.zeros(do.shape[0], T, va.shape[-1] - 64)
    ref = AO.plain_grads(qa.float(), ka.float(), va.float(), torch.cat([do, pad], -1), mask, scale=0.12)
    s = math.sqrt(0.5 / 0.12)
    dqa = ref["dq"][..., 64:]
    c = ct.to(torch.float64).transpose(0, 1)[None]
    sn = st.to(torch.float64).transpose(0, 1)[None]
    ref["dcoeff_cos"] = s * (dqa[..., :K] * c + dqa[..., K:2 * K] * sn)
    ref["dcoeff_sin"] = s * (dqa[..., :K] * sn - dqa[..., K:2 * K] * c)
    for n in ("out", "dq", "dk", "dv"):
        err = (res[n].double().cpu() - ref[n][..., :64]).abs().max().item()
        assert err < 2e-2, (n, err)
    for n in ("dcoeff_cos", "dcoeff_sin"):
        scale_ = ref[n].abs().max().item()
        err = (res[n].double().cpu() - ref[n]).abs().max().item()
        assert err < 2e-2 * max(1.0, scale_), (n, err, scale_)


def test_c5_full_length_sampled_rows_match_block_sparse_oracle():
    """C5 at full length (T = 2^20, block size 256, 2 heads as each GPU holds
    at 8 GPUs): the forward on a sample of q blocks against the oracle's
    block-sparse restatement of the same rows; the backward runs clean."""
    from scope_b200.synth import CONFIGS, make_inputs
    cfg = CONFIGS["c5"]
    x = make_inputs(cfg, device=DEV, seed=0, heads=slice(0, 2))
    QB = cfg.T // cfg.block_size
    from scope_b200 import PointerBlockMaskBuilder
    b = PointerBlockMaskBuilder(num_heads=2, M=cfg.M, pointer_local_blocks=cfg.local_eff,
                                pointer_half_blocks=cfg.half_blocks, pointer_global_blocks=cfg.global_blocks,
                                pointer_budget_blocks=cfg.budget_blocks, pointer_budget_is_total=cfg.budget_is_total,
                                pointer_budget_temp=cfg.budget_temp)
    bm = b.select_and_build(pointer_logits=x["logits"], gumbel=x["gumbel"], tau=cfg.select_tau, docs=x["docs"],
                            budget_rep=x["budget_rep"], block_size=cfg.block_size)
    assert bm.BLOCK_SIZE[0] == 256 and bm.num_q_blocks == QB
    q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
    ct, st = trig_tables(x["omegas"], cfg.T)
    cc, cs = x["coeff_cos"].detach().requires_grad_(True), x["coeff_sin"].detach().requires_grad_(True)
    sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, impl="qk_aug")
    device_errors(DEV)
    out = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12)
    out.backward(x["do"][None])
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    for t in (out, q.grad, k.grad, v.grad, cc.grad, cs.grad):
        assert torch.isfinite(t).all()
    # sampled rows: the oracle on the fine (128-row) tiles of the same mask
    fine = bm.kernel_tiles(128)
    rows = [0, 1, 777, 4095, 6000, 8191]
    ctc, stc = ct.cpu(), st.cpu()
    qa, ka, va = AO.qk_aug_inputs(x["q"].detach().cpu(), x["k"].detach().cpu(), x["v"].detach().cpu(),
                                  x["coeff_cos"].cpu(), x["coeff_sin"].cpu(), ctc, stc, beta=0.5, scale=0.12)
    ref, _ = AO.block_sparse_forward(qa, ka, va, fine.kv_num_blocks[0].cpu(), fine.kv_indices[0].cpu(),
                                     x["docs"].cpu(), scale=0.12, block_size=128, q_blocks=rows)
    for r in rows:
        sl = slice(r * 128, (r + 1) * 128)
        err = (out[0][:, sl].float().cpu() - ref[:, sl, :64]).abs().max().item()
        assert err < 2e-2, (r, err)
