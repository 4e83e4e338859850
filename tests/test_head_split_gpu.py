"""Head sharding on one GPU: the layer run on heads [0, H/2) and [H/2, H) as
two separate calls (what two ranks of a 2-GPU run compute) against the
full-H call.  The per-head inputs are seeded per head, so each half must
reproduce its heads of the full run: masks bit-identical, forward outputs
and lse identical, gradients equal up to the summation order of split kv
rows (fp32 partial sums added in arrival order)."""
import pytest
import torch

from scope_b200 import SpectralScoreMod, device_errors, flex_attention, trig_tables
from scope_b200.synth import BETA, CONFIGS, SCALE, build_config_mask, make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(cfg, heads, head_major):
    x = make_inputs(cfg, device=DEV, seed=3, heads=heads)
    bm = build_config_mask(cfg, x)
    L = {n: x[n].detach().requires_grad_(True) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")}
    ct, st = trig_tables(x["omegas"], cfg.T)
    sm = SpectralScoreMod(coeff_cos=L["coeff_cos"], coeff_sin=L["coeff_sin"], cos_tab=ct, sin_tab=st, beta=BETA,
                          impl="qk_aug")
    out, lse = flex_attention(L["q"][None], L["k"][None], L["v"][None], bm, score_mod=sm, scale=SCALE,
                              return_lse=True, head_major_out=head_major)
    out.backward(x["do"][None])
    g = {n: L[n].grad for n in L}
    return bm, out[0].detach(), lse[0], g


def test_two_head_halves_reproduce_the_full_layer():
    cfg = CONFIGS["c2"]
    H = 4
    device_errors(DEV)
    full = _layer(cfg, slice(0, H), False)
    halves = [_layer(cfg, slice(0, H // 2), True), _layer(cfg, slice(H // 2, H), True)]
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    bm_f, out_f, lse_f, g_f = full
    for i, (bm, out, lse, g) in enumerate(halves):
        hs = slice(i * H // 2, (i + 1) * H // 2)
        assert torch.equal(bm.kv_num_blocks, bm_f.kv_num_blocks[:, hs])
        assert torch.equal(bm.kv_indices, bm_f.kv_indices[:, hs])
        assert torch.equal(bm.q_bitmap, bm_f.q_bitmap[hs])
        assert out.is_contiguous()                      # head-major [H/N, T, D]
        assert torch.equal(out, out_f[hs])
        assert torch.equal(lse, lse_f[hs])
        for n in g:
            err = (g[n].float() - g_f[n][hs].float()).abs().max().item()
            scale = max(1.0, g_f[n][hs].abs().max().item())
            assert err <= 1e-2 * scale, (n, err)
