"""The attention op under torch.compile, as the reference compiles its layer
(scoped_medium.py:37-69): the custom op's registrations (schema, fake
tensor, autograd, AOT dispatch) checked by torch.library.opcheck, and a
compiled function calling flex_attention with the spectral bias giving the
eager results, forward and backward."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(T=512, H=2, K=8, seed=3):
    from scope_b200 import build_mask, trig_tables
    from scope_b200.synth import gumbel_noise, radius_prior_logits
    g = torch.Generator().manual_seed(seed)
    QB = T // 128
    gd = torch.Generator(device=DEV).manual_seed(seed)
    logits = radius_prior_logits(H, QB, generator=gd, device=DEV, mu_blocks=2)
    gum = gumbel_noise((H, QB, QB), generator=gd, device=DEV)
    brep = torch.randn(H, QB, 2, generator=g).to(DEV)
    bm = build_mask(H=H, T=T, block_size=128, M=2, device=DEV, docs=torch.zeros(T, dtype=torch.int32, device=DEV),
                    sel_logits=logits, sel_gumbel=gum, sel_tau=0.5, budget_rep=brep, local_blocks=2, half_blocks=1,
                    global_blocks=1, budget_blocks=2, budget_is_total=False, budget_temp=0.5)
    q, k, v = (torch.randn(1, T, H, 64, generator=g).to(DEV, torch.bfloat16).transpose(1, 2) for _ in range(3))
    cc, cs = (torch.randn(H, T, K, generator=g).to(DEV) * 0.1 for _ in range(2))
    w = torch.tensor([math.pi * 2.0 ** (-i) for i in range(K)], device=DEV)
    ct, st = trig_tables(w, T)
    return bm, q, k, v, cc, cs, ct, st


def test_opcheck_sparse_attn():
    import scope_b200  # noqa: F401  (registers the ops)
    bm, q, k, v, cc, cs, ct, st = _case()
    args = (q[0].detach().requires_grad_(True), k[0].detach().requires_grad_(True), v[0].detach().requires_grad_(True),
            bm.kv_num_blocks[0], bm.kv_indices[0], bm.q_bitmap, bm.block_info, bm.docs, cc, cs, ct, st, None, None,
            None, None, 0.12, 0.5, 2, 0, 0.0, 1.0, 128, 0)
    torch.library.opcheck(torch.ops.scope.sparse_attn.default, args,
                          test_utils=("test_schema", "test_autograd_registration", "test_faketensor",
                                      "test_aot_dispatch_dynamic"))


def test_compiled_layer_matches_eager():
    from scope_b200 import SpectralScoreMod, flex_attention
    bm, q, k, v, cc, cs, ct, st = _case()

    def layer(q, k, v, cc, cs):
        sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, impl="qk_aug")
        out = flex_attention(q, k, v, bm, score_mod=sm, scale=0.12)
        return out.float().square().sum()

    res = {}
    for name, fn in (("eager", layer), ("compiled", torch.compile(layer))):
        leaves = [t.detach().requires_grad_(True) for t in (q, k, v, cc, cs)]
        loss = fn(*leaves)
        loss.backward()
        torch.cuda.synchronize()
        res[name] = [loss.detach()] + [t.grad for t in leaves]
    # the attention op runs the same kernels; Inductor's fused square().sum() may
    # round the loss (and so dout = 2 out) differently from eager in the last bit,
    # and dq and the coefficient gradients are fp32 partial sums added in arrival
    # order (a last-bit difference can move a bf16 result by one step)
    for n, a, b in zip(("loss", "dq", "dk", "dv", "dcc", "dcs"), res["eager"], res["compiled"]):
        tol = 1e-5 if n in ("loss", "dk", "dv") else 1e-2
        torch.testing.assert_close(b.float(), a.float(), rtol=tol, atol=tol)
