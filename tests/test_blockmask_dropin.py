"""The attention drop-in takes a torch BlockMask (the type the reference's
build_pointer_blockmask returns, model/attn_bias.py:851-874) as well as a
ScopeBlockMask: the same lists through ``to_flex()`` give bit-identical
outputs, dK and dV (dQ up to the order its fp32 partials are added in).  Masks the kernels cannot honour (full blocks,
non-square blocks) are rejected before any launch."""
import math

import pytest
import torch
from torch.nn.attention.flex_attention import BlockMask

from scope_b200 import SpectralScoreMod, build_mask, device_errors, flex_attention, trig_tables
from scope_b200.mask import ScopeBlockMask


def _cpu_blockmask(full: bool, bs=(128, 128)):
    H, QB = 1, 4
    kvn = torch.tensor([[[1, 2, 2, 3]]], dtype=torch.int32)
    kvi = torch.zeros(1, H, QB, QB, dtype=torch.int32)
    for qb in range(QB):
        kvi[0, 0, qb, :qb + 1] = torch.arange(qb + 1)
    fn = torch.zeros_like(kvn)
    if full:
        fn[0, 0, 3] = 1
    return BlockMask.from_kv_blocks(kvn, kvi, fn, torch.zeros_like(kvi), BLOCK_SIZE=bs)


def test_blockmask_with_full_blocks_is_rejected():
    with pytest.raises(ValueError, match="full blocks"):
        ScopeBlockMask.from_flex(_cpu_blockmask(True))


def test_blockmask_with_non_square_blocks_is_rejected():
    with pytest.raises(ValueError, match="BLOCK_SIZE"):
        ScopeBlockMask.from_flex(_cpu_blockmask(False, bs=(128, 64)))


@pytest.mark.gpu
@pytest.mark.parametrize("multi_doc", [False, True])
def test_torch_blockmask_gives_identical_results(multi_doc):
    dev = "cuda"
    H, T, K = 2, 4096, 16
    g = torch.Generator().manual_seed(17)
    QB = T // 128
    docs = torch.zeros(T, dtype=torch.int32)
    if multi_doc:
        docs[[1000, 2500]] = 1
        docs = docs.cumsum(0).to(torch.int32)
    logits = torch.randn(H, QB, QB, generator=g).to(dev)
    gum = (-torch.log(-torch.log(torch.empty(H, QB, QB).uniform_(1e-6, 1.0, generator=g)))).to(dev)
    brep = torch.randn(H, QB, 4, generator=g).to(dev)
    bm = build_mask(H=H, T=T, block_size=128, M=4, device=dev, docs=docs.to(dev), sel_logits=logits, sel_gumbel=gum,
                    sel_tau=0.5, budget_rep=brep, local_blocks=4, half_blocks=1, global_blocks=1, budget_blocks=4,
                    budget_is_total=False, budget_temp=0.5, layout="flex_padded")
    tbm = bm.to_flex()
    assert isinstance(tbm, BlockMask)
    q, k, v, do = (torch.randn(1, T, H, 64, generator=g).to(dev, torch.bfloat16).transpose(1, 2) for _ in range(4))
    W = torch.randn(64, 2 * K, generator=g) * 0.02
    c = (q[0].float().cpu() @ W).to(dev)
    w = torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32, device=dev)
    ct, st = trig_tables(w, T)

    def run(mask, **kw):
        ql, kl, vl = (t.detach().requires_grad_(True) for t in (q, k, v))
        cc = c[..., :K].contiguous().requires_grad_(True)
        cs = c[..., K:].contiguous().requires_grad_(True)
        sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, impl="qk_aug")
        out = flex_attention(ql, kl, vl, mask, score_mod=sm, scale=0.12, **kw)
        out.backward(do)
        return [out, ql.grad, kl.grad, vl.grad, cc.grad, cs.grad]

    device_errors(dev)
    a = run(bm)
    b = run(tbm, docs=docs.to(dev))
    torch.cuda.synchronize()
    assert device_errors(dev) == 0
    # out, dk, dv: the same kernels on the same lists, bit for bit; dq and the
    # coefficient gradients are sums of fp32 partials added in arrival order
    for n, x, y in zip(("out", "dq", "dk", "dv", "dcoeff_cos", "dcoeff_sin"), a, b):
        if n in ("out", "dk", "dv"):
            assert torch.equal(x, y), n
        else:
            tol = 1e-2 * max(1.0, x.abs().max().item())
            assert (x.float() - y.float()).abs().max().item() <= tol, n
