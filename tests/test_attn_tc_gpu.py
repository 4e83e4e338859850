"""Tensor-core (tcgen05 / TMEM / TMA) attention vs the float64 oracle and vs
the CUDA-core kernel on the same inputs.  bf16 tolerance 2e-2 max-abs."""
import math

import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO
from scope_b200 import SpectralScoreMod, aug_dims, build_mask, device_errors, flex_attention, trig_tables
from scope_b200.mask import ScopeBlockMask, block_info
from scope_b200.synth import radius_prior_logits, gumbel_noise

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(T, H, K, slope, docs_kind, seed, M=4, half=1, local=3, glob=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    QB = T // 128
    docs = torch.zeros(T, dtype=torch.int32)
    if docs_kind == "multi":
        cuts = torch.tensor([T // 5 + 37, T // 2, T // 2 + 300])
        d = torch.zeros(T, dtype=torch.int32)
        d[cuts] = 1
        docs = d.cumsum(0).to(torch.int32)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    logits = radius_prior_logits(H, QB, generator=gd, device=DEV, mu_blocks=4)
    gum = gumbel_noise((H, QB, QB), generator=gd, device=DEV)
    brep = torch.randn(H, QB, M, generator=g).to(DEV)
    bm = build_mask(H=H, T=T, block_size=128, M=M, device=DEV, docs=docs.to(DEV), sel_logits=logits,
                    sel_gumbel=gum, sel_tau=0.5, budget_rep=brep, local_blocks=local, half_blocks=half,
                    global_blocks=glob, budget_blocks=4, budget_is_total=False, budget_temp=0.5)
    qkv = [torch.randn(T, H, 64, generator=g) for _ in range(3)]
    x = {"q": qkv[0].transpose(0, 1), "k": qkv[1].transpose(0, 1), "v": qkv[2].transpose(0, 1)}
    if K:
        W = torch.randn(64, 2 * K, generator=g) * 0.02
        c = x["q"] @ W
        x["coeff_cos"], x["coeff_sin"] = c[..., :K].contiguous(), c[..., K:].contiguous()
        x["slope"] = 0.01 * torch.tanh(torch.randn(H, T, generator=g)) if slope else None
        x["omegas"] = torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32)
    return bm, x, docs


def _run(bm, x, K, cuda_cores=False):
    q, k, v = (x[n].transpose(0, 1).contiguous().to(DEV, torch.bfloat16).transpose(0, 1) for n in ("q", "k", "v"))
    sm = None
    if K:
        ct, st = trig_tables(x["omegas"].to(DEV), q.shape[1])
        sm = SpectralScoreMod(coeff_cos=x["coeff_cos"].to(DEV), coeff_sin=x["coeff_sin"].to(DEV), cos_tab=ct,
                              sin_tab=st, beta=0.5, slope=None if x["slope"] is None else x["slope"].to(DEV),
                              impl="qk_aug")
    return flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12, return_lse=True,
                          cuda_cores=cuda_cores)


def _oracle(bm, x, K, docs):
    T = x["q"].shape[1]
    mask = AO.dense_mask(bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), T, 128,
                         docs=docs.numpy())
    q, k, v = (x[n].to(torch.bfloat16) for n in ("q", "k", "v"))
    if K:
        ct, st = AO.trig_tables(x["omegas"], T)
        qa, ka, va = AO.qk_aug_inputs(q, k, v, x["coeff_cos"], x["coeff_sin"], ct, st, beta=0.5, scale=0.12,
                                      slope=x["slope"])
    else:
        qa, ka, va = q, k, v
    out, lse = AO.attention(qa.float(), ka.float(), va.float(), mask, scale=0.12)
    return out[..., :64], lse


def _maxabs(a, b):
    return (a.detach().double().cpu() - b.detach().double().cpu()).abs().max().item()


@pytest.mark.parametrize("K,slope", [(0, False), (8, False), (8, True), (16, False), (16, True), (32, False)])
@pytest.mark.parametrize("docs_kind", ["single", "multi"])
def test_tc_forward_matches_oracle(K, slope, docs_kind):
    T, H = 2048, 2
    bm, x, docs = _inputs(T, H, K, slope, docs_kind, seed=7 + K)
    if K:
        assert aug_dims(K, slope) in (16, 32, 48, 64)
    device_errors(DEV)
    out, lse = _run(bm, x, K)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    ro, rl = _oracle(bm, x, K, docs)
    assert _maxabs(out[0], ro) < 2e-2
    assert _maxabs(lse[0], rl) < 2e-2
    oc, lc = _run(bm, x, K, cuda_cores=True)
    assert _maxabs(out[0], oc[0]) < 2e-2
    assert _maxabs(lse[0], lc[0]) < 1e-2


@pytest.mark.parametrize("K", [0, 16])
def test_tc_forward_long_lists_match_cuda_cores(K):
    """Deeper pipelines (more kv blocks per query block) at larger T."""
    T, H = 16384, 2
    bm, x, docs = _inputs(T, H, K, False, "multi", seed=3, M=8, half=3, local=8, glob=2)
    assert int(bm.kv_num_blocks.max()) > 16
    out, lse = _run(bm, x, K)
    oc, lc = _run(bm, x, K, cuda_cores=True)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    assert _maxabs(out[0], oc[0]) < 2e-2
    assert _maxabs(lse[0], lc[0]) < 1e-2


def test_tc_forward_empty_rows_and_bad_indices():
    """A row with no kv blocks gives zeros and lse=-inf; a kv index outside
    [0, QB) is skipped (masked) and reported in the device error word."""
    T, H, QB = 1024, 1, 8
    kv_num = np.array([[1, 0, 2, 2, 3, 1, 2, 2]], dtype=np.int32)
    kv_idx = np.zeros((1, QB, 4), dtype=np.int32)
    for qb in range(QB):
        kv_idx[0, qb, :3] = [qb, max(qb - 1, 0), 0]
    kv_idx[0, 6, 1] = 99            # out of range: skipped
    bits = np.zeros((1, QB, 1), dtype=np.uint32)
    for qb in range(QB):
        for kb in kv_idx[0, qb, :kv_num[0, qb]]:
            if 0 <= kb < QB:
                bits[0, kb, 0] |= np.uint32(1 << qb)
    bm = ScopeBlockMask(torch.from_numpy(kv_num)[None].to(DEV), torch.from_numpy(kv_idx)[None].to(DEV),
                        torch.from_numpy(bits.view(np.int32)).to(DEV), block_info(None, T, 128, device=DEV),
                        (128, 128), (T, T))
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(H, T, 64, generator=g).to(DEV, torch.bfloat16) for _ in range(3))
    device_errors(DEV)
    out, lse = flex_attention(q[None], k[None], v[None], bm, scale=0.12, return_lse=True)
    torch.cuda.synchronize()
    assert device_errors(DEV) & 0x1
    assert torch.all(out[0, 0, 128:256] == 0)
    assert torch.all(torch.isneginf(lse[0, 0, 128:256]))
    kv_ok = kv_idx.copy()
    kv_num_ok = kv_num.copy()
    kv_num_ok[0, 6] = 1             # the same row without the skipped entry
    mask = AO.dense_mask(kv_num_ok, kv_ok, T, 128, docs=None)
    ro, rl = AO.attention(q[0:1].float().cpu(), k[0:1].float().cpu(), v[0:1].float().cpu(), mask, scale=0.12)
    rows = torch.cat([torch.arange(0, 128), torch.arange(256, T)])
    assert _maxabs(out[0, 0][rows], ro[0][rows]) < 2e-2


def _grads(bm, x, K, do, cuda_cores=False):
    q, k, v = (x[n].transpose(0, 1).contiguous().to(DEV, torch.bfloat16).transpose(0, 1).requires_grad_(True)
               for n in ("q", "k", "v"))
    sm, leaves = None, {}
    if K:
        ct, st = trig_tables(x["omegas"].to(DEV), q.shape[1])
        cc = x["coeff_cos"].to(DEV).requires_grad_(True)
        cs = x["coeff_sin"].to(DEV).requires_grad_(True)
        sl = None if x["slope"] is None else x["slope"].to(DEV).requires_grad_(True)
        leaves = {"dcoeff_cos": cc, "dcoeff_sin": cs}
        if sl is not None:
            leaves["dslope"] = sl
        sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, slope=sl, impl="qk_aug")
    out = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12, cuda_cores=cuda_cores)
    out.backward(do.to(DEV, torch.bfloat16)[None])
    res = {"out": out[0], "dq": q.grad, "dk": k.grad, "dv": v.grad}
    res.update({n: t.grad for n, t in leaves.items()})
    return res


def _oracle_grads(bm, x, K, docs, do):
    T = x["q"].shape[1]
    mask = AO.dense_mask(bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), T, 128,
                         docs=docs.numpy())
    q, k, v = (x[n].to(torch.bfloat16) for n in ("q", "k", "v"))
    do = do.to(torch.bfloat16).float()
    if not K:
        return AO.plain_grads(q.float(), k.float(), v.float(), do, mask, scale=0.12)
    ct, st = AO.trig_tables(x["omegas"], T)
    qa, ka, va = AO.qk_aug_inputs(q, k, v, x["coeff_cos"], x["coeff_sin"], ct, st, beta=0.5, scale=0.12,
                                  slope=x["slope"])
    pad = torch.zeros(do.shape[0], T, va.shape[-1] - 64)
    ref = AO.plain_grads(qa.float(), ka.float(), va.float(), torch.cat([do, pad], -1), mask, scale=0.12)
    s = math.sqrt(0.5 / 0.12)
    dqa = ref["dq"][..., 64:]
    c = ct.to(torch.float64).transpose(0, 1)[None]
    sn = st.to(torch.float64).transpose(0, 1)[None]
    ref["dcoeff_cos"] = s * (dqa[..., :K] * c + dqa[..., K:2 * K] * sn)
    ref["dcoeff_sin"] = s * (dqa[..., :K] * sn - dqa[..., K:2 * K] * c)
    if x["slope"] is not None:
        ref["dslope"] = -s * dqa[..., 2 * K]
    for n in ("out", "dq", "dk", "dv"):
        ref[n] = ref[n][..., :64]
    return ref


@pytest.mark.parametrize("K,slope", [(0, False), (8, False), (16, False), (16, True), (32, False)])
@pytest.mark.parametrize("docs_kind", ["single", "multi"])
def test_tc_backward_matches_oracle(K, slope, docs_kind):
    T, H = 2048, 2
    bm, x, docs = _inputs(T, H, K, slope, docs_kind, seed=11 + K)
    do = torch.randn(H, T, 64, generator=torch.Generator().manual_seed(5))
    device_errors(DEV)
    res = _grads(bm, x, K, do)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    ref = _oracle_grads(bm, x, K, docs, do)
    for n in ("out", "dq", "dk", "dv"):
        assert _maxabs(res[n], ref[n]) < 2e-2, n
    for n in ("dcoeff_cos", "dcoeff_sin", "dslope"):
        if n in res:
            scale = max(1.0, ref[n].abs().max().item())
            assert _maxabs(res[n], ref[n]) < 2e-2 * scale, (n, _maxabs(res[n], ref[n]), scale)


@pytest.mark.parametrize("K,T,docs_kind", [(0, 8192, "multi"), (16, 16384, "single"), (16, 32768, "multi")])
def test_tc_backward_long_lists_match_cuda_cores(K, T, docs_kind):
    """Long q lists: the global block is seen by every q block of its document,
    so at T >= 16384 its dK/dV list is cut into chunks that meet in the fp32
    slot buffer; compare with the CUDA-core backward on the same inputs."""
    H = 2 if T <= 16384 else 1
    bm, x, docs = _inputs(T, H, K, False, docs_kind, seed=4, M=8, half=3, local=8, glob=2)
    if T >= 16384:
        assert int(bm.q_num_blocks.max()) > 64      # at least one split row
    do = torch.randn(H, T, 64, generator=torch.Generator().manual_seed(6))
    a = _grads(bm, x, K, do)
    b = _grads(bm, x, K, do, cuda_cores=True)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    for n in a:
        scale = max(1.0, b[n].abs().max().item())
        assert _maxabs(a[n], b[n]) < 2e-2 * scale, n
