"""The sampled-row oracle (one block row at a time, full sequence length)
against the dense float64 oracle on small cases: the forward, dq and the
coefficient gradients of sampled query blocks, dk / dv of sampled kv
blocks, with and without the qk_aug dims, slope and documents."""
import math

import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO


def _lists(rng, H, QB, W):
    kv_num = np.zeros((H, QB), np.int32)
    kv_idx = np.zeros((H, QB, W), np.int32)
    for h in range(H):
        for qb in range(QB):
            cand = sorted(set([qb, 0] + list(rng.integers(0, qb + 1, size=3))))
            kv_num[h, qb] = len(cand)
            kv_idx[h, qb, :len(cand)] = cand
    return kv_num, kv_idx


@pytest.mark.parametrize("K,slope,multi_doc", [(0, False, False), (8, False, True), (8, True, True)])
def test_sampled_rows_match_dense_oracle(K, slope, multi_doc):
    rng = np.random.default_rng(3 + K)
    g = torch.Generator().manual_seed(5 + K)
    H, T, bs = 2, 1024, 128
    QB = T // bs
    kv_num, kv_idx = _lists(rng, H, QB, 6)
    docs = None
    if multi_doc:
        d = torch.zeros(T, dtype=torch.int32)
        d[[300, 700]] = 1
        docs = d.cumsum(0).to(torch.int32)
    q, k, v, do = (torch.randn(H, T, 64, generator=g).to(torch.bfloat16).float() for _ in range(4))
    kw = {}
    if K:
        W = torch.randn(64, 2 * K, generator=g) * 0.02
        c = q @ W
        ct, st = AO.trig_tables(AO.config_omegas(K), T)
        kw = dict(beta=0.5, coeff_cos=c[..., :K].contiguous(), coeff_sin=c[..., K:].contiguous(), cos_tab=ct,
                  sin_tab=st, slope=(0.01 * torch.randn(H, T, generator=g)) if slope else None)
    o = AO.SampledRows(q, k, v, do, kv_num, kv_idx, docs, block_size=bs, scale=0.12, **kw)
    mask = AO.dense_mask(kv_num, kv_idx, T, bs, docs=None if docs is None else docs.numpy())
    if K:
        qa, ka, va = AO.qk_aug_inputs(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
                                      kw["coeff_cos"], kw["coeff_sin"], kw["cos_tab"], kw["sin_tab"], beta=0.5,
                                      scale=0.12, slope=kw["slope"])
        pad = torch.zeros(H, T, va.shape[-1] - 64)
        ref = AO.plain_grads(qa.float(), ka.float(), va.float(), torch.cat([do, pad], -1), mask, scale=0.12)
        s = math.sqrt(0.5 / 0.12)
        dqa = ref["dq"][..., 64:]
        cc = kw["cos_tab"].to(torch.float64).T[None]
        sn = kw["sin_tab"].to(torch.float64).T[None]
        ref["dcoeff_cos"] = s * (dqa[..., :K] * cc + dqa[..., K:2 * K] * sn)
        ref["dcoeff_sin"] = s * (dqa[..., :K] * sn - dqa[..., K:2 * K] * cc)
        if slope:
            ref["dslope"] = -s * dqa[..., 2 * K]
    else:
        ref = AO.plain_grads(q, k, v, do, mask, scale=0.12)
    for h, qb in [(0, 0), (1, 3), (0, QB - 1)]:
        got = o.q_block(h, qb)
        sl = slice(qb * bs, (qb + 1) * bs)
        for n in got:
            want = ref[n][h, sl]
            if n in ("out", "dq"):
                want = want[..., :64]
            fin = torch.isfinite(want)
            assert torch.equal(fin, torch.isfinite(got[n])), n
            assert (got[n][fin] - want[fin]).abs().max().item() < 1e-9, n
    for h, kb in [(0, 0), (1, 2), (1, QB - 1)]:
        got = o.kv_block(h, kb)
        sl = slice(kb * bs, (kb + 1) * bs)
        assert got["q_blocks"] >= 1
        for n in ("dk", "dv"):
            assert (got[n] - ref[n][h, sl, :64]).abs().max().item() < 1e-9, n
