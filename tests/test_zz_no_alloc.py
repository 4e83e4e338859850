"""The allocation-free backward entry point (scope_attn_bwd_static_scratch).

Callers that cannot allocate device memory or pass a workspace — a plugin host
that owns all device memory, a binding with no device allocator — use this
variant; its scratch is a
fixed-size device array inside the library.  These tests call it through the
C ABI and compare it with the regular entry point (which gets a workspace
from the caller) on the same inputs, twice in a row, since every call reuses
the same array.  This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

from scope_b200 import SpectralScoreMod, _lib, build_mask, flex_attention, trig_tables
from scope_b200.attention import _attn_args, _new_like_layout, _prepare_aug, BIAS_MODES
from scope_b200.mask import _stream

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(seed=0, T=2048, H=2, K=16):
    g = torch.Generator().manual_seed(seed)
    QB = T // 128
    logits = torch.randn(H, QB, QB, generator=g).to(DEV)
    gum = torch.empty(H, QB, QB).uniform_(1e-6, 1.0, generator=g)
    gum = (-torch.log(-torch.log(gum))).to(DEV)
    brep = torch.randn(H, QB, 4, generator=g).to(DEV)
    bm = build_mask(H=H, T=T, block_size=128, M=4, device=DEV, sel_logits=logits, sel_gumbel=gum, sel_tau=0.5,
                    budget_rep=brep, local_blocks=4, half_blocks=1, global_blocks=1, budget_blocks=4,
                    budget_is_total=False, budget_temp=0.5)
    q, k, v, do = (torch.randn(T, H, 64, generator=g).to(DEV, torch.bfloat16).transpose(0, 1) for _ in range(4))
    W = torch.randn(64, 2 * K, generator=g) * 0.02
    c = (q.float().cpu() @ W).to(DEV)
    cc, cs = c[..., :K].contiguous(), c[..., K:].contiguous()
    w = torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32, device=DEV)
    ct, st = trig_tables(w, T)
    sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=ct, sin_tab=st, beta=0.5, impl="qk_aug")
    out, lse = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12, return_lse=True)
    return dict(bm=bm, q=q, k=k, v=v, do=do, cc=cc, cs=cs, ct=ct, st=st, out=out[0], lse=lse[0])


def _bwd(x, entry: str):
    """One backward through the C ABI; returns its gradients."""
    q, k, v = x["q"], x["k"], x["v"]
    bm = x["bm"]
    q_aug, k_aug = _prepare_aug(q, x["cc"], x["cs"], None, x["ct"], x["st"], 0.5, 0.12, BIAS_MODES["qk_aug"])
    a = _attn_args(q, k, v, x["out"], x["lse"], bm.kv_num_blocks[0], bm.kv_indices[0], bm.q_bitmap,
                   bm.block_info, None, x["cc"], x["cs"], x["ct"], x["st"], None, None, None, None, 0.12, 0.5,
                   BIAS_MODES["qk_aug"], 0, 0.0, 1.0, 128, q_aug, k_aug)
    do = x["do"]
    dq, dk, dv = _new_like_layout(q), _new_like_layout(k), _new_like_layout(v)
    dcc, dcs = torch.empty_like(x["cc"]), torch.empty_like(x["cs"])
    a.dout, a.do_sh, a.do_st = do.data_ptr(), do.stride(0), do.stride(1)
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.dq_sh, a.dq_st, a.dk_sh, a.dk_st, a.dv_sh, a.dv_st = (dq.stride(0), dq.stride(1), dk.stride(0), dk.stride(1),
                                                             dv.stride(0), dv.stride(1))
    a.dcoeff_cos, a.dcoeff_sin = dcc.data_ptr(), dcs.data_ptr()
    L = _lib.lib()
    keep = None
    if entry == "workspace":
        n = L.scope_workspace_bytes(ctypes.byref(a))
        keep = torch.empty(n + 256, dtype=torch.uint8, device=DEV)
        a.workspace = (keep.data_ptr() + 255) // 256 * 256
        a.workspace_bytes = n
        st = L.scope_attn_bwd(ctypes.byref(a), _stream(q.device))
    else:
        a.workspace, a.workspace_bytes = None, 0
        st = L.scope_attn_bwd_static_scratch(ctypes.byref(a), _stream(q.device))
    _lib.check(st, entry)
    torch.cuda.synchronize()
    return {"dq": dq, "dk": dk, "dv": dv, "dcoeff_cos": dcc, "dcoeff_sin": dcs}


def test_static_scratch_backward_matches_workspace_backward_twice():
    x = _case()
    ref = _bwd(x, "workspace")
    for _ in range(2):                      # the array keeps the previous call's contents
        got = _bwd(x, "static")
        for n, t in ref.items():
            err = (got[n].float() - t.float()).abs().max().item()
            assert err < 2e-2, (n, err)
    assert _lib.device_errors(DEV) == 0


def test_static_scratch_rejects_problems_over_its_limit():
    L = _lib.lib()
    a = _lib.ScopeAttnArgs()
    a.H, a.T, a.block_size = 64, 1 << 20, 128   # needs over 2*64*2^20*4 bytes of scratch
    assert L.scope_workspace_bytes(ctypes.byref(a)) > L.scope_static_scratch_bytes()
    assert L.scope_attn_bwd_static_scratch(ctypes.byref(a), None) == -6
    with pytest.raises(ValueError, match="workspace"):
        _lib.check(-6, "scope_attn_bwd_static_scratch")
