"""Dense float64 restatement of the SCOPE attention call (TEST ORACLE ONLY).

Restates what ``flex_attention(q, k, v, block_mask=BlockMask, score_mod=...,
scale=0.12)`` computes at scoped_medium.py:459-466 with the BlockMask built by
model/attn_bias.py:623-874 (every listed block is a *partial* block, so the
document-causal mask_mod of model/attn_bias.py:674-679 applies everywhere),
and the qk_aug variant of scoped_medium.py:380-423.  Everything is evaluated
densely over [H, T, T] in float64 so autograd gives the gradients that flex's
CPU path cannot (it has no backward on CPU).  Sizes are meant for T up to a
few thousand.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def trig_tables(omegas: torch.Tensor, L: int):
    """bf16 cos/sin tables over distances 0..L-1: bf16(cos(fp32(w*d)))
    (model/attn_bias.py:330-339), computed on the CPU in float32."""
    D = torch.arange(L, dtype=torch.float32)
    w = omegas.to(torch.float32)
    ph = w[:, None] * D[None, :]
    return torch.cos(ph).to(torch.bfloat16), torch.sin(ph).to(torch.bfloat16)


def config_omegas(K: int) -> torch.Tensor:
    """ω_k = π·2^-k (the benchmark configurations' frequencies)."""
    return torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32)


def reference_omegas(K: int, L_train: int, L_max: int) -> torch.Tensor:
    """logspace(log10(2π/L_max), log10(2π/L_train), K) (model/attn_bias.py:220-225)."""
    w_min = 2 * math.pi / L_max
    w_max = 2 * math.pi / L_train
    return torch.logspace(math.log10(w_min), math.log10(w_max), K, dtype=torch.float32)


def dense_mask(kv_num, kv_idx, T: int, block_size: int, docs=None,
               full_kv_num=None, full_kv_idx=None, causal: bool = True):
    """Boolean [H, T, T] visibility: listed partial blocks AND mask_mod
    (q >= k and docs[q] == docs[k]); listed full blocks without mask_mod."""
    kv_num = torch.as_tensor(np.asarray(kv_num)).long()
    kv_idx = torch.as_tensor(np.asarray(kv_idx)).long()
    H, QB = kv_num.shape
    KB = T // block_size
    blk = torch.zeros(H, QB, KB, dtype=torch.bool)
    for h in range(H):
        for q in range(QB):
            n = int(kv_num[h, q])
            blk[h, q, kv_idx[h, q, :n]] = True
    i = torch.arange(T)
    elem = torch.ones(T, T, dtype=torch.bool)
    if causal:
        elem = i[:, None] >= i[None, :]
    if docs is not None:
        d = torch.as_tensor(np.asarray(docs)).long()
        elem = elem & (d[:, None] == d[None, :])
    m = blk.repeat_interleave(block_size, 1).repeat_interleave(block_size, 2) & elem[None]
    if full_kv_num is not None:
        fb = torch.zeros(H, QB, KB, dtype=torch.bool)
        fn = torch.as_tensor(np.asarray(full_kv_num)).long()
        fi = torch.as_tensor(np.asarray(full_kv_idx)).long()
        for h in range(H):
            for q in range(QB):
                n = int(fn[h, q])
                fb[h, q, fi[h, q, :n]] = True
        m = m | fb.repeat_interleave(block_size, 1).repeat_interleave(block_size, 2)
    return m


def spectral_bias(T: int, coeff_cos, coeff_sin, cos_tab, sin_tab, *, b0=None, slope=None,
                  delta_main=None, width=None, gate: str = "none", lam: float = 0.2,
                  tau: float = 64.0):
    """bias[h,i,j] of the score_mod closure (scoped_medium.py:425-457), float64.

    Δ = max(i-j, 0); Σ_k A_k cos_tab[k,Δ] + B_k sin_tab[k,Δ] accumulated per
    frequency in order; minus b0; plus slope·Δ; minus λ·gate((|Δ-Δ_main|-width)/τ).
    coeff_* are [H,T,K] (float64 leaves allowed for autograd)."""
    i = torch.arange(T)
    delta = (i[:, None] - i[None, :]).clamp(min=0)
    ct = cos_tab.to(torch.float64)
    st = sin_tab.to(torch.float64)
    K = ct.shape[0]
    bias = torch.zeros(coeff_cos.shape[0], T, T, dtype=torch.float64)
    for k in range(K):
        bias = bias + coeff_cos[:, :, k:k + 1] * ct[k][delta][None] + coeff_sin[:, :, k:k + 1] * st[k][delta][None]
    df = delta.to(torch.float64)[None]
    if b0 is not None:
        bias = bias - b0[:, :, None]
    if slope is not None:
        bias = bias + slope[:, :, None] * df
    if gate != "none" and lam > 0:
        x = ((df - delta_main[:, :, None]).abs() - width[:, :, None]) / tau
        if gate == "relu":
            bias = bias - lam * torch.relu(x)
        else:
            bias = bias - lam * torch.nn.functional.softplus(x)
    return bias


def qk_aug_inputs(q, k, v, coeff_cos, coeff_sin, cos_tab, sin_tab, *, beta: float, scale: float,
                  slope=None, align: int = 16):
    """Augmented Q/K/V of scoped_medium.py:380-423 ([H,T,*] layout, B=1).

    q_pos = [A·cos_t + B·sin_t, A·sin_t − B·cos_t, (−slope)]·s,
    k_pos = [cos_t, sin_t, (pos)]·s with s = sqrt(beta/scale), cast to the
    dtype of q; V padded with zeros; the head dim padded to ``align``."""
    H, T, D = q.shape
    s = math.sqrt(beta / float(scale))
    cos_t = cos_tab.transpose(0, 1).to(torch.float32)
    sin_t = sin_tab.transpose(0, 1).to(torch.float32)
    cb = cos_t[None].expand(H, T, -1)
    sb = sin_t[None].expand(H, T, -1)
    Qcos = coeff_cos * cb + coeff_sin * sb
    Qsin = coeff_cos * sb - coeff_sin * cb
    q_pos = torch.cat([Qcos, Qsin], dim=-1)
    k_pos = torch.cat([cb, sb], dim=-1)
    if slope is not None:
        pos = torch.arange(T, dtype=torch.float32)
        q_pos = torch.cat([q_pos, (-slope).unsqueeze(-1)], dim=-1)
        k_pos = torch.cat([k_pos, pos[None, :, None].expand(H, T, 1)], dim=-1)
    q_pos = (q_pos * s).to(q.dtype)
    k_pos = (k_pos * s).to(q.dtype)
    pad = q_pos.shape[-1]
    qa = torch.cat([q, q_pos], -1)
    ka = torch.cat([k, k_pos], -1)
    va = torch.cat([v, v.new_zeros(H, T, pad)], -1)
    if align > 1:
        da = qa.shape[-1]
        extra = (da + align - 1) // align * align - da
        if extra:
            z = qa.new_zeros(H, T, extra)
            qa, ka, va = torch.cat([qa, z], -1), torch.cat([ka, z], -1), torch.cat([va, z], -1)
    return qa, ka, va


def attention(q, k, v, mask, *, scale: float, bias=None, beta: float = 1.0):
    """Dense masked softmax attention in float64; returns (out [H,T,Dv],
    lse [H,T] natural log).  Rows with no visible key give 0 and -inf."""
    qd, kd, vd = q.to(torch.float64), k.to(torch.float64), v.to(torch.float64)
    s = torch.einsum("htd,hsd->hts", qd, kd) * scale
    if bias is not None:
        s = s + beta * bias
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[..., None])
    p = torch.where(mask, p, torch.zeros_like(p))
    out = torch.einsum("hts,hsd->htd", p, vd)
    return out, lse


def score_mod_attention(q, k, v, mask, *, scale, beta, coeff_cos, coeff_sin, cos_tab, sin_tab,
                        b0=None, slope=None, delta_main=None, width=None, gate="none",
                        lam=0.2, tau=64.0):
    """flex_attention with the spectral score_mod, densely (float64)."""
    T = q.shape[1]
    bias = spectral_bias(T, coeff_cos.to(torch.float64), coeff_sin.to(torch.float64), cos_tab, sin_tab,
                         b0=None if b0 is None else b0.to(torch.float64),
                         slope=None if slope is None else slope.to(torch.float64),
                         delta_main=None if delta_main is None else delta_main.to(torch.float64),
                         width=None if width is None else width.to(torch.float64),
                         gate=gate, lam=lam, tau=tau)
    return attention(q, k, v, mask, scale=scale, bias=bias, beta=beta)


def score_mod_grads(q, k, v, do, mask, *, scale, beta, coeff_cos, coeff_sin, cos_tab, sin_tab,
                    b0=None, slope=None, delta_main=None, width=None, gate="none", lam=0.2, tau=64.0):
    """Forward + float64 autograd backward of the score_mod path.  Returns a
    dict: out, lse, dq, dk, dv, dcoeff_cos, dcoeff_sin (+ db0, dslope,
    ddelta_main, dwidth for the terms that are given)."""
    leaves = {}

    def leaf(name, t):
        if t is None:
            return None
        x = t.detach().to(torch.float64).clone().requires_grad_(True)
        leaves[name] = x
        return x

    ql, kl, vl = leaf("q", q), leaf("k", k), leaf("v", v)
    cc, cs = leaf("coeff_cos", coeff_cos), leaf("coeff_sin", coeff_sin)
    b0l, sl = leaf("b0", b0), leaf("slope", slope)
    dml, wl = leaf("delta_main", delta_main), leaf("width", width)
    T = q.shape[1]
    bias = spectral_bias(T, cc, cs, cos_tab, sin_tab, b0=b0l, slope=sl, delta_main=dml, width=wl,
                         gate=gate, lam=lam, tau=tau)
    out, lse = attention(ql, kl, vl, mask, scale=scale, bias=bias, beta=beta)
    out.backward(do.to(torch.float64))
    res = {"out": out.detach(), "lse": lse.detach()}
    for n, x in leaves.items():
        res["d" + n] = x.grad
    return res


def plain_grads(q, k, v, do, mask, *, scale):
    """Forward + autograd backward of plain masked attention (float64),
    e.g. on qk_aug-augmented inputs."""
    ql = q.detach().to(torch.float64).clone().requires_grad_(True)
    kl = k.detach().to(torch.float64).clone().requires_grad_(True)
    vl = v.detach().to(torch.float64).clone().requires_grad_(True)
    out, lse = attention(ql, kl, vl, mask, scale=scale)
    out.backward(do.to(torch.float64))
    return {"out": out.detach(), "lse": lse.detach(), "dq": ql.grad, "dk": kl.grad, "dv": vl.grad}


def qk_aug_grads(q, k, v, do, mask, *, scale, beta, coeff_cos, coeff_sin, cos_tab, sin_tab, slope=None):
    """qk_aug path end to end in float64 autograd, with the augmented dims
    built in float64 from the given inputs (no dtype cast), returning
    out, lse, dq, dk, dv, dcoeff_cos, dcoeff_sin (+ dslope)."""
    H, T, D = q.shape
    s = math.sqrt(beta / float(scale))
    ql = q.detach().to(torch.float64).clone().requires_grad_(True)
    kl = k.detach().to(torch.float64).clone().requires_grad_(True)
    vl = v.detach().to(torch.float64).clone().requires_grad_(True)
    cc = coeff_cos.detach().to(torch.float64).clone().requires_grad_(True)
    cs = coeff_sin.detach().to(torch.float64).clone().requires_grad_(True)
    sl = None if slope is None else slope.detach().to(torch.float64).clone().requires_grad_(True)
    ct = cos_tab.to(torch.float64).transpose(0, 1)[None].expand(H, T, -1)
    st = sin_tab.to(torch.float64).transpose(0, 1)[None].expand(H, T, -1)
    qp = [cc * ct + cs * st, cc * st - cs * ct]
    kp = [ct, st]
    if sl is not None:
        qp.append(-sl.unsqueeze(-1))
        kp.append(torch.arange(T, dtype=torch.float64)[None, :, None].expand(H, T, 1))
    qa = torch.cat([ql] + [x * s for x in qp], -1)
    ka = torch.cat([kl] + [x * s for x in kp], -1)
    out, lse = attention(qa, ka, vl, mask, scale=scale)
    out.backward(do.to(torch.float64))
    res = {"out": out.detach(), "lse": lse.detach(), "dq": ql.grad, "dk": kl.grad, "dv": vl.grad,
           "dcoeff_cos": cc.grad, "dcoeff_sin": cs.grad}
    if sl is not None:
        res["dslope"] = sl.grad
    return res


def block_sparse_forward(q, k, v, kv_num, kv_idx, docs, *, scale: float, block_size: int = 128,
                         q_blocks=None):
    """Block-sparse forward at full sequence length, fp32 on the CPU: what
    flex_attention computes for a BlockMask whose listed blocks are all partial
    (document-causal mask_mod, model/attn_bias.py:674-679), one q block at a
    time over the gathered keys of its list.  Used as the timed CPU baseline
    where torch's compiled CPU flex kernel cannot be built (Inductor's CPU
    template needs AVX-512 / AVX2 micro-GEMMs); results agree with `attention`.

    q, k: [H, T, Dqk]; v: [H, T, Dv]; kv_num [H, QB]; kv_idx [H, QB, W];
    docs [T].  q_blocks: optional iterable of q block indices (a bounded
    sample); returns (out [H, T, Dv] fp32, zero outside the sample, and the
    number of (q block, kv block) pairs processed)."""
    H, T, _ = q.shape
    bs = block_size
    QB = T // bs
    qf, kf, vf = q.float(), k.float(), v.float()
    docs = docs.long()
    out = torch.zeros(H, T, v.shape[-1], dtype=torch.float32)
    pairs = 0
    rows = range(QB) if q_blocks is None else q_blocks
    for h in range(H):
        for qb in rows:
            n = int(kv_num[h, qb])
            if n == 0:
                continue
            blocks = kv_idx[h, qb, :n].long()
            pairs += n
            cols = (blocks[:, None] * bs + torch.arange(bs)[None, :]).reshape(-1)
            i = torch.arange(qb * bs, (qb + 1) * bs)
            s = (qf[h, i] @ kf[h, cols].T) * scale
            vis = (i[:, None] >= cols[None, :]) & (docs[i][:, None] == docs[cols][None, :])
            s = s.masked_fill(~vis, float("-inf"))
            m = s.amax(dim=-1, keepdim=True)
            m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
            p = torch.exp(s - m)
            l = p.sum(dim=-1, keepdim=True)
            out[h, i] = (p @ vf[h, cols]) / torch.where(l > 0, l, torch.ones_like(l))
    return out, pairs


class SampledRows:
    """Forward and gradients of the qk_aug attention call on a SAMPLE of
    query blocks and kv blocks at full sequence length, in float64 (TEST
    ORACLE ONLY).

    Restates scoped_medium.py:380-423 (the augmented dims, cast to q's dtype
    as the reference casts them) followed by flex_attention
    (scoped_medium.py:422, every listed block partial with the
    document-causal mask_mod of model/attn_bias.py:674-679) and its autograd
    backward, one block row at a time, so sizes like T = 2^17 (16 heads) and
    2^20 stay within seconds of CPU time:

    * ``q_block(h, qb)``: out, lse, dq (first 64 dims) and the gradient of
      the augmented q dims of the 128 query rows of (h, qb), from the kv
      blocks of its list (dq = scale · dS · K over the whole row);
    * ``kv_block(h, kb)``: dk and dv of the kv rows of (h, kb), summed over
      every query block whose list holds kb (each of those rows' lse and
      delta = rowsum(dO ∘ out) from its own full list).

    q, k, v, do: [H, T, 64] (CPU, the bf16 values as float); coeff_cos /
    coeff_sin [H, T, K] float32; cos_tab / sin_tab [K, >= T] bf16; slope
    [H, T] or None; kv_num [H, QB]; kv_idx [H, QB, W]; docs [T] or None."""

    def __init__(self, q, k, v, do, kv_num, kv_idx, docs, *, block_size, scale, beta=None, coeff_cos=None,
                 coeff_sin=None, cos_tab=None, sin_tab=None, slope=None, aug_dtype=torch.bfloat16):
        self.q, self.k, self.v, self.do = q, k, v, do
        self.kv_num = np.asarray(kv_num)
        self.kv_idx = np.asarray(kv_idx)
        self.docs = None if docs is None else torch.as_tensor(np.asarray(docs)).long()
        self.bs, self.scale = int(block_size), float(scale)
        self.cc, self.cs, self.slope = coeff_cos, coeff_sin, slope
        self.ct, self.st = cos_tab, sin_tab
        self.aug = coeff_cos is not None
        self.aug_dtype = aug_dtype
        self.s = math.sqrt(beta / float(scale)) if self.aug else 0.0
        self.K = 0 if not self.aug else coeff_cos.shape[-1]
        self._rowcache = {}

    # augmented rows (scoped_medium.py:380-402), cast like the reference
    def _q_rows(self, h, rows):
        q = self.q[h, rows].to(torch.float64)
        if not self.aug:
            return q
        c = self.ct[:, rows].to(torch.float32).T
        sn = self.st[:, rows].to(torch.float32).T
        A, B = self.cc[h, rows].to(torch.float32), self.cs[h, rows].to(torch.float32)
        parts = [A * c + B * sn, A * sn - B * c]
        if self.slope is not None:
            parts.append((-self.slope[h, rows].to(torch.float32))[:, None])
        qp = (torch.cat(parts, -1) * self.s).to(self.aug_dtype).to(torch.float64)
        return torch.cat([q, qp], -1)

    def _k_rows(self, h, rows):
        k = self.k[h, rows].to(torch.float64)
        if not self.aug:
            return k
        c = self.ct[:, rows].to(torch.float32).T
        sn = self.st[:, rows].to(torch.float32).T
        parts = [c, sn]
        if self.slope is not None:
            parts.append(rows.to(torch.float32)[:, None])
        kp = (torch.cat(parts, -1) * self.s).to(self.aug_dtype).to(torch.float64)
        return torch.cat([k, kp], -1)

    def _row(self, h, qb):
        """P, dS, the gathered columns and out / lse of one query block."""
        key = (h, qb)
        if key in self._rowcache:
            return self._rowcache[key]
        bs = self.bs
        n = int(self.kv_num[h, qb])
        i = torch.arange(qb * bs, (qb + 1) * bs)
        blocks = torch.as_tensor(self.kv_idx[h, qb, :n].astype(np.int64))
        cols = (blocks[:, None] * bs + torch.arange(bs)[None, :]).reshape(-1)
        qa = self._q_rows(h, i)
        ka = self._k_rows(h, cols)
        s = (qa @ ka.T) * self.scale
        vis = i[:, None] >= cols[None, :]
        if self.docs is not None:
            vis = vis & (self.docs[i][:, None] == self.docs[cols][None, :])
        s = s.masked_fill(~vis, float("-inf"))
        lse = torch.logsumexp(s, -1)
        fin = torch.isfinite(lse)
        p = torch.exp(s - torch.where(fin, lse, torch.zeros_like(lse))[:, None])
        p = torch.where(vis, p, torch.zeros_like(p))
        vv = self.v[h, cols].to(torch.float64)
        out = p @ vv
        do = self.do[h, i].to(torch.float64)
        dp = do @ vv.T
        delta = (do * out).sum(-1)
        ds = p * (dp - delta[:, None])
        res = dict(i=i, cols=cols, p=p, ds=ds, out=out, lse=lse, qa=qa, ka=ka, do=do)
        self._rowcache[key] = res
        return res

    def q_block(self, h, qb):
        r = self._row(h, qb)
        dqa = (r["ds"] @ r["ka"]) * self.scale
        res = {"out": r["out"], "lse": r["lse"], "dq": dqa[:, :64]}
        if self.aug:
            K, s = self.K, self.s
            dg = dqa[:, 64:]
            i = r["i"]
            c = self.ct[:, i].to(torch.float64).T
            sn = self.st[:, i].to(torch.float64).T
            res["dcoeff_cos"] = s * (dg[:, :K] * c + dg[:, K:2 * K] * sn)
            res["dcoeff_sin"] = s * (dg[:, :K] * sn - dg[:, K:2 * K] * c)
            if self.slope is not None:
                res["dslope"] = -s * dg[:, 2 * K]
        return res

    def q_list(self, h, kb):
        n = self.kv_num[h]
        W = self.kv_idx.shape[-1]
        listed = (self.kv_idx[h] == kb) & (np.arange(W)[None, :] < n[:, None])
        return np.nonzero(listed.any(1))[0]

    def kv_block(self, h, kb):
        bs = self.bs
        dk = torch.zeros(bs, 64, dtype=torch.float64)
        dv = torch.zeros(bs, 64, dtype=torch.float64)
        qbs = self.q_list(h, kb)
        for qb in qbs:
            r = self._row(h, int(qb))
            sel = (r["cols"] >= kb * bs) & (r["cols"] < (kb + 1) * bs)
            p, ds = r["p"][:, sel], r["ds"][:, sel]
            dv += p.T @ r["do"]
            dk += (ds.T @ r["qa"][:, :64]) * self.scale
            self._rowcache.pop((h, int(qb)), None)
        return {"dk": dk, "dv": dv, "q_blocks": len(qbs)}


def teacher_block_mass(q, k, docs, *, scale: float, q_pos=None, k_pos=None, block_size: int = 128):
    """Teacher block mass of scoped_medium.py:1793-1819, in float64: for each
    head and query block, the dense document-causal softmax over all keys of
    (q k^T + q_pos k_pos^T) * scale, each row's probabilities summed over the
    keys of every kv block and over the block's query rows.

    q, k [H, T, D] and q_pos [H, T, P], k_pos [H, T, P] or [T, P] (the
    reference's augmented dims, already scaled by sqrt(beta / scale) and cast
    to q's dtype), docs [T].  Returns mass [H, QB, QB] (float64); entry
    [h, qb, kb] is zero above the diagonal and sums to block_size over kb."""
    H, T, _ = q.shape
    bs = block_size
    QB = T // bs
    qd, kd = q.double(), k.double()
    docs = torch.as_tensor(docs).long()
    if q_pos is not None:
        qp = q_pos.double()
        kp = k_pos.double()
        if kp.dim() == 2:
            kp = kp[None].expand(H, T, -1)
    kblk = torch.arange(T) // bs
    mass = torch.zeros(H, QB, QB, dtype=torch.float64)
    for qb in range(QB):
        i = torch.arange(qb * bs, (qb + 1) * bs)
        s = torch.einsum("hid,hjd->hij", qd[:, i], kd) * scale
        if q_pos is not None:
            s = s + torch.einsum("hid,hjd->hij", qp[:, i], kp) * scale
        vis = (i[:, None] >= torch.arange(T)[None, :]) & (docs[i][:, None] == docs[None, :])
        s = s.masked_fill(~vis[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        colsum = p.sum(dim=1)                                    # [H, T]
        mass[:, qb].index_add_(1, kblk, colsum)
    return mass
