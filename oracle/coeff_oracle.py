"""CPU restatement of the SpectralBias coefficient block (TEST INFRASTRUCTURE).

Only the tests and the fixture generator use this module; the product path
is the CUDA kernel behind ``scope_spectral_coeffs``.  It restates, with torch
on the CPU, what model/attn_bias.py computes:

* ``mlp``: the per-query MLP of ``SpectralBias._mlp_forward``
  (model/attn_bias.py:306-324): two linears in the dtype of q (bf16) with a
  SiLU between them, weights shared by the heads or one set per head.
* ``heads``: the rest of ``SpectralBias.forward`` (model/attn_bias.py:419-478)
  from the MLP output y: delta* = sigmoid * cap, mu, sigma, pi = softmax,
  slope = c tanh, the Gaussian weights a_mk over log omega normalised over k,
  coeff_cos/sin = sum_m pi_m a_mk cos/sin(w_k delta*_m), b0, delta_main, width.
* ``reg_loss``: the training regularisers (model/attn_bias.py:480-506).

Pinned against the reference's own outputs by tests/golden/coeff_*.npz.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def hidden(q: torch.Tensor, w1, b1) -> torch.Tensor:
    """silu(linear(q, w1, b1)) in q's dtype: the MLP's hidden activations."""
    dt = q.dtype
    if w1.dim() == 2:
        return F.silu(F.linear(q, w1.to(dt), b1.to(dt)))
    return F.silu(torch.einsum("bhld,hkd->bhlk", q, w1.to(dt)) + b1.to(dt)[None, :, None, :])


def mlp(q: torch.Tensor, w1, b1, w2, b2) -> torch.Tensor:
    """y = linear(silu(linear(q, w1, b1)), w2, b2) in q's dtype.

    q [1,H,T,D]; shared weights w1 [hid,D], b1 [hid], w2 [n_out,hid],
    b2 [n_out], or per head with a leading H dim (model/attn_bias.py:309-324)."""
    dt = q.dtype
    if w1.dim() == 2:
        x = F.silu(F.linear(q, w1.to(dt), b1.to(dt)))
        return F.linear(x, w2.to(dt), b2.to(dt))
    x = torch.einsum("bhld,hkd->bhlk", q, w1.to(dt)) + b1.to(dt)[None, :, None, :]
    x = F.silu(x)
    return torch.einsum("bhlk,hok->bhlo", x, w2.to(dt)) + b2.to(dt)[None, :, None, :]


def heads(y: torch.Tensor, *, M: int, omegas, log_omegas, delta_cap: float, logw_min, logw_max,
          use_slope: bool, subtract_b0: bool, c_scale: float, width_min: float, width_max: float,
          eps: float) -> dict:
    """The outputs of SpectralBias.forward from the float32 MLP output y [...,n_out]."""
    y = y.float()
    d_raw, mu_raw, sg_raw, pi_logit, budget = (y[..., i * M:(i + 1) * M] for i in range(5))
    cap = torch.tensor(float(delta_cap), dtype=torch.float32)
    delta_star = torch.sigmoid(d_raw) * cap
    lo = torch.as_tensor(logw_min, dtype=torch.float32)
    hi = torch.as_tensor(logw_max, dtype=torch.float32)
    mu = lo + (hi - lo) * torch.sigmoid(mu_raw)
    sigma = 0.25 + 1.75 * torch.sigmoid(sg_raw)
    pi = torch.softmax(pi_logit, dim=-1)
    slope = c_scale * torch.tanh(y[..., 5 * M]) if use_slope else torch.zeros_like(y[..., 0])
    lw = torch.as_tensor(log_omegas, dtype=torch.float32)
    w = torch.as_tensor(omegas, dtype=torch.float32)
    # Gaussian bump over log omega per pointer, normalised over the K frequencies
    a = torch.exp(-((lw - mu[..., None]) ** 2) / (2 * (sigma[..., None] ** 2)))
    a = a / (a.sum(dim=-1, keepdim=True) + eps)
    ph = w * delta_star[..., None]
    wgt = pi[..., None] * a
    coeff_cos = (wgt * torch.cos(ph)).sum(dim=-2)
    coeff_sin = (wgt * torch.sin(ph)).sum(dim=-2)
    b0 = coeff_cos.sum(dim=-1) if subtract_b0 else torch.zeros_like(coeff_cos[..., 0])
    delta_main = torch.gather(delta_star, -1, pi.argmax(dim=-1, keepdim=True)).squeeze(-1)
    width = width_min + (width_max - width_min) * torch.sigmoid(mu.mean(dim=-1))
    return dict(coeff_cos=coeff_cos, coeff_sin=coeff_sin, slope=slope, b0=b0, delta_star=delta_star, pi=pi,
                budget_logits=budget, delta_main=delta_main, width=width, mu=mu, sigma=sigma, a_hat=a)


def reg_loss(r: dict, *, omegas, T: int, M: int, delta_cap: float, eps: float, lambda_omega: float = 1e-5,
             lambda_zero_mean: float = 1e-4, lambda_entropy: float = 1e-4, pi_entropy_floor_frac: float = 0.25,
             lambda_delta_edge: float = 0.0, delta_edge_eps: float = 0.0):
    """The training regularisers of SpectralBias.forward (model/attn_bias.py:480-506)
    from the outputs of ``heads``: the omega penalty on the normalised Gaussian
    weights, the entropy floor on pi, the zero-mean bias term and the delta-edge
    term."""
    w = torch.as_tensor(omegas, dtype=torch.float32)
    reg = torch.zeros((), dtype=torch.float32)
    if lambda_omega > 0:
        reg = reg + lambda_omega * ((w ** 2) * r["a_hat"].square()).sum(dim=-1).mean()
    if lambda_entropy > 0:
        ent = -(r["pi"] * (r["pi"] + eps).log()).sum(dim=-1)
        h_floor = float(pi_entropy_floor_frac) * math.log(M)
        if h_floor > 0:
            reg = reg + lambda_entropy * F.relu(ent.new_tensor(h_floor) - ent).mean()
    if lambda_zero_mean > 0:
        d = torch.arange(T, dtype=torch.float32)
        cos_mean = torch.cos(w[:, None] * d[None, :]).mean(dim=-1)
        sin_mean = torch.sin(w[:, None] * d[None, :]).mean(dim=-1)
        mean_b = ((r["coeff_cos"] * cos_mean).sum(-1) + (r["coeff_sin"] * sin_mean).sum(-1)
                  + r["slope"] * (0.5 * float(T - 1)) - r["b0"])
        reg = reg + lambda_zero_mean * mean_b.mean().square()
    if lambda_delta_edge > 0:
        u = (r["delta_star"] / max(float(delta_cap), 1.0)).clamp(min=0.0, max=1.0)
        edge = F.relu(delta_edge_eps - u) + F.relu(u - (1.0 - delta_edge_eps))
        reg = reg + lambda_delta_edge * edge.mean()
    return reg
