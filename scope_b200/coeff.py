"""The coefficient block of SpectralBias.forward on the GPU.

``SpectralCoefficients`` holds what the reference's ``SpectralBias`` holds for
this block (model/attn_bias.py:83-160, 220-227, 290-324): the MLP weights
(shared by the heads or one set per head), the log-spaced omegas and the
knobs; ``forward(q)`` returns what ``SpectralBias.forward`` returns
(model/attn_bias.py:381-622) with the trig tables of ``trig_tables``.  The
MLP and the mixture run in one CUDA kernel (``scope_spectral_coeffs``);
``spectral_coefficients`` is the functional form.

Training mode (``train()``) adds the reference's regularisers to reg_loss
(model/attn_bias.py:480-506): the omega penalty from a per-token term the
kernel writes, the entropy floor, the zero-mean and the delta-edge terms from
the block's outputs, all differentiable.

Backward: when q or a weight requires grad, the outputs carry autograd
history.  The gradient up to the MLP output runs in a CUDA kernel
(``scope_spectral_coeffs_bwd``: the chain rule through the mixture, the
normalisation over frequencies, the softmax and the squashing functions);
with weights shared by the heads (the reference's default) the MLP's own
backward is one tensor-core kernel (``scope_spectral_mlp_bwd``); with one
weight set per head it replays the reference's torch ops on the GPU (two
bf16 linears and a SiLU, model/attn_bias.py:306-324).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .attention import trig_tables
from .mask import _stream

OUT_NAMES = ("coeff_cos", "coeff_sin", "slope", "b0", "delta_star", "pi", "budget_logits", "delta_main", "width")


@dataclass
class CoeffOutputs:
    coeff_cos: Tensor      # [1,H,T,K] f32
    coeff_sin: Tensor      # [1,H,T,K]
    slope: Tensor          # [1,H,T]
    b0: Tensor             # [1,H,T]
    delta_star: Tensor     # [1,H,T,M]
    pi: Tensor             # [1,H,T,M]
    budget_logits: Tensor  # [1,H,T,M]
    delta_main: Tensor     # [1,H,T]
    width: Tensor          # [1,H,T]
    mlp_out: Optional[Tensor] = None   # [1,H,T,n_out] bf16 when requested
    omega_reg: Optional[Tensor] = None  # [1,H,T]: sum_m sum_k w_k^2 a_hat_mk^2, when requested


def _mlp_torch(q: Tensor, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor) -> Tensor:
    """The reference's MLP ops (model/attn_bias.py:306-324) in q's dtype: used to
    carry dL/dy to q and the weights."""
    dt = q.dtype
    if w1.dim() == 2:
        x = torch.nn.functional.silu(torch.nn.functional.linear(q, w1.to(dt), b1.to(dt)))
        return torch.nn.functional.linear(x, w2.to(dt), b2.to(dt))
    x = torch.einsum("bhld,hkd->bhlk", q, w1.to(dt)) + b1.to(dt)[None, :, None, :]
    x = torch.nn.functional.silu(x)
    return torch.einsum("bhlk,hok->bhlo", x, w2.to(dt)) + b2.to(dt)[None, :, None, :]


def coeff_dy(y: Tensor, grads, *, omegas: Tensor, log_omegas: Tensor, M: int, delta_cap: float, logw_min: float,
             logw_max: float, use_slope: bool, subtract_b0: bool, c_scale: float, width_min: float, width_max: float,
             eps: float, padded_bf16: bool = False) -> Tensor:
    """dL/dy from the MLP output y (bf16) and the upstream gradients of
    (coeff_cos, coeff_sin, slope, b0, delta_star, pi, budget_logits,
    delta_main, width[, omega_reg]), any of them None: [1,H,T,n_out] f32, or
    with ``padded_bf16`` the bf16 rows [H*T, n_out rounded up to 16] (zero
    padded) that the MLP backward reads."""
    _, H, T, n_out = y.shape
    K = omegas.numel()
    dev = y.device
    if padded_bf16:
        dy = torch.empty(H * T, (n_out + 15) // 16 * 16, device=dev, dtype=torch.bfloat16)
    else:
        dy = torch.empty(1, H, T, n_out, device=dev, dtype=torch.float32)
    g = [None if t is None else t.to(device=dev, dtype=torch.float32).contiguous() for t in grads]
    g += [None] * (10 - len(g))
    a = _lib.ScopeCoeffBwdArgs()
    a.H, a.T, a.K, a.M, a.use_slope, a.subtract_b0 = H, T, K, M, int(use_slope), int(subtract_b0)
    yc = y.contiguous()
    a.mlp_out = yc.data_ptr()
    names = ("dcoeff_cos", "dcoeff_sin", "dslope", "db0", "ddelta_star", "dpi", "dbudget_logits", "ddelta_main",
             "dwidth", "domega_reg")
    for n, t in zip(names, g):
        setattr(a, n, None if t is None else t.data_ptr())
    om = omegas.to(device=dev, dtype=torch.float32).contiguous()
    lom = log_omegas.to(device=dev, dtype=torch.float32).contiguous()
    a.omegas, a.log_omegas = om.data_ptr(), lom.data_ptr()
    a.delta_cap, a.logw_min, a.logw_max = float(delta_cap), float(logw_min), float(logw_max)
    a.c_scale, a.width_min, a.width_max, a.eps = float(c_scale), float(width_min), float(width_max), float(eps)
    if padded_bf16:
        a.dy_bf16, a.dy_ld = dy.data_ptr(), dy.shape[-1]
    else:
        a.dy = dy.data_ptr()
    a.err_flag = _lib.err_word_ptr(dev)
    _lib.check(_lib.lib().scope_spectral_coeffs_bwd(ctypes.byref(a), _stream(dev)), "scope_spectral_coeffs_bwd")
    return dy


def mlp_backward(q: Tensor, w1: Tensor, b1: Tensor, w2: Tensor, dy: Tensor, needs, n_out: Optional[int] = None) -> tuple:
    """Gradients of the shared-weight MLP (model/attn_bias.py:306-318) from
    dL/dy: (dq, dW1, db1, dW2, db2) in the inputs' dtypes (None where not
    needed), from one launch of ``scope_spectral_mlp_bwd``.  ``dy`` is
    [1,H,T,n_out] f32, or already the bf16 rows [H*T, n_out rounded up to 16]
    (zero padded; give ``n_out``) that ``coeff_dy(padded_bf16=True)`` writes.
    The reference back-propagates dy cast to y's dtype (bf16) through its bf16
    linears; its weight gradients are bf16 results cast to the weights' dtype,
    which the fp32 sums of the kernel are rounded to here."""
    q4 = q if q.dim() == 4 else q[None]
    _, H, T, D = q4.shape
    dev = q4.device
    if dy.dtype == torch.bfloat16 and dy.dim() == 2:
        dyb = dy
    else:
        n_out = dy.shape[-1]
        dyb = torch.zeros(H * T, (n_out + 15) // 16 * 16, device=dev, dtype=torch.bfloat16)
        dyb[:, :n_out] = dy.reshape(H * T, n_out)
    bf = lambda t: t.detach().to(device=dev, dtype=torch.bfloat16).contiguous()  # noqa: E731
    w1b, b1b, w2b = bf(w1), bf(b1), bf(w2)
    q3 = q4[0].detach()
    dq = torch.empty(1, H, T, D, device=dev, dtype=torch.bfloat16)
    f32 = dict(device=dev, dtype=torch.float32)
    dw1, db1, dw2 = torch.zeros(w1.shape, **f32), torch.zeros(b1.shape, **f32), torch.zeros(w2.shape, **f32)
    a = _lib.ScopeCoeffMlpBwdArgs()
    a.H, a.T, a.n_out = H, T, n_out
    a.q, a.q_sh, a.q_st = q3.data_ptr(), q3.stride(0), q3.stride(1)
    a.w1, a.b1, a.w2 = w1b.data_ptr(), b1b.data_ptr(), w2b.data_ptr()
    a.dy, a.dq = dyb.data_ptr(), dq.data_ptr()
    a.dw1, a.db1, a.dw2 = dw1.data_ptr(), db1.data_ptr(), dw2.data_ptr()
    a.err_flag = _lib.err_word_ptr(dev)
    _lib.check(_lib.lib().scope_spectral_mlp_bwd(ctypes.byref(a), _stream(dev)), "scope_spectral_mlp_bwd")
    db2 = dyb[:, :n_out].sum(0, dtype=torch.float32)
    rnd = lambda g, like: g.to(torch.bfloat16).to(like.dtype)  # noqa: E731
    out = (dq if q.dim() == 4 else dq[0], rnd(dw1, w1), rnd(db1, b1), rnd(dw2, w2), rnd(db2, w2))
    return tuple(g if need else None for g, need in zip(out, needs))


class _CoeffFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, w1, b1, w2, b2, kw):
        o = _coeff_forward(q, w1, b1, w2, b2, **kw, return_mlp=True, return_omega=True)
        ctx.mark_non_differentiable(o.mlp_out)
        ctx.save_for_backward(q, w1, b1, w2, b2, o.mlp_out)
        ctx.kw = kw
        return tuple(getattr(o, n) for n in OUT_NAMES) + (o.mlp_out, o.omega_reg)

    @staticmethod
    def backward(ctx, *grads):
        q, w1, b1, w2, b2, y = ctx.saved_tensors
        kw = {k: v for k, v in ctx.kw.items() if k not in ("return_mlp",)}
        if w1.dim() == 2:
            # weights shared by the heads (the reference's default): dL/dy straight into the padded
            # bf16 rows the fused tensor-core MLP backward reads
            dyb = coeff_dy(y, list(grads[:9]) + [grads[10]], **kw, padded_bf16=True)
            return mlp_backward(q, w1, b1, w2, dyb, ctx.needs_input_grad[:5], n_out=y.shape[-1]) + (None,)
        dy = coeff_dy(y, list(grads[:9]) + [grads[10]], **kw)
        # one weight set per head: the reference's MLP ops replayed through autograd
        leaves = [t.detach().requires_grad_(need) for t, need in zip((q, w1, b1, w2, b2), ctx.needs_input_grad[:5])]
        n_out = dy.shape[-1]
        pad = (-n_out) % 16
        with torch.enable_grad():
            q4 = leaves[0] if leaves[0].dim() == 4 else leaves[0][None]
            w2p, b2p = leaves[3], leaves[4]
            if pad:
                # zero output rows change no real row of y, dx or dW2, and give the
                # library GEMMs a multiple-of-16 output width
                w2p = torch.nn.functional.pad(w2p, (0, 0, 0, pad))
                b2p = torch.nn.functional.pad(b2p, (0, pad))
                dy = torch.nn.functional.pad(dy, (0, pad))
            yr = _mlp_torch(q4, leaves[1], leaves[2], w2p, b2p)
            # the reference's y.float() passes its gradient back cast to y's dtype
            torch.autograd.backward(yr, dy.to(yr.dtype))
        return tuple(t.grad if need else None for t, need in zip(leaves, ctx.needs_input_grad[:5])) + (None,)


def spectral_coefficients(q: Tensor, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor, *, omegas: Tensor,
                          log_omegas: Optional[Tensor] = None, M: int, delta_cap: float, logw_min: float,
                          logw_max: float, use_slope: bool = True, subtract_b0: bool = True, c_scale: float = 0.01,
                          width_min: float = 32.0, width_max: float = 256.0, eps: float = 1e-9,
                          return_mlp: bool = False, return_omega: bool = False) -> CoeffOutputs:
    """The coefficient block (see ``_coeff_forward`` for the shapes); with
    autograd history when grad mode is on and q or a weight requires grad."""
    lom = log_omegas if log_omegas is not None else omegas.float().log()
    kw = dict(omegas=omegas, log_omegas=lom, M=M, delta_cap=delta_cap, logw_min=logw_min, logw_max=logw_max,
              use_slope=use_slope, subtract_b0=subtract_b0, c_scale=c_scale, width_min=width_min,
              width_max=width_max, eps=eps)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, w1, b1, w2, b2)):
        outs = _CoeffFn.apply(q, w1, b1, w2, b2, kw)
        return CoeffOutputs(*outs[:9], mlp_out=outs[9].detach() if return_mlp else None,
                            omega_reg=outs[10] if return_omega else None)
    return _coeff_forward(q, w1, b1, w2, b2, **kw, return_mlp=return_mlp, return_omega=return_omega)


def _coeff_forward(q: Tensor, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor, *, omegas: Tensor,
                          log_omegas: Optional[Tensor] = None, M: int, delta_cap: float, logw_min: float,
                          logw_max: float, use_slope: bool = True, subtract_b0: bool = True, c_scale: float = 0.01,
                          width_min: float = 32.0, width_max: float = 256.0, eps: float = 1e-9,
                          return_mlp: bool = False, return_omega: bool = False) -> CoeffOutputs:
    """q [1,H,T,64] or [H,T,64] bf16 (any head/token strides, last dim
    contiguous); w1 [hid,64] / b1 [hid] / w2 [n_out,hid] / b2 [n_out] shared,
    or with a leading H dim per head, in q's dtype (the reference casts its
    weights to q's dtype); n_out = 5M + use_slope; hid = 128."""
    if q.dim() == 4:
        if q.shape[0] != 1:
            raise ValueError("spectral_coefficients: batch must be 1 (as the reference's flex path)")
        q3 = q[0]
    else:
        q3 = q
    if q3.dtype != torch.bfloat16 or not q3.is_cuda:
        raise TypeError("spectral_coefficients: q must be a CUDA bf16 tensor")
    H, T, D = q3.shape
    if q3.stride(2) != 1:
        raise ValueError("spectral_coefficients: q's last dim must be contiguous")
    per_head = w1.dim() == 3
    n_out = 5 * M + (1 if use_slope else 0)
    K = omegas.numel()
    dev = q3.device
    bf = lambda t: t.to(device=dev, dtype=torch.bfloat16).contiguous()
    w1, b1, w2, b2 = (bf(t.detach()) for t in (w1, b1, w2, b2))
    if w2.shape[-2] != n_out or b2.shape[-1] != n_out:
        raise ValueError(f"spectral_coefficients: w2/b2 must have {n_out} outputs (5M + use_slope)")
    om = omegas.to(device=dev, dtype=torch.float32).contiguous()
    lom = (log_omegas if log_omegas is not None else omegas.float().log()).to(device=dev, dtype=torch.float32)
    lom = lom.contiguous()
    f32 = dict(device=dev, dtype=torch.float32)
    out = CoeffOutputs(
        coeff_cos=torch.empty(1, H, T, K, **f32), coeff_sin=torch.empty(1, H, T, K, **f32),
        slope=torch.empty(1, H, T, **f32), b0=torch.empty(1, H, T, **f32),
        delta_star=torch.empty(1, H, T, M, **f32), pi=torch.empty(1, H, T, M, **f32),
        budget_logits=torch.empty(1, H, T, M, **f32), delta_main=torch.empty(1, H, T, **f32),
        width=torch.empty(1, H, T, **f32),
        mlp_out=torch.empty(1, H, T, n_out, device=dev, dtype=torch.bfloat16) if return_mlp else None,
        omega_reg=torch.empty(1, H, T, **f32) if return_omega else None)
    a = _lib.ScopeCoeffArgs()
    a.H, a.T, a.D, a.hidden, a.K, a.M = H, T, D, w1.shape[-2], K, M
    a.use_slope, a.subtract_b0 = int(use_slope), int(subtract_b0)
    q3 = q3.detach()
    a.q, a.q_sh, a.q_st = q3.data_ptr(), q3.stride(0), q3.stride(1)
    a.w_heads = H if per_head else 1
    a.w1, a.b1, a.w2, a.b2 = w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr()
    a.omegas, a.log_omegas = om.data_ptr(), lom.data_ptr()
    a.delta_cap = float(delta_cap)
    a.logw_min, a.logw_max = float(logw_min), float(logw_max)
    a.c_scale, a.width_min, a.width_max, a.eps = float(c_scale), float(width_min), float(width_max), float(eps)
    for n in OUT_NAMES:
        setattr(a, n, getattr(out, n).data_ptr())
    a.mlp_out = out.mlp_out.data_ptr() if return_mlp else None
    a.omega_reg = out.omega_reg.data_ptr() if return_omega else None
    a.err_flag = _lib.err_word_ptr(dev)
    _lib.check(_lib.lib().scope_spectral_coeffs(ctypes.byref(a), _stream(dev)), "scope_spectral_coeffs")
    return out


class SpectralCoefficients:
    """The coefficient block of a SpectralBias: same constructor knobs for the
    block (model/attn_bias.py:83-160), weights initialised as the reference
    initialises them (model/attn_bias.py:290-304) unless loaded with
    ``load_weights``."""

    def __init__(self, *, head_dim: int, num_heads: int, L_train: int, L_max: int = 1_000_000, K: int = 6,
                 M: int = 2, w_min: Optional[float] = None, w_max: Optional[float] = None,
                 share_across_heads: bool = True, use_slope: bool = True, c_scale: float = 0.01,
                 width_min: float = 32.0, width_max: float = 256.0, delta_star_max: Optional[int] = None,
                 subtract_b0: bool = True, eps: float = 1e-9, lambda_omega: float = 1e-5,
                 lambda_zero_mean: float = 1e-4, lambda_entropy: float = 1e-4, pi_entropy_floor_frac: float = 0.25,
                 lambda_delta_edge: float = 0.0, delta_edge_eps: float = 0.0, device="cuda", seed: int = 0):
        if head_dim != 64:
            raise ValueError("SpectralCoefficients: head_dim must be 64")
        self.H, self.K, self.M = num_heads, K, M
        self.use_slope, self.subtract_b0 = use_slope, subtract_b0
        self.c_scale, self.width_min, self.width_max, self.eps = c_scale, width_min, width_max, eps
        w_min = float(w_min) if w_min is not None else 2 * math.pi / L_max
        w_max = float(w_max) if w_max is not None else 2 * math.pi / L_train
        self.omegas = torch.logspace(math.log10(w_min), math.log10(w_max), K, dtype=torch.float32).to(device)
        self.log_omegas = self.omegas.log()
        self.logw_min = float(torch.tensor(math.log(w_min), dtype=torch.float32))
        self.logw_max = float(torch.tensor(math.log(w_max), dtype=torch.float32))
        self.delta_star_max = int(delta_star_max) if delta_star_max is not None else int(L_train - 1)
        self.delta_star_max_active = self.delta_star_max
        hid, n_out = max(128, 2 * head_dim), 5 * M + (1 if use_slope else 0)
        g = torch.Generator().manual_seed(seed)
        Hw = 1 if share_across_heads else num_heads
        b1_ = math.sqrt(3) * 0.5 * head_dim ** -0.5
        self.w1 = ((torch.rand(Hw, hid, head_dim, generator=g) * 2 - 1) * b1_)
        self.b1 = torch.zeros(Hw, hid)
        self.w2 = torch.zeros(Hw, n_out, hid)
        self.b2 = torch.zeros(Hw, n_out)
        self.b2[:, :M] = torch.linspace(-6.0, -4.0, M)   # delta* starts small (the reference's output init)
        self.share = share_across_heads
        self.device = device
        self.training = False
        self.lambda_omega, self.lambda_zero_mean, self.lambda_entropy = lambda_omega, lambda_zero_mean, lambda_entropy
        self.pi_entropy_floor_frac = pi_entropy_floor_frac
        self.lambda_delta_edge, self.delta_edge_eps_active = lambda_delta_edge, delta_edge_eps

    def train(self, mode: bool = True):
        """Training mode adds the regularisers to reg_loss (model/attn_bias.py:480-506)."""
        self.training = bool(mode)
        return self

    def eval(self):
        return self.train(False)

    def _reg_loss(self, o: CoeffOutputs, T: int, delta_cap: float) -> Tensor:
        """The reference's training regularisers (model/attn_bias.py:480-506) from
        the block's outputs; the omega penalty from the kernel's per-token term."""
        dev = o.coeff_cos.device
        reg = torch.zeros((), device=dev, dtype=torch.float32)
        if self.lambda_omega > 0:
            reg = reg + self.lambda_omega * (o.omega_reg.mean() / self.M)
        if self.lambda_entropy > 0:
            ent = -(o.pi * (o.pi + self.eps).log()).sum(dim=-1)
            h_floor = float(self.pi_entropy_floor_frac) * math.log(self.M)
            if h_floor > 0:
                reg = reg + self.lambda_entropy * torch.relu(ent.new_tensor(h_floor) - ent).mean()
        if self.lambda_zero_mean > 0:
            d = torch.arange(T, device=dev, dtype=torch.float32)
            w = self.omegas.to(dev)
            cos_mean = torch.cos(w[:, None] * d[None, :]).mean(dim=-1)
            sin_mean = torch.sin(w[:, None] * d[None, :]).mean(dim=-1)
            mean_b = ((o.coeff_cos * cos_mean).sum(dim=-1) + (o.coeff_sin * sin_mean).sum(dim=-1)
                      + o.slope * (0.5 * float(T - 1)) - o.b0)
            reg = reg + self.lambda_zero_mean * mean_b.mean().square()
        if self.lambda_delta_edge > 0:
            denom = max(delta_cap, 1.0)
            u = (o.delta_star / denom).clamp(min=0.0, max=1.0)
            e = self.delta_edge_eps_active
            edge = torch.relu(e - u) + torch.relu(u - (1.0 - e))
            reg = reg + self.lambda_delta_edge * edge.mean()
        return reg

    def set_delta_star_max_active(self, *, max_tokens: int):
        """As SpectralBias.set_delta_star_max_active (model/attn_bias.py:366-371)."""
        if max_tokens < 0:
            raise ValueError("max_tokens must be >= 0")
        self.delta_star_max_active = min(int(max_tokens), self.delta_star_max)

    def load_weights(self, w1: Tensor, b1: Tensor, w2: Tensor, b2: Tensor):
        """Weights in the reference's layout: shared [hid,D], [hid], [n_out,hid],
        [n_out], or per head with a leading H dim."""
        if w1.dim() == 2:
            w1, b1, w2, b2 = w1[None], b1[None], w2[None], b2[None]
        # kept as given: tensors that require grad receive the block's weight gradients
        self.w1, self.b1, self.w2, self.b2 = w1, b1, w2, b2
        self.share = self.w1.shape[0] == 1

    def forward(self, q: Tensor, *, return_mlp: bool = False):
        """q [1,H,T,64] bf16 -> the outputs of SpectralBias.forward: coeff_cos,
        coeff_sin, slope, b0, delta_star, pi, budget_logits, delta_main, width,
        cos_wD, sin_wD, reg_loss (0)."""
        T = q.shape[-2]
        w = (lambda t: t[0]) if self.share else (lambda t: t)
        cap = float(min(max(self.delta_star_max_active, 0), T - 1))
        o = spectral_coefficients(
            q, w(self.w1), w(self.b1), w(self.w2), w(self.b2), omegas=self.omegas, log_omegas=self.log_omegas,
            M=self.M, delta_cap=cap, logw_min=self.logw_min,
            logw_max=self.logw_max, use_slope=self.use_slope, subtract_b0=self.subtract_b0, c_scale=self.c_scale,
            width_min=self.width_min, width_max=self.width_max, eps=self.eps, return_mlp=return_mlp,
            return_omega=self.training and self.lambda_omega > 0)
        cos_wD, sin_wD = trig_tables(self.omegas, T)
        reg = self._reg_loss(o, T, cap) if self.training else torch.zeros((), device=q.device)
        res = tuple(getattr(o, n) for n in OUT_NAMES) + (cos_wD, sin_wD, reg)
        return (res, o.mlp_out) if return_mlp else res

    __call__ = forward
