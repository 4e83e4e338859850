"""Seeded synthetic inputs for the SCOPE benchmark configurations.

The reference quotes no dataset for this path; the configurations describe
seeded synthetic tensors (q, k, v ~ N(0,1), spectral coefficients from a
seeded linear map of q, pointer logits from a log-normal radius prior plus
N(0,1) noise, Gumbel noise from a seed).  This module produces exactly those,
on any device, from ``torch.Generator`` seeds.

Layout: q/k/v/dO are allocated as [T, H, D] and returned as the [H, T, D]
head-major *views* that the reference passes to flex_attention
(``q.transpose(1, 2)`` of a [B, T, H, D] tensor, scoped_medium.py:459-466),
so the kernels see the same strides the reference path does.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class Config:
    name: str
    H: int
    T: int
    D: int = 64
    block_size: int = 128
    dtype: str = "bf16"
    K: int = 8
    sliding_window_blocks: int = 1
    local_blocks: int = 1
    half_blocks: int = 0
    global_blocks: int = 0
    M: int = 4                      # pointer peaks selected per query block
    select_tau: float = 0.5         # Gumbel top-k temperature of the selection
    budget_blocks: int = 0          # radius budget (reference semantics)
    budget_is_total: bool = False
    budget_temp: float = 0.5
    prior: str = "radius"           # "radius" (log-normal prior + noise) | "normal"
    backward: bool = True
    extra: dict = field(default_factory=dict)

    @property
    def QB(self) -> int:
        return self.T // self.block_size

    @property
    def local_eff(self) -> int:
        # Both bands end at the query block, so their union is the wider one.
        return max(self.sliding_window_blocks, self.local_blocks)


CONFIGS = {
    "c1": Config("c1", H=4, T=2048, dtype="fp32", K=8, sliding_window_blocks=2, local_blocks=1,
                 global_blocks=1, M=2, select_tau=1.0, prior="normal", backward=False),
    "c2": Config("c2", H=16, T=65536, K=8, sliding_window_blocks=8, global_blocks=1, M=4,
                 select_tau=0.5),
    "c3": Config("c3", H=16, T=131072, K=16, sliding_window_blocks=8, local_blocks=2, half_blocks=4,
                 global_blocks=1, M=8, select_tau=0.5, budget_blocks=8, budget_is_total=False,
                 budget_temp=0.5),
    "c5": Config("c5", H=16, T=1048576, block_size=256, K=16, sliding_window_blocks=4, global_blocks=1,
                 M=8, select_tau=0.5),
}

SCALE = 0.12   # CausalSelfAttention.attn_scale, scoped_medium.py:327
BETA = 0.5     # spectral_beta, scoped_medium.py:696


def config_omegas(K: int) -> torch.Tensor:
    """ω_k = π·2^-k, k = 0..K-1 (benchmark configurations)."""
    return torch.tensor([math.pi * 2.0 ** (-k) for k in range(K)], dtype=torch.float32)


def radius_prior_logits(H: int, QB: int, *, generator: torch.Generator, device,
                        sigma: float = 1.5, mu_blocks: int = 8, noise: bool = True) -> torch.Tensor:
    """Pointer logits [H, QB, QB] float32 over candidate blocks kb for each
    query block qb: a log-normal prior over the offset o = qb - kb,
    -(ln(o+1) - ln(mu_blocks))^2 / (2 sigma^2) - ln(o+1), plus N(0,1) noise.
    Entries with kb > qb are not candidates (the selection ignores them)."""
    qb = torch.arange(QB, device=device, dtype=torch.float32)
    o = (qb[:, None] - qb[None, :]).clamp(min=0)
    lo = torch.log1p(o)
    mu = math.log(mu_blocks)
    prior = -((lo - mu) ** 2) / (2 * sigma * sigma) - lo
    out = torch.empty(H, QB, QB, device=device, dtype=torch.float32)
    if noise:
        out.normal_(generator=generator)
    else:
        out.zero_()
    out += prior[None]
    return out


def gumbel_noise(shape, *, generator: torch.Generator, device, eps: float = 1e-9) -> torch.Tensor:
    """g = -log(-log(u + eps) + eps), u ~ U(0,1), float32 (the reference's
    form, model/attn_bias.py:770-771)."""
    u = torch.rand(shape, generator=generator, device=device, dtype=torch.float32)
    return -torch.log(-torch.log(u + eps) + eps)


def make_inputs(cfg: Config, *, device="cuda", seed: int = 0, heads: slice | None = None,
                with_grad_inputs: bool | None = None, docs: torch.Tensor | None = None):
    """All inputs of one layer of the configuration.

    Returns a dict with q, k, v (and dO when the config has a backward),
    coeff_cos / coeff_sin [H,T,K] float32 = q·W_c, q·W_s (W ~ N(0, 0.02)),
    omegas [K], docs [T] int32 (single document unless given), pointer
    logits and Gumbel noise [H,QB,QB] for the selection, budget_rep [H,QB,M]
    ~ N(0,1).  ``heads`` restricts the head-dependent tensors to a slice
    (head-sharded runs draw the full tensors' seeds per head, so every rank
    sees the same values for its heads as a 1-GPU run would).
    """
    dev = torch.device(device)
    dt = torch.float32 if cfg.dtype == "fp32" else torch.bfloat16
    H, T, D, QB = cfg.H, cfg.T, cfg.D, cfg.QB
    hs = heads if heads is not None else slice(0, H)
    hl = list(range(H))[hs]
    need_grad = cfg.backward if with_grad_inputs is None else with_grad_inputs

    def per_head(shape_tail, fn_seed_offset, kind="normal", std=1.0):
        parts = []
        for h in hl:
            g = torch.Generator(device=dev)
            g.manual_seed(seed * 1000003 + fn_seed_offset * 1009 + h)
            x = torch.empty(shape_tail, device=dev, dtype=torch.float32)
            if kind == "normal":
                x.normal_(0.0, std, generator=g)
            parts.append(x)
        return torch.stack(parts, 0)

    def btd(off):
        x = per_head((T, D), off)                       # [h, T, D] fp32
        y = torch.empty(T, len(hl), D, device=dev, dtype=dt)
        y.copy_(x.transpose(0, 1))
        return y.transpose(0, 1)                         # [h, T, D] view, stride_t = h*D

    out = {"q": btd(1), "k": btd(2), "v": btd(3)}
    if need_grad:
        out["do"] = btd(4)
    gw = torch.Generator(device=dev)
    gw.manual_seed(seed * 1000003 + 77)
    W = torch.empty(D, 2 * cfg.K, device=dev, dtype=torch.float32).normal_(0.0, 0.02, generator=gw)
    qf = out["q"].to(torch.float32)
    coeff = torch.matmul(qf, W)                            # [h, T, 2K]
    out["coeff_cos"] = coeff[..., : cfg.K].contiguous()
    out["coeff_sin"] = coeff[..., cfg.K:].contiguous()
    out["omegas"] = config_omegas(cfg.K).to(dev)
    if docs is None:
        docs = torch.zeros(T, dtype=torch.int32, device=dev)
    out["docs"] = docs.to(device=dev, dtype=torch.int32)
    # pointer selection inputs
    lg, gg, br = [], [], []
    for h in hl:
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000003 + 5 * 1009 + h)
        if cfg.prior == "radius":
            lg.append(radius_prior_logits(1, QB, generator=g, device=dev, mu_blocks=max(cfg.local_eff, 1))[0])
        else:
            lg.append(torch.empty(QB, QB, device=dev).normal_(generator=g))
        gg.append(gumbel_noise((QB, QB), generator=g, device=dev))
        br.append(torch.empty(QB, cfg.M, device=dev).normal_(generator=g))
    out["logits"] = torch.stack(lg, 0)
    out["gumbel"] = torch.stack(gg, 0)
    out["budget_rep"] = torch.stack(br, 0)
    return out


def doc_ids_from_tokens(input_seq: torch.Tensor, eod_token_id: int = 50256) -> torch.Tensor:
    """docs = (input_seq == EOD).cumsum(0) (scoped_medium.py:588)."""
    return (input_seq == eod_token_id).cumsum(0).to(torch.int32)


def config_builder(cfg: Config, num_heads: int | None = None, *, debug_stats: bool = False):
    """The pointer block-mask builder with the configuration's knobs."""
    from .mask import PointerBlockMaskBuilder
    return PointerBlockMaskBuilder(
        num_heads=cfg.H if num_heads is None else num_heads, M=cfg.M, pointer_local_blocks=cfg.local_eff,
        pointer_half_blocks=cfg.half_blocks, pointer_global_blocks=cfg.global_blocks,
        pointer_budget_blocks=cfg.budget_blocks, pointer_budget_is_total=cfg.budget_is_total,
        pointer_budget_temp=cfg.budget_temp, debug_stats=debug_stats)


def build_config_mask(cfg: Config, x: dict, builder=None):
    """The configuration's mask from the inputs of ``make_inputs``: Gumbel
    top-M selection over the pointer logits fused with the build."""
    b = builder if builder is not None else config_builder(cfg, x["logits"].shape[0])
    return b.select_and_build(pointer_logits=x["logits"], gumbel=x["gumbel"], tau=cfg.select_tau, docs=x["docs"],
                              budget_rep=x["budget_rep"], block_size=cfg.block_size)
