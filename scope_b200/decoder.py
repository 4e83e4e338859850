"""A SCOPE decoder built on this package's ops (configuration C4), trained
data-parallel.

The block structure follows the reference's GPT (scoped_medium.py:310-622):
merged QKV weights with QK RMS-norm and rotary embeddings, value embeddings
mixed into v on the first and last three layers, the x0 residual mix and the
U-net skip connections, a relu^2 MLP, logits soft-capped as
30 * sigmoid(logits / 7.5) and a cross entropy over shifted targets.  Each
layer's attention is the reference's SCOPE attention
(CausalSelfAttention.forward, scoped_medium.py:334-479) on this package:

  q (pre-rotary) -> SpectralCoefficients (the coefficient block, one CUDA kernel)
                 -> PointerBlockMaskBuilder.build_pointer_blockmask (delta*, pi,
                    budget logits of the representative rows; one CUDA kernel)
                 -> flex_attention(q, k, v, mask, SpectralScoreMod(qk_aug))
                    (tcgen05 forward and backward)

Differences from the reference, by design of configuration C4: 24 layers of
16 heads x 64 head dims (the reference: 16 x 8 x 128), attention on every
layer (the reference skips layer 7), one pointer mask per layer built from
that layer's coefficients, a bf16 lm_head (the reference's fp8 lm_head is not
part of this path) and AdamW for every parameter (the reference's Muon is not
part of this path).

Data parallelism: ``BucketedAllReduce`` keeps the gradients as views of a few
flat buckets and all-reduces each bucket (NCCL, average) as soon as the
backward has produced all of its gradients, so the exchange overlaps the rest
of the backward -- the reference all-reduces parameter by parameter after the
backward (scoped_medium.py:2523-2524).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from .attention import SpectralScoreMod, flex_attention
from .coeff import SpectralCoefficients
from .mask import EOD_TOKEN_ID, PointerBlockMaskBuilder


def norm(x: Tensor) -> Tensor:
    return F.rms_norm(x, (x.size(-1),))


class CastedLinear(nn.Linear):
    """fp32 weights used in the activations' dtype (scoped_medium.py:268-285)."""

    def __init__(self, in_features: int, out_features: int):
        super().__init__(in_features, out_features, bias=False)
        bound = (3 ** 0.5) * 0.5 * in_features ** -0.5
        with torch.no_grad():
            self.weight.uniform_(-bound, bound)

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight.type_as(x))


class Rotary(nn.Module):
    """Rotary embedding over half of the head dims with the reference's
    frequencies (scoped_medium.py:288-308): 1024^(-k/(D/4-1)) for D/4
    frequencies, then D/4 zero frequencies."""

    def __init__(self, dim: int, max_seq_len: int):
        super().__init__()
        freqs = (1 / 1024) ** torch.linspace(0, 1, steps=dim // 4, dtype=torch.float32)
        freqs = torch.cat([freqs, freqs.new_zeros(dim // 4)])
        t = torch.arange(max_seq_len, dtype=torch.float32)
        theta = torch.outer(t, freqs)
        self.cos = nn.Buffer(theta.cos(), persistent=False)
        self.sin = nn.Buffer(theta.sin(), persistent=False)

    def forward(self, x: Tensor) -> Tensor:          # [B, T, H, D]
        T = x.size(-3)
        cos, sin = self.cos[None, :T, None, :], self.sin[None, :T, None, :]
        x1, x2 = x.to(torch.float32).chunk(2, dim=-1)
        return torch.cat((x1 * cos + x2 * sin, x2 * cos - x1 * sin), -1).type_as(x)


class ScopeAttention(nn.Module):
    """The SCOPE attention of one layer (scoped_medium.py:334-479, qk_aug mode)."""

    def __init__(self, dim: int, num_heads: int, head_dim: int, max_seq_len: int, *, K: int, M: int,
                 local_blocks: int, half_blocks: int, budget_blocks: int, global_blocks: int, seed: int):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        hdim = num_heads * head_dim
        bound = (3 ** 0.5) * 0.5 * dim ** -0.5
        self.qkv_w = nn.Parameter(torch.empty(3, hdim, dim).uniform_(-bound, bound))
        self.lambdas = nn.Parameter(torch.tensor([0.5, 0.5]))
        self.rotary = Rotary(head_dim, max_seq_len)
        self.c_proj = CastedLinear(hdim, dim)
        with torch.no_grad():
            self.c_proj.weight.zero_()
        self.attn_scale = 0.12
        self.beta = 0.5
        # the coefficient block (SpectralBias.forward) with trainable MLP weights
        self.sc = SpectralCoefficients(head_dim=head_dim, num_heads=num_heads, L_train=max_seq_len, K=K, M=M,
                                       use_slope=True, seed=seed, device="cpu")
        self.sc_w1 = nn.Parameter(self.sc.w1[0].clone())
        self.sc_b1 = nn.Parameter(self.sc.b1[0].clone())
        self.sc_w2 = nn.Parameter(self.sc.w2[0].clone())
        self.sc_b2 = nn.Parameter(self.sc.b2[0].clone())
        self.builder = PointerBlockMaskBuilder(num_heads=num_heads, M=M, pointer_local_blocks=local_blocks,
                                               pointer_half_blocks=half_blocks, pointer_budget_blocks=budget_blocks,
                                               pointer_budget_is_total=False, pointer_budget_temp=0.5,
                                               pointer_global_blocks=global_blocks)

    def _coeff_block(self, q_bhtd: Tensor):
        sc = self.sc
        if sc.omegas.device != q_bhtd.device:
            sc.omegas = sc.omegas.to(q_bhtd.device)
            sc.log_omegas = sc.log_omegas.to(q_bhtd.device)
        sc.load_weights(self.sc_w1, self.sc_b1, self.sc_w2, self.sc_b2)
        return sc(q_bhtd)

    def attend(self, x: Tensor, ve: Optional[Tensor], docs: Tensor, keep: Optional[dict] = None) -> Tensor:
        """[1, T, H*D] attention output before the output projection; ``keep``
        (a dict) receives the layer's intermediate tensors."""
        B, T = x.size(0), x.size(1)
        H, D = self.num_heads, self.head_dim
        q, k, v = F.linear(x, self.qkv_w.flatten(end_dim=1).type_as(x)).view(B, T, 3 * H, D).chunk(3, dim=-2)
        q, k = norm(q), norm(k)
        q_for_bias = q.transpose(1, 2)                      # [B, H, T, D] before rotary
        q, k = self.rotary(q), self.rotary(k)
        v = self.lambdas[0] * v + (self.lambdas[1] * ve.view_as(v) if ve is not None else 0)
        (cc, cs, slope, _b0, delta_star, pi, budget_logits, _dm, _w, cos_t, sin_t, _reg) = self._coeff_block(q_for_bias)
        bm = self.builder.build_pointer_blockmask(docs=docs, delta_star=delta_star.detach(), pi=pi.detach(),
                                                  budget_logits=budget_logits.detach(), block_size=128)
        sm = SpectralScoreMod(coeff_cos=cc, coeff_sin=cs, cos_tab=cos_t, sin_tab=sin_t, beta=self.beta,
                              slope=slope, impl="qk_aug")
        y = flex_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), bm, score_mod=sm,
                           scale=self.attn_scale)
        self.last_mask = bm
        if keep is not None:
            keep.update(q=q, k=k, v=v, coeff_cos=cc, coeff_sin=cs, slope=slope, cos_tab=cos_t, sin_tab=sin_t,
                        mask=bm, y=y)
        return y.transpose(1, 2).contiguous().view(B, T, H * D)

    def forward(self, x: Tensor, ve: Optional[Tensor], docs: Tensor) -> Tensor:
        return self.c_proj(self.attend(x, ve, docs))


class MLP(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.c_fc = CastedLinear(dim, 4 * dim)
        self.c_proj = CastedLinear(4 * dim, dim)
        with torch.no_grad():
            self.c_proj.weight.zero_()

    def forward(self, x: Tensor) -> Tensor:
        return self.c_proj(F.relu(self.c_fc(x)).square())


class Block(nn.Module):
    def __init__(self, dim: int, num_heads: int, head_dim: int, max_seq_len: int, layer: int, **attn_kw):
        super().__init__()
        self.attn = ScopeAttention(dim, num_heads, head_dim, max_seq_len, seed=1000 + layer, **attn_kw)
        self.mlp = MLP(dim)
        self.lambdas = nn.Parameter(torch.tensor([1.0, 0.0]))

    def forward(self, x: Tensor, ve: Optional[Tensor], x0: Tensor, docs: Tensor) -> Tensor:
        x = self.lambdas[0] * x + self.lambdas[1] * x0
        x = x + self.attn(norm(x), ve, docs)
        return x + self.mlp(norm(x))


class ScopeDecoder(nn.Module):
    """Configuration C4 by default: 24 layers, d_model 1024, 16 heads x 64,
    MLP 4x, vocab 50304; every layer K = 8 spectral frequencies and the pointer
    mask at block size 128 with an 8-block local band and 4 pointer blocks per
    query block."""

    def __init__(self, *, vocab_size: int = 50304, num_layers: int = 24, model_dim: int = 1024, num_heads: int = 16,
                 head_dim: int = 64, max_seq_len: int = 65536, K: int = 8, M: int = 4, local_blocks: int = 8,
                 half_blocks: int = 0, budget_blocks: int = 0, global_blocks: int = 0):
        super().__init__()
        if num_layers % 2 or num_layers < 6:
            raise ValueError("num_layers must be even and at least 6")
        self.embed = nn.Embedding(vocab_size, model_dim)
        self.value_embeds = nn.ModuleList([nn.Embedding(vocab_size, model_dim) for _ in range(3)])
        kw = dict(K=K, M=M, local_blocks=local_blocks, half_blocks=half_blocks, budget_blocks=budget_blocks,
                  global_blocks=global_blocks)
        self.blocks = nn.ModuleList([Block(model_dim, num_heads, head_dim, max_seq_len, i, **kw)
                                     for i in range(num_layers)])
        self.lm_head = CastedLinear(model_dim, vocab_size)
        with torch.no_grad():
            self.lm_head.weight.zero_()
        self.skip_weights = nn.Parameter(torch.ones(num_layers // 2))
        for m in self.modules():
            if isinstance(m, nn.Embedding):
                m.bfloat16()

    def forward(self, input_seq: Tensor, target_seq: Tensor) -> Tensor:
        docs = (input_seq == EOD_TOKEN_ID).cumsum(0).to(torch.int32)
        ve = [e(input_seq) for e in self.value_embeds]
        n_layers = len(self.blocks)
        ve = [ve[0], ve[1], ve[2]] + [None] * (n_layers - 6) + [ve[0], ve[1], ve[2]]
        x = x0 = norm(self.embed(input_seq)[None])
        skips: List[Tensor] = []
        n = len(self.skip_weights)
        for i, blk in enumerate(self.blocks):
            if i >= n:
                x = x + self.skip_weights[i - n] * skips.pop()
            x = blk(x, ve[i], x0, docs)
            if i < n:
                skips.append(x)
        x = norm(x)
        logits = 30 * torch.sigmoid(self.lm_head(x).float() / 7.5)
        return F.cross_entropy(logits.view(-1, logits.size(-1)), target_seq)

    def attention_pairs(self) -> int:
        """Active (q block, kv block) pairs summed over the layers' last masks."""
        return int(sum(int(b.attn.last_mask.kv_num_blocks.sum().item()) for b in self.blocks
                       if getattr(b.attn, "last_mask", None) is not None))

    def flops_per_token(self) -> float:
        """6 x the matmul parameters (the embeddings are lookups)."""
        n = sum(p.numel() for name, p in self.named_parameters() if "embed" not in name and p.dim() >= 2)
        return 6.0 * n


class BucketedAllReduce:
    """Gradients as views of flat per-dtype buckets of about ``bucket_mb``,
    filled in the order the backward produces them (the reverse of
    registration); each bucket is all-reduced (mean over ranks) as soon as its
    last gradient has been accumulated, on the process group's stream, so the
    exchange overlaps the rest of the backward.  ``zero_grad()`` before the
    backward, ``wait()`` after it and before the optimizer step."""

    def __init__(self, params, group=None, bucket_mb: float = 64.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.params = [p for p in params if p.requires_grad]
        cap = int(bucket_mb * (1 << 20))
        self.buckets = []                 # (flat buffer, [params], [offsets])
        cur, size, dtype = [], 0, None
        for p in reversed(self.params):
            nbytes = p.numel() * p.element_size()
            if cur and (p.dtype != dtype or size + nbytes > cap):
                self._close(cur, dtype)
                cur, size = [], 0
            cur.append(p)
            size += nbytes
            dtype = p.dtype
        if cur:
            self._close(cur, dtype)
        self.pending = [0] * len(self.buckets)
        self.works = []
        self._avg = dist.get_backend(group) == "nccl"
        for bi, (_, ps, _) in enumerate(self.buckets):
            for p in ps:
                p.register_post_accumulate_grad_hook(lambda _p, bi=bi: self._ready(bi))

    def _close(self, ps, dtype):
        n = sum(p.numel() for p in ps)
        buf = torch.zeros(n, dtype=dtype, device=ps[0].device)
        offs, o = [], 0
        for p in ps:
            p.grad = buf[o:o + p.numel()].view_as(p)
            offs.append(o)
            o += p.numel()
        self.buckets.append((buf, ps, offs))

    def zero_grad(self):
        for bi, (buf, ps, offs) in enumerate(self.buckets):
            buf.zero_()
            for p, o in zip(ps, offs):
                if p.grad is None or p.grad.data_ptr() != buf[o:].data_ptr():
                    p.grad = buf[o:o + p.numel()].view_as(p)
            self.pending[bi] = len(ps)
        self.works = []

    def _ready(self, bi):
        self.pending[bi] -= 1
        if self.pending[bi] == 0:
            buf = self.buckets[bi][0]
            op = dist.ReduceOp.AVG if self._avg else dist.ReduceOp.SUM
            self.works.append((bi, dist.all_reduce(buf, op=op, group=self.group, async_op=True)))

    def wait(self):
        for bi, w in self.works:
            w.wait()
            if not self._avg:
                self.buckets[bi][0].div_(self.world)
        if len(self.works) != len(self.buckets):
            raise RuntimeError("a gradient bucket was not complete after the backward")
        self.works = []


def synthetic_tokens(T: int, vocab: int = 50304, *, seed: int, device) -> tuple[Tensor, Tensor]:
    """One sequence of T + 1 token ids uniform over the vocab: inputs and the
    shifted-by-one targets (configuration C4's synthetic data)."""
    g = torch.Generator().manual_seed(seed)
    seq = torch.randint(0, vocab, (T + 1,), generator=g, dtype=torch.int64)
    seq = seq.to(device)
    return seq[:-1], seq[1:]
