"""Teacher block mass on the tensor cores.

Drop-in for the dense loop of the reference's spectral teacher
(scoped_medium.py:1793-1819)::

    teacher_mass = torch.zeros((Hh, num_blocks, num_blocks), ...)
    for qb in range(num_blocks):
        scores = q_block @ k_sel^T * scale (+ q_pos_block @ k_pos^T * scale)
        ... document-causal mask, softmax, column sums scattered into kv blocks
        teacher_mass[:, qb, :] = mass

becomes::

    teacher_mass = scope_b200.teacher_block_mass(q_sel, k_sel, docs, scale=attn.attn_scale,
                                                 q_pos=q_pos, k_pos=k_pos)

One launch of the forward kernel's mass variant (scope_block_mass in the C
ABI): per (head, query block) the kv blocks from the document start of the
block's first row to the diagonal, each 128 x 128 score tile formed once for
the row statistics and once for the probabilities, no [T, T] scores in HBM.
Scores stay in float32 from the bf16 inputs; the reference's bf16 matmuls
round each score to bf16 before its softmax, which moves a block's mass
(out of 128) by up to about 0.05 on unit-variance q and k at 4,096 tokens.
Runs under no_grad, as the reference's.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .attention import DTYPES, BIAS_MODES
from .mask import _stream, block_info

BLOCK = 128


def _pad_cols(t: Tensor, width: int) -> Tensor:
    out = t.new_zeros(*t.shape[:-1], width)
    out[..., : t.shape[-1]] = t
    return out


@torch.no_grad()
def teacher_block_mass(q: Tensor, k: Tensor, docs: Optional[Tensor] = None, *, scale: float,
                       q_pos: Optional[Tensor] = None, k_pos: Optional[Tensor] = None) -> Tensor:
    """mass[h, qb, kb]: the dense document-causal softmax of
    (q k^T + q_pos k_pos^T) * scale summed over the rows of query block qb and
    the keys of kv block kb ([H, QB, QB] float32; zero above the diagonal,
    each (h, qb) row summing to 128).

    q, k: [H, T, 64] (or [1, H, T, 64]) bf16, the reference's q_sel / k_sel.
    q_pos [H, T, P] and k_pos [H, T, P] or [T, P] (P <= 64): its augmented
    dims, already scaled by sqrt(beta / scale) and cast to bf16; the key side
    is the same for every head in the reference (trig tables and positions),
    so only head 0 of a 3-D k_pos is read.  docs [T]: document ids, runs of
    equal ids (the reference's cumulative separator count); None = one
    document.  T must be a multiple of 128."""
    if q.dim() == 4 and q.shape[0] == 1:
        q, k = q[0], k[0]
    if q.dim() != 3 or k.shape != q.shape:
        raise ValueError("q and k must be [H, T, 64] (or [1, H, T, 64]) of one shape")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise TypeError("teacher_block_mass takes bf16 q and k")
    H, T, D = q.shape
    if D != 64 or T % BLOCK:
        raise ValueError("head_dim must be 64 and T a multiple of 128")
    if not q.is_cuda or not k.is_cuda:
        raise RuntimeError("scope_b200 ops run on CUDA tensors only")
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    dev = q.device
    QB = T // BLOCK
    qa = ka = None
    if (q_pos is None) != (k_pos is None):
        raise ValueError("q_pos and k_pos go together")
    if q_pos is not None:
        if q_pos.dim() == 4 and q_pos.shape[0] == 1:
            q_pos = q_pos[0]
        if k_pos.dim() == 4 and k_pos.shape[0] == 1:
            k_pos = k_pos[0]
        if k_pos.dim() == 3:
            k_pos = k_pos[0]
        P = q_pos.shape[-1]
        if q_pos.shape != (H, T, P) or k_pos.shape != (T, P) or P > 64:
            raise ValueError("q_pos must be [H, T, P] and k_pos [H, T, P] or [T, P] with P <= 64")
        da = (P + 15) // 16 * 16
        qa = _pad_cols(q_pos.to(torch.bfloat16), da).contiguous()
        ka = _pad_cols(k_pos.to(torch.bfloat16), da).contiguous()
    d = None
    if docs is not None:
        d = docs.to(device=dev, dtype=torch.int32).contiguous()
        if d.numel() != T:
            raise ValueError("docs must have T entries")
    info = block_info(d, T, BLOCK, device=dev) if d is not None else None
    mass = torch.empty(H, QB, QB, dtype=torch.float32, device=dev)
    a = _lib.ScopeAttnArgs()
    a.H, a.T, a.D, a.block_size = H, T, D, BLOCK
    a.dtype = DTYPES[torch.bfloat16]
    a.q, a.k = q.data_ptr(), k.data_ptr()
    a.q_sh, a.q_st = q.stride(0), q.stride(1)
    a.k_sh, a.k_st = k.stride(0), k.stride(1)
    a.docs = _lib.ptr(d)
    a.block_info = _lib.ptr(info)
    a.scale = float(scale)
    a.bias_mode = BIAS_MODES["qk_aug"] if qa is not None else BIAS_MODES["none"]
    a.q_aug, a.k_aug = _lib.ptr(qa), _lib.ptr(ka)
    a.d_aug = 0 if qa is None else qa.shape[-1]
    a.err_flag = _lib.err_word_ptr(dev)
    st = _lib.lib().scope_block_mass(ctypes.byref(a), mass.data_ptr(), _stream(dev))
    _lib.check(st, "scope_block_mass")
    return mass
