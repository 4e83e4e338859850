"""Block-sparse SCOPE attention as a torch custom op over the C ABI.

Drop-in for the reference's attention call (scoped_medium.py:459-466)::

    flex_attention(q, k, v, block_mask=bm, score_mod=<spectral closure>, scale=0.12)

becomes::

    scope_b200.flex_attention(q, k, v, block_mask=bm, score_mod=SpectralScoreMod(...), scale=0.12)

A C ABI cannot take the Python closures, so the tensors the reference's
score_mod and mask_mod capture (coefficients, trig tables, b0, slope,
Δ_main, width, the document ids) travel explicitly: ``SpectralScoreMod``
holds the score_mod's, ``ScopeBlockMask`` the mask_mod's.

The op is registered with ``torch.library.custom_op`` + ``register_fake`` +
``register_autograd`` the way the reference registers its fp8 matmul
(``nanogpt::mm``, scoped_medium.py:74-154), so it composes with autograd and
torch.compile without any Triton.  Forward and backward each run our CUDA
kernels on the current stream; nothing here computes attention in PyTorch.
"""
import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .mask import ScopeBlockMask, _stream

DTYPES = {torch.float32: 0, torch.bfloat16: 1}
BIAS_MODES = {"none": 0, "score_mod": 1, "qk_aug": 2}
GATES = {"none": 0, "softplus": 1, "relu": 2}
OP_CUDA_CORES, OP_HEAD_MAJOR_OUT = 0x1, 0x2     # `flags` of the custom ops


def aug_dims(K: int, slope: bool) -> int:
    """Augmented head dims of the qk_aug mode: 2K (+1 with slope), padded to 16."""
    need = 2 * K + (1 if slope else 0)
    return (need + 15) // 16 * 16


@dataclass
class SpectralScoreMod:
    """What the reference's spectral score_mod closure captures
    (scoped_medium.py:425-457): per-query Fourier coefficients [.., H, T, K]
    (float32), the bf16 trig tables [K, L], beta, and optionally b0, slope,
    Δ_main and width [.., H, T] with the gate settings.  ``impl`` picks the
    reference's two spectral implementations: "score_mod" (exact closure
    semantics) or "qk_aug" (augmented Q/K dims, scoped_medium.py:380-423; the
    reference default, which drops b0 and the gate)."""
    coeff_cos: Tensor
    coeff_sin: Tensor
    cos_tab: Tensor
    sin_tab: Tensor
    beta: float = 0.5
    b0: Optional[Tensor] = None
    slope: Optional[Tensor] = None
    delta_main: Optional[Tensor] = None
    width: Optional[Tensor] = None
    gate: str = "none"
    ramp_lambda: float = 0.2
    tau: float = 64.0
    impl: str = "qk_aug"


def _hd(t: Optional[Tensor], rank: int) -> Optional[Tensor]:
    """Drop a leading batch dim of size 1 from a tensor whose unbatched rank is
    ``rank``, as a view (squeeze, whose backward is a view too; indexing with
    t[0] would make autograd materialise a zero tensor and copy every gradient
    into it)."""
    if t is None:
        return None
    return t.squeeze(0) if t.dim() == rank + 1 and t.shape[0] == 1 else t


def _attn_args(q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs,
               coeff_cos, coeff_sin, cos_tab, sin_tab, b0, slope, delta_main, width,
               scale, beta, bias_mode, gate, gate_lambda, gate_tau, block_size, q_aug, k_aug, cuda_cores=False):
    a = _lib.ScopeAttnArgs()
    H, T, D = q.shape
    a.H, a.T, a.D, a.block_size = H, T, D, block_size
    a.dtype = DTYPES[q.dtype]
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.q_sh, a.q_st = q.stride(0), q.stride(1)
    a.k_sh, a.k_st = k.stride(0), k.stride(1)
    a.v_sh, a.v_st = v.stride(0), v.stride(1)
    a.out = out.data_ptr()
    a.o_sh, a.o_st = out.stride(0), out.stride(1)
    a.lse = lse.data_ptr()
    a.kv_num, a.kv_indices = kv_num.data_ptr(), kv_indices.data_ptr()
    a.kv_stride = kv_indices.shape[-1]
    a.q_bitmap = _lib.ptr(q_bitmap)
    a.block_info = _lib.ptr(block_info)
    a.docs = _lib.ptr(docs)
    a.scale = scale
    a.bias_mode = bias_mode
    if coeff_cos is not None:
        a.K = coeff_cos.shape[-1]
    a.coeff_cos, a.coeff_sin = _lib.ptr(coeff_cos), _lib.ptr(coeff_sin)
    a.cos_tab, a.sin_tab = _lib.ptr(cos_tab), _lib.ptr(sin_tab)
    if cos_tab is not None:
        a.tab_len = cos_tab.shape[-1]
    a.b0, a.slope = _lib.ptr(b0), _lib.ptr(slope)
    a.delta_main, a.width = _lib.ptr(delta_main), _lib.ptr(width)
    a.gate, a.beta, a.gate_lambda, a.gate_tau = gate, beta, gate_lambda, gate_tau
    a.q_aug, a.k_aug = _lib.ptr(q_aug), _lib.ptr(k_aug)
    a.d_aug = 0 if q_aug is None else q_aug.shape[-1]
    a.flags = _lib.FLAG_CUDA_CORES if cuda_cores else 0
    a.err_flag = _lib.err_word_ptr(q.device)
    return a


def _check_inputs(q, k, v, kv_num, kv_indices, block_size):
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must be [H, T, D] (or [1, H, T, D]) of one shape")
    if q.dtype not in DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must all be float32 or all bfloat16")
    for t in (q, k, v):
        if t.stride(-1) != 1:
            raise ValueError("the head dim of q, k, v must be contiguous")
        if not t.is_cuda:
            raise RuntimeError("scope_b200 attention runs on CUDA tensors only")
    H, T, D = q.shape
    if D != 64:
        raise ValueError("head_dim must be 64")
    if T % block_size:
        raise ValueError("T must be a multiple of the block size")
    if tuple(kv_num.shape[-2:]) != (H, T // block_size):
        raise ValueError("block mask does not match q (heads or q blocks)")


def _smod_on_tensor_cores(q, coeff_cos, bias_mode, block_size, cuda_cores) -> bool:
    """score_mod runs on the tensor-core kernels (its Fourier sum in augmented
    dims, the slope and gate terms per element) for bf16 inputs in 128-token
    blocks with K <= 16; otherwise on the CUDA cores."""
    return (bias_mode == BIAS_MODES["score_mod"] and q.dtype == torch.bfloat16 and block_size == 128
            and not cuda_cores and coeff_cos is not None and coeff_cos.shape[-1] <= 16)


def _prepare_aug(q, coeff_cos, coeff_sin, slope, cos_tab, sin_tab, beta, scale, bias_mode, block_size=128,
                 cuda_cores=False):
    """Augmented dims: qk_aug mode (with the slope column when there is a
    slope), or the score_mod mode's Fourier sum alone on the tensor cores."""
    if bias_mode == BIAS_MODES["score_mod"] and _smod_on_tensor_cores(q, coeff_cos, bias_mode, block_size, cuda_cores):
        slope = None
    elif bias_mode != BIAS_MODES["qk_aug"]:
        return None, None
    H, T, _ = q.shape
    K = coeff_cos.shape[-1]
    da = aug_dims(K, slope is not None)
    q_aug = torch.empty(H, T, da, dtype=q.dtype, device=q.device)
    k_aug = torch.empty(T, da, dtype=q.dtype, device=q.device)
    st = _lib.lib().scope_qk_aug_prepare(
        coeff_cos.data_ptr(), coeff_sin.data_ptr(), _lib.ptr(slope), cos_tab.data_ptr(), sin_tab.data_ptr(),
        cos_tab.shape[-1], H, T, K, da, beta, scale, DTYPES[q.dtype], q_aug.data_ptr(), k_aug.data_ptr(),
        _stream(q.device))
    _lib.check(st, "scope_qk_aug_prepare")
    return q_aug, k_aug


def _new_like_layout(x: Tensor) -> Tensor:
    """[H,T,D] output laid out as [T,H,D] in memory (what the reference's
    .transpose(1, 2).contiguous() wants next), returned as an [H,T,D] view."""
    H, T, D = x.shape
    return torch.empty(T, H, D, dtype=x.dtype, device=x.device).permute(1, 0, 2)


@torch.library.custom_op("scope::sparse_attn", mutates_args=())
def sparse_attn(q: Tensor, k: Tensor, v: Tensor, kv_num: Tensor, kv_indices: Tensor, q_bitmap: Tensor,
                block_info: Tensor, docs: Optional[Tensor], coeff_cos: Optional[Tensor],
                coeff_sin: Optional[Tensor], cos_tab: Optional[Tensor], sin_tab: Optional[Tensor],
                b0: Optional[Tensor], slope: Optional[Tensor], delta_main: Optional[Tensor],
                width: Optional[Tensor], scale: float, beta: float, bias_mode: int, gate: int,
                gate_lambda: float, gate_tau: float, block_size: int,
                flags: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Returns out, lse and (qk_aug mode, and score_mod on the tensor cores) the
    augmented dims q_aug / k_aug, which the backward reuses; empty tensors
    otherwise.  ``flags``:
    OP_CUDA_CORES, OP_HEAD_MAJOR_OUT (out stored [H, T, D] instead of the
    [T, H, D] storage of the reference's layout)."""
    _check_inputs(q, k, v, kv_num, kv_indices, block_size)
    H, T, D = q.shape
    cuda_cores = bool(flags & OP_CUDA_CORES)
    out = torch.empty(H, T, D, dtype=q.dtype, device=q.device) if flags & OP_HEAD_MAJOR_OUT else _new_like_layout(q)
    lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
    q_aug, k_aug = _prepare_aug(q, coeff_cos, coeff_sin, slope, cos_tab, sin_tab, beta, scale, bias_mode,
                                block_size, cuda_cores)
    a = _attn_args(q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin,
                   cos_tab, sin_tab, b0, slope, delta_main, width, scale, beta, bias_mode, gate, gate_lambda,
                   gate_tau, block_size, q_aug, k_aug, cuda_cores)
    _lib.check(_lib.lib().scope_attn_fwd(ctypes.byref(a), _stream(q.device)), "scope_attn_fwd")
    if q_aug is None:
        q_aug, k_aug = q.new_empty(0), q.new_empty(0)
    return out, lse, q_aug, k_aug


@sparse_attn.register_fake
def _(q, k, v, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin, cos_tab, sin_tab,
      b0, slope, delta_main, width, scale, beta, bias_mode, gate, gate_lambda, gate_tau, block_size, flags):
    H, T, D = q.shape
    out = q.new_empty(H, T, D) if flags & OP_HEAD_MAJOR_OUT else q.new_empty(T, H, D).permute(1, 0, 2)
    if bias_mode == BIAS_MODES["qk_aug"] or _smod_on_tensor_cores(q, coeff_cos, bias_mode, block_size,
                                                                  bool(flags & OP_CUDA_CORES)):
        da = aug_dims(coeff_cos.shape[-1], slope is not None and bias_mode == BIAS_MODES["qk_aug"])
        qa, ka = q.new_empty(H, T, da), q.new_empty(T, da)
    else:
        qa, ka = q.new_empty(0), q.new_empty(0)
    return out, q.new_empty(H, T, dtype=torch.float32), qa, ka


@torch.library.custom_op("scope::sparse_attn_bwd", mutates_args=())
def sparse_attn_bwd(dout: Tensor, q: Tensor, k: Tensor, v: Tensor, out: Tensor, lse: Tensor, kv_num: Tensor,
                    kv_indices: Tensor, q_bitmap: Tensor, block_info: Tensor, docs: Optional[Tensor],
                    coeff_cos: Optional[Tensor], coeff_sin: Optional[Tensor], cos_tab: Optional[Tensor],
                    sin_tab: Optional[Tensor], b0: Optional[Tensor], slope: Optional[Tensor],
                    delta_main: Optional[Tensor], width: Optional[Tensor], q_aug: Optional[Tensor],
                    k_aug: Optional[Tensor], scale: float, beta: float,
                    bias_mode: int, gate: int, gate_lambda: float, gate_tau: float, block_size: int,
                    want_bias_grads: bool, flags: int) -> list[Tensor]:
    H, T, D = q.shape
    cuda_cores = bool(flags & OP_CUDA_CORES)
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    dq, dk, dv = _new_like_layout(q), _new_like_layout(k), _new_like_layout(v)
    if q_aug is None or q_aug.numel() == 0:
        q_aug, k_aug = _prepare_aug(q, coeff_cos, coeff_sin, slope, cos_tab, sin_tab, beta, scale, bias_mode,
                                    block_size, cuda_cores)
    a = _attn_args(q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin,
                   cos_tab, sin_tab, b0, slope, delta_main, width, scale, beta, bias_mode, gate, gate_lambda,
                   gate_tau, block_size, q_aug, k_aug, cuda_cores)
    a.dout, a.do_sh, a.do_st = dout.data_ptr(), dout.stride(0), dout.stride(1)
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.dq_sh, a.dq_st = dq.stride(0), dq.stride(1)
    a.dk_sh, a.dk_st = dk.stride(0), dk.stride(1)
    a.dv_sh, a.dv_st = dv.stride(0), dv.stride(1)
    # absent gradients are returned as distinct empty tensors (custom ops may not alias outputs)
    dcc, dcs, db0, dsl, ddm, dw = (q.new_empty(0, dtype=torch.float32) for _ in range(6))
    if want_bias_grads and coeff_cos is not None:
        dcc = torch.empty_like(coeff_cos)
        dcs = torch.empty_like(coeff_sin)
        a.dcoeff_cos, a.dcoeff_sin = dcc.data_ptr(), dcs.data_ptr()
        if slope is not None:
            dsl = torch.empty_like(slope)
            a.dslope = dsl.data_ptr()
        if bias_mode == BIAS_MODES["score_mod"]:
            if b0 is not None:
                db0 = torch.empty_like(b0)
                a.db0 = db0.data_ptr()
            if gate != 0 and delta_main is not None:
                ddm, dw = torch.empty_like(delta_main), torch.empty_like(width)
                a.ddelta_main, a.dwidth = ddm.data_ptr(), dw.data_ptr()
    nbytes = _lib.lib().scope_workspace_bytes(ctypes.byref(a))
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=q.device)
    base = ws.data_ptr()
    a.workspace = (base + 255) // 256 * 256
    a.workspace_bytes = nbytes
    _lib.check(_lib.lib().scope_attn_bwd(ctypes.byref(a), _stream(q.device)), "scope_attn_bwd")
    return [dq, dk, dv, dcc, dcs, db0, dsl, ddm, dw]


@sparse_attn_bwd.register_fake
def _(dout, q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin, cos_tab,
      sin_tab, b0, slope, delta_main, width, q_aug, k_aug, scale, beta, bias_mode, gate, gate_lambda, gate_tau,
      block_size, want_bias_grads, flags):
    H, T, D = q.shape
    mk = lambda x: x.new_empty(T, H, D).permute(1, 0, 2)  # noqa: E731
    e = lambda: q.new_empty(0, dtype=torch.float32)  # noqa: E731
    dcc = torch.empty_like(coeff_cos) if (want_bias_grads and coeff_cos is not None) else e()
    dcs = torch.empty_like(coeff_sin) if (want_bias_grads and coeff_sin is not None) else e()
    dsl = torch.empty_like(slope) if (want_bias_grads and coeff_cos is not None and slope is not None) else e()
    sm = bias_mode == BIAS_MODES["score_mod"] and want_bias_grads and coeff_cos is not None
    db0 = torch.empty_like(b0) if (sm and b0 is not None) else e()
    ddm = torch.empty_like(delta_main) if (sm and gate != 0 and delta_main is not None) else e()
    dw = torch.empty_like(width) if (sm and gate != 0 and delta_main is not None) else e()
    return [mk(q), mk(k), mk(v), dcc, dcs, db0, dsl, ddm, dw]


_TENSOR_ARGS = ("q", "k", "v", "kv_num", "kv_indices", "q_bitmap", "block_info", "docs", "coeff_cos",
                "coeff_sin", "cos_tab", "sin_tab", "b0", "slope", "delta_main", "width")


def _setup_context(ctx, inputs, output):
    (q, k, v, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin, cos_tab, sin_tab,
     b0, slope, delta_main, width, scale, beta, bias_mode, gate, gate_lambda, gate_tau, block_size,
     flags) = inputs
    out, lse, q_aug, k_aug = output
    ctx.mark_non_differentiable(lse, q_aug, k_aug)
    ctx.save_for_backward(q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos,
                          coeff_sin, cos_tab, sin_tab, b0, slope, delta_main, width, q_aug, k_aug)
    ctx.scal = (scale, beta, bias_mode, gate, gate_lambda, gate_tau, block_size, flags)


def _backward(ctx, dout, dlse, dq_aug, dk_aug):
    (q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs, coeff_cos, coeff_sin, cos_tab,
     sin_tab, b0, slope, delta_main, width, q_aug, k_aug) = ctx.saved_tensors
    scale, beta, bias_mode, gate, gate_lambda, gate_tau, block_size, flags = ctx.scal
    nig = ctx.needs_input_grad
    want_bias = any(nig[i] for i in (8, 9, 12, 13, 14, 15))
    g = torch.ops.scope.sparse_attn_bwd(dout, q, k, v, out, lse, kv_num, kv_indices, q_bitmap, block_info, docs,
                                        coeff_cos, coeff_sin, cos_tab, sin_tab, b0, slope, delta_main, width,
                                        q_aug, k_aug, scale, beta, bias_mode, gate, gate_lambda, gate_tau,
                                        block_size, want_bias, flags)
    dq, dk, dv, dcc, dcs, db0, dsl, ddm, dw = g
    pick = lambda t: t if (t is not None and t.numel() > 0) else None  # noqa: E731
    return (dq, dk, dv, None, None, None, None, None, pick(dcc), pick(dcs), None, None, pick(db0), pick(dsl),
            pick(ddm), pick(dw), None, None, None, None, None, None, None, None)


sparse_attn.register_autograd(_backward, setup_context=_setup_context)


def flex_attention(query: Tensor, key: Tensor, value: Tensor, block_mask,
                   score_mod: Optional[SpectralScoreMod] = None, scale: Optional[float] = None,
                   return_lse: bool = False, cuda_cores: bool = False, docs: Optional[Tensor] = None,
                   head_major_out: bool = False):
    """Block-sparse attention with the SCOPE spectral bias, same call shape
    as torch's flex_attention: q, k, v [1, H, T, D] (any head/token strides,
    contiguous D), ``block_mask`` from the pointer builder (``ScopeBlockMask``)
    or a torch ``BlockMask`` such as the reference builder returns (then
    ``docs`` carries the document ids its document_causal mask_mod captures,
    see ``ScopeBlockMask.from_flex``), ``score_mod`` the captured
    spectral-bias state or None.  Returns [1, H, T, D] in the input dtype (and
    the [1, H, T] float32 natural-log lse with ``return_lse``).
    ``cuda_cores`` runs the CUDA-core kernels even where the tensor-core
    kernels apply (to cross-check the two).  ``head_major_out`` stores the
    output as [H, T, D] (a head shard's slice of the [H, T, D] all-gather
    buffer) instead of the [T, H, D] storage the reference's layout has."""
    squeeze = query.dim() == 4
    if squeeze and query.shape[0] != 1:
        raise ValueError("batch size must be 1 (as in the reference)")
    if not isinstance(block_mask, ScopeBlockMask):
        block_mask = ScopeBlockMask.from_flex(block_mask, docs=docs)
    elif docs is not None:
        raise ValueError("docs= goes with a torch BlockMask; a ScopeBlockMask carries its own")
    q, k, v = (_hd(t, 3) for t in (query, key, value))
    D = q.shape[-1]
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    if block_mask.BLOCK_SIZE[0] > 128:
        block_mask = block_mask.kernel_tiles(128)    # e.g. a block-size-256 mask (config C5)
    bs = block_mask.BLOCK_SIZE[0]
    kv_num = block_mask.kv_num_blocks[0]
    kv_idx = block_mask.kv_indices[0]
    docs = block_mask.docs
    args = dict(coeff_cos=None, coeff_sin=None, cos_tab=None, sin_tab=None, b0=None, slope=None,
                delta_main=None, width=None, beta=0.0, bias_mode=0, gate=0, gate_lambda=0.0, gate_tau=1.0)
    if score_mod is not None:
        sm = score_mod
        if sm.impl not in ("score_mod", "qk_aug"):
            raise ValueError("SpectralScoreMod.impl must be score_mod|qk_aug")
        if sm.gate not in GATES:
            raise ValueError("gate must be one of: none|softplus|relu")
        f32 = lambda t, rank: None if t is None else _hd(t, rank).to(torch.float32).contiguous()  # noqa: E731
        args.update(coeff_cos=f32(sm.coeff_cos, 3), coeff_sin=f32(sm.coeff_sin, 3),
                    cos_tab=sm.cos_tab.to(torch.bfloat16).contiguous(),
                    sin_tab=sm.sin_tab.to(torch.bfloat16).contiguous(), slope=f32(sm.slope, 2),
                    beta=float(sm.beta), bias_mode=BIAS_MODES[sm.impl])
        if sm.impl == "score_mod":
            args.update(b0=f32(sm.b0, 2), delta_main=f32(sm.delta_main, 2), width=f32(sm.width, 2),
                        gate=GATES[sm.gate] if sm.ramp_lambda > 0 else 0, gate_lambda=float(sm.ramp_lambda),
                        gate_tau=float(sm.tau))
    out, lse, _, _ = torch.ops.scope.sparse_attn(q, k, v, kv_num, kv_idx, block_mask.q_bitmap, block_mask.block_info,
                                           docs, args["coeff_cos"], args["coeff_sin"], args["cos_tab"],
                                           args["sin_tab"], args["b0"], args["slope"], args["delta_main"],
                                           args["width"], sc, args["beta"], args["bias_mode"], args["gate"],
                                           args["gate_lambda"], args["gate_tau"], bs,
                                           (OP_CUDA_CORES if cuda_cores else 0) |
                                           (OP_HEAD_MAJOR_OUT if head_major_out else 0))
    if squeeze:
        out, lse = out.unsqueeze(0), lse.unsqueeze(0)
    return (out, lse) if return_lse else out


def trig_tables(omegas: Tensor, L: int) -> tuple[Tensor, Tensor]:
    """bf16 tables cos/sin(fp32(w_k d)), d in [0, L) (model/attn_bias.py:326-340)."""
    w = omegas.to(torch.float32).contiguous()
    K = w.numel()
    c = torch.empty(K, L, dtype=torch.bfloat16, device=w.device)
    s = torch.empty(K, L, dtype=torch.bfloat16, device=w.device)
    st = _lib.lib().scope_trig_tables(w.data_ptr(), K, L, c.data_ptr(), s.data_ptr(), _stream(w.device))
    _lib.check(st, "scope_trig_tables")
    return c, s
