"""Pointer block-mask builder: the host side of the reference's
``SpectralBias.build_pointer_blockmask`` (model/attn_bias.py:623-874).

``PointerBlockMaskBuilder`` carries the same knobs as SpectralBias's pointer
options (model/attn_bias.py:99-113) and the same schedule setters
(model/attn_bias.py:342-377), but keeps the schedule state as host integers,
so building a mask needs no device->host sync (the reference reads three
device scalars with ``.item()`` per call, model/attn_bias.py:702,703,769).
Every build is one launch of the CUDA builder through the C ABI.

The result, ``ScopeBlockMask``, holds the BlockMask fields the attention
kernels read (``kv_num_blocks``, ``kv_indices``) plus the q-side bitmap that
replaces torch's dense transpose; ``to_flex()`` turns it into a torch
``BlockMask`` when the reference layout is wanted.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import torch

from . import _lib

EOD_TOKEN_ID = 50256


@dataclass
class ScopeBlockMask:
    """Block-sparse visibility of one layer (B = 1), in the BlockMask layout.

    kv_num_blocks [1,H,QB] int32, kv_indices [1,H,QB,W] int32 (the first
    kv_num_blocks entries of a row are the visible kv blocks, ascending);
    q_bitmap [H,QB,ceil(QB/32)] int32 (bit qb of row (h,kb) set when kb is
    visible from qb); block_info [4,QB] int32 (doc-start blocks for the
    pointer clamp and local band, per-block doc min/max); docs [T] int32 or
    None (then the mask_mod is plain causal)."""
    kv_num_blocks: torch.Tensor
    kv_indices: torch.Tensor
    q_bitmap: torch.Tensor
    block_info: torch.Tensor
    BLOCK_SIZE: tuple
    seq_lengths: tuple
    docs: torch.Tensor | None = None
    stats: torch.Tensor | None = None
    r_m: torch.Tensor | None = None
    centres: torch.Tensor | None = None
    max_kv: int = 0
    stats_layout: tuple = ()
    _q_cache: tuple | None = field(default=None, repr=False)
    _tiles: "ScopeBlockMask | None" = field(default=None, repr=False)

    @property
    def num_heads(self) -> int:
        return self.kv_num_blocks.shape[1]

    @property
    def num_q_blocks(self) -> int:
        return self.kv_num_blocks.shape[2]

    def q_lists(self, with_indices: bool = True):
        """(q_num_blocks [1,H,KB], q_indices [1,H,KB,QB]) in torch's
        _transpose_ordered layout, from the bitmap (one kernel launch)."""
        if self._q_cache is None or (with_indices and self._q_cache[1] is None):
            H, QB = self.num_heads, self.num_q_blocks
            dev = self.kv_num_blocks.device
            q_num = torch.empty(1, H, QB, dtype=torch.int32, device=dev)
            q_idx = torch.empty(1, H, QB, QB, dtype=torch.int32, device=dev) if with_indices else None
            st = _lib.lib().scope_mask_transpose(self.q_bitmap.data_ptr(), H, QB, q_num.data_ptr(),
                                                 _lib.ptr(q_idx), _stream(dev))
            _lib.check(st, "scope_mask_transpose")
            self._q_cache = (q_num, q_idx)
        return self._q_cache

    @property
    def q_num_blocks(self):
        return self.q_lists(False)[0]

    @property
    def q_indices(self):
        return self.q_lists(True)[1]

    def kernel_tiles(self, tile: int = 128) -> "ScopeBlockMask":
        """The same visibility on `tile`-row blocks, the tile the attention
        kernels run: a mask built at block_size 2*tile (config C5 builds at
        256) is refined by one kernel launch (fine lists, q-side bitmap,
        block_info at the fine block size); a mask already at `tile` is
        returned as is."""
        bs = self.BLOCK_SIZE[0]
        if bs == tile:
            return self
        if bs != 2 * tile:
            raise ValueError(f"block size {bs}: the kernels tile at {tile} (block sizes {tile} and {2 * tile})")
        if self._tiles is None:
            H, QB = self.num_heads, self.num_q_blocks
            T = self.seq_lengths[0]
            dev = self.kv_num_blocks.device
            QF = 2 * QB
            kvi = self.kv_indices[0]
            w = 2 * kvi.shape[-1]
            kv_num = torch.empty(1, H, QF, dtype=torch.int32, device=dev)
            kv_idx = torch.zeros(1, H, QF, w, dtype=torch.int32, device=dev)
            qbm = torch.zeros(H, QF, (QF + 31) // 32, dtype=torch.int32, device=dev)
            st = _lib.lib().scope_mask_refine(self.kv_num_blocks.data_ptr(), kvi.data_ptr(), H, QB, kvi.shape[-1],
                                              kv_num.data_ptr(), kv_idx.data_ptr(), w, qbm.data_ptr(),
                                              _lib.err_word_ptr(dev), _stream(dev))
            _lib.check(st, "scope_mask_refine")
            info = block_info(self.docs, T, tile, device=dev)
            self._tiles = ScopeBlockMask(kv_num, kv_idx, qbm, info, (tile, tile), self.seq_lengths, docs=self.docs,
                                         max_kv=2 * self.max_kv)
        return self._tiles

    @classmethod
    def from_flex(cls, block_mask, docs: torch.Tensor | None = None) -> "ScopeBlockMask":
        """The kernels' view of a torch ``BlockMask`` (B = 1), e.g. the one the
        reference's ``build_pointer_blockmask`` returns (model/attn_bias.py:
        851-874): its kv lists as they are, the q-side bitmap from the lists
        (one kernel launch), ``block_info`` from ``docs``.  A C ABI cannot run
        the BlockMask's ``mask_mod``, so the document ids it captures travel as
        ``docs`` ([T], None for a plain causal mask_mod); the reference's
        document_causal mask_mod (model/attn_bias.py:674-679) is the one the
        kernels apply.  Full blocks (listed blocks that skip the mask_mod) are
        not supported: the reference's masks have none, and a mask with any is
        rejected (checking that reads one device flag back to the host)."""
        bs_q, bs_kv = block_mask.BLOCK_SIZE
        if bs_q != bs_kv or bs_q not in (128, 256):
            raise ValueError(f"BlockMask.BLOCK_SIZE {block_mask.BLOCK_SIZE}: the kernels take square 128 or 256 blocks")
        kvn, kvi = block_mask.kv_num_blocks, block_mask.kv_indices
        if kvn.dim() != 3 or kvn.shape[0] != 1 or kvi.dim() != 4 or kvi.shape[:3] != kvn.shape:
            raise ValueError("BlockMask lists must be kv_num_blocks [1,H,QB] and kv_indices [1,H,QB,W]")
        fkn = block_mask.full_kv_num_blocks
        if fkn is not None and bool((fkn != 0).any()):
            raise ValueError("BlockMask with full blocks: the kernels apply the mask_mod to every listed block")
        T_q, T_kv = block_mask.seq_lengths
        H, QB = kvn.shape[1], kvn.shape[2]
        if T_q != T_kv or T_q != QB * bs_q:
            raise ValueError("BlockMask must cover T query and T key positions (T = QB * BLOCK_SIZE)")
        dev = kvn.device
        kvn = kvn.to(torch.int32).contiguous()
        kvi = kvi.to(torch.int32).contiguous()
        words = (QB + 31) // 32
        qbm = torch.zeros(H, QB, words, dtype=torch.int32, device=dev)
        st = _lib.lib().scope_mask_bitmap_from_lists(kvn.data_ptr(), kvi.data_ptr(), H, QB, kvi.shape[-1],
                                                     qbm.data_ptr(), _lib.err_word_ptr(dev), _stream(dev))
        _lib.check(st, "scope_mask_bitmap_from_lists")
        d = None if docs is None else docs.to(device=dev, dtype=torch.int32).contiguous()
        info = block_info(d, T_q, bs_q, device=dev)
        return cls(kvn, kvi, qbm, info, (bs_q, bs_q), (T_q, T_q), docs=d, max_kv=kvi.shape[-1])

    def pointer_stats(self) -> dict:
        """The reference's pointer statistics (model/attn_bias.py:839-849):
        kv_unique_hist, ptr_radius_hist, ptr_extra_sum_hist, radius0 count."""
        if self.stats is None:
            return {}
        a, b, c = self.stats_layout
        s = self.stats
        return {"kv_unique_hist": s[:a], "ptr_radius_hist": s[a:a + b],
                "ptr_extra_sum_hist": s[a + b:a + b + c], "radius0_count": s[a + b + c]}

    def to_flex(self):
        """A torch BlockMask with the same visibility (every block partial,
        document-causal mask_mod), for interop with flex_attention."""
        from torch.nn.attention.flex_attention import BlockMask
        docs = self.docs

        def document_causal(b, h, q_idx, kv_idx):
            causal = q_idx >= kv_idx
            if docs is None:
                return causal
            return causal & (docs[q_idx] == docs[kv_idx])

        q_num, q_idx = self.q_lists(True)
        H, QB = self.num_heads, self.num_q_blocks
        kvi = self.kv_indices
        if kvi.shape[-1] != QB:
            pad = torch.empty(1, H, QB, QB, dtype=torch.int32, device=kvi.device)
            w = min(kvi.shape[-1], QB)
            pad[..., :w] = kvi[..., :w]
            if w < QB:
                pad[..., w:] = kvi[..., :1]
            kvi = pad
        z = torch.zeros_like(self.kv_num_blocks)
        zi = torch.zeros_like(kvi)
        return BlockMask(self.seq_lengths, self.kv_num_blocks, kvi, z, zi, q_num, q_idx, z, zi,
                         self.BLOCK_SIZE, document_causal)


def _stream(dev) -> int:
    if dev.type != "cuda":
        raise RuntimeError("scope_b200 ops run on CUDA tensors only")
    return torch.cuda.current_stream(dev).cuda_stream


def block_info(docs: torch.Tensor | None, T: int, block_size: int, *, device, doc_clamp: bool = True,
               reset_active: bool = False, reset_len: int = 0) -> torch.Tensor:
    """[4, QB] int32: doc_start_blk_ptr, doc_start_blk_local (model/attn_bias.py:681-709),
    per-block doc min and max."""
    if T % block_size:
        raise ValueError(f"T={T} is not a multiple of block_size={block_size}")
    QB = T // block_size
    out = torch.empty(4, QB, dtype=torch.int32, device=device)
    d = None
    if docs is not None:
        d = docs.to(device=device, dtype=torch.int32).contiguous()
        if d.numel() != T:
            raise ValueError("docs must have T entries")
    st = _lib.lib().scope_block_info(_lib.ptr(d), T, block_size, int(doc_clamp), int(reset_active),
                                     int(reset_len), out.data_ptr(), _stream(torch.device(device)))
    _lib.check(st, "scope_block_info")
    return out


def build_mask(*, H: int, T: int, block_size: int, M: int, device,
               docs: torch.Tensor | None = None,
               sel_logits: torch.Tensor | None = None, sel_gumbel: torch.Tensor | None = None,
               sel_tau: float = 1.0,
               delta_rep: torch.Tensor | None = None, budget_rep: torch.Tensor | None = None,
               peak_gumbel: torch.Tensor | None = None, gumbel_k: int = 0, gumbel_tau: float = 1.0,
               local_blocks: int = 1, half_blocks: int = 0, half_active: int | None = None,
               ptr_enabled: bool = True, global_blocks: int = 0, global_active: int | None = None,
               radius_mode: str = "pi", budget_blocks: int = 0, budget_is_total: bool = True,
               budget_temp: float = 1.0, doc_clamp: bool = True, reset_active: bool = False,
               reset_len: int = 0, layout: str = "compact", stats: bool = False,
               debug: bool = False) -> ScopeBlockMask:
    """One call of the CUDA builder with every knob explicit (resolved as
    model/attn_bias.py:666-672,724-734,810-820 resolve them)."""
    dev = torch.device(device)
    if T % block_size:
        raise ValueError(f"T={T} is not a multiple of block_size={block_size}")
    QB = T // block_size
    if not (1 <= M <= 16):
        raise ValueError("M (pointer peaks) must be in [1, 16]")
    L = min(max(1, int(local_blocks)), QB)
    p = max(0, int(half_blocks))
    ha = p if half_active is None else int(half_active)
    G = min(max(0, int(global_blocks)), QB)
    ga = G if global_active is None else min(max(int(global_active), 0), G)
    if radius_mode not in ("fixed", "pi"):
        raise ValueError("radius_mode must be one of: fixed|pi")
    bv = max(0, int(budget_blocks))
    if budget_is_total:
        cap = L + M + 2 * M * p
        extra = max(min(bv, cap) - L - M, 0)
    else:
        extra = bv
    brem = min(extra // 2, M * p)
    info = block_info(docs, T, block_size, device=dev, doc_clamp=doc_clamp,
                      reset_active=reset_active, reset_len=reset_len)
    max_kv = int(_lib.lib().scope_mask_max_kv(L, M, p, G))
    if layout == "flex_padded":
        W = QB
    elif layout == "compact":
        W = max_kv
    else:
        raise ValueError("layout must be compact|flex_padded")
    kv_num = torch.empty(1, H, QB, dtype=torch.int32, device=dev)
    kv_idx = torch.empty(1, H, QB, W, dtype=torch.int32, device=dev)
    words = (QB + 31) // 32
    qbm = torch.zeros(H, QB, words, dtype=torch.int32, device=dev)
    n_stats = (max_kv + 1) + (p + 1) + (max(1, p * M) + 1) + 1
    st_t = torch.zeros(n_stats, dtype=torch.int32, device=dev) if stats else None
    r_m = torch.empty(H, QB, M, dtype=torch.int32, device=dev) if debug else None
    cen = torch.empty(H, QB, M, dtype=torch.int32, device=dev) if debug else None

    a = _lib.ScopeMaskArgs()
    a.H, a.QB, a.M, a.block_size = H, QB, M, block_size
    keep = []
    if sel_logits is not None:
        if delta_rep is not None:
            raise ValueError("pass exactly one of: pointer logits | delta_rep")
        for t in (sel_logits, sel_gumbel):
            if t is None or t.dtype != torch.float32 or t.dim() != 3 or t.stride(-1) != 1:
                raise ValueError("pointer logits and Gumbel noise must be float32 [H,QB,QB] with unit last stride")
        if sel_logits.shape != sel_gumbel.shape or sel_logits.stride() != sel_gumbel.stride():
            raise ValueError("pointer logits and Gumbel noise must share shape and strides")
        if sel_logits.shape[0] != H or sel_logits.shape[1] != QB or sel_logits.shape[2] < QB:
            raise ValueError("pointer logits must be [H, QB, >=QB]")
        a.sel_logits, a.sel_gumbel = sel_logits.data_ptr(), sel_gumbel.data_ptr()
        a.sel_head_stride, a.sel_row_stride = sel_logits.stride(0), sel_logits.stride(1)
        a.sel_tau = max(float(sel_tau), 1e-6)
    elif delta_rep is not None:
        if delta_rep.dtype != torch.float32 or tuple(delta_rep.shape) != (H, QB, M):
            raise ValueError("delta_rep must be float32 [H, QB, M]")
        a.delta_rep = delta_rep.data_ptr()
        a.delta_head_stride, a.delta_row_stride, a.delta_m_stride = delta_rep.stride()
    else:
        raise ValueError("pass exactly one of: pointer logits | delta_rep")
    if budget_rep is not None:
        if budget_rep.dtype != torch.float32 or tuple(budget_rep.shape) != (H, QB, M):
            raise ValueError("budget_rep must be float32 [H, QB, M]")
        a.budget_rep = budget_rep.data_ptr()
        a.budget_head_stride, a.budget_row_stride, a.budget_m_stride = budget_rep.stride()
    elif radius_mode == "pi" and brem > 0:
        raise ValueError("budget_rep is required for the 'pi' radius mode with a positive budget")
    k = int(gumbel_k)
    if peak_gumbel is not None and 0 < k < M and p > 0:
        pg = peak_gumbel.to(device=dev, dtype=torch.float32).contiguous()
        keep.append(pg)
        a.peak_gumbel, a.gumbel_k, a.gumbel_tau = pg.data_ptr(), k, max(float(gumbel_tau), 1e-6)
    a.block_info = info.data_ptr()
    a.local_blocks, a.half_blocks, a.half_active = L, p, ha
    a.ptr_enabled = int(bool(ptr_enabled))
    a.global_max, a.global_active = G, ga
    a.radius_mode = 1 if radius_mode == "pi" else 0
    a.budget_rem = brem
    a.budget_temp = max(float(budget_temp), 1e-6)
    a.kv_num, a.kv_indices = kv_num.data_ptr(), kv_idx.data_ptr()
    a.kv_stride, a.flex_padded = W, int(layout == "flex_padded")
    a.q_bitmap = qbm.data_ptr()
    a.r_m_out, a.centres_out = _lib.ptr(r_m), _lib.ptr(cen)
    a.stats = _lib.ptr(st_t)
    a.err_flag = _lib.err_word_ptr(dev)
    st = _lib.lib().scope_mask_build(ctypes.byref(a), _stream(dev))
    _lib.check(st, "scope_mask_build")
    d = None if docs is None else docs.to(device=dev, dtype=torch.int32)
    return ScopeBlockMask(kv_num, kv_idx, qbm, info, (block_size, block_size), (T, T), docs=d, stats=st_t,
                          r_m=r_m, centres=cen, max_kv=max_kv,
                          stats_layout=(max_kv + 1, p + 1, max(1, p * M) + 1))


class PointerBlockMaskBuilder:
    """Pointer-mask knobs and schedule state of SpectralBias
    (model/attn_bias.py:75-218, 342-377), building masks on the GPU."""

    def __init__(self, *, num_heads: int, M: int, use_pointer_mask: bool = True,
                 pointer_local_blocks: int = 16, pointer_half_blocks: int = 4, pointer_global_blocks: int = 0,
                 pointer_budget_blocks: int = 0, pointer_budget_is_total: bool = True,
                 pointer_budget_temp: float = 1.0, pointer_radius_mode: str = "pi",
                 pointer_qblock_rep: str = "last", pointer_doc_clamp: bool = True,
                 gumbel_topk: bool = False, gumbel_topk_k: int = 0, gumbel_topk_tau: float = 1.0,
                 gumbel_topk_seed: int = 0, pointer_reset_len: int = 0, eps: float = 1e-9,
                 debug_stats: bool = False):
        if M <= 0:
            raise ValueError("M must be positive")
        self.num_heads, self.M = int(num_heads), int(M)
        self.use_pointer_mask = bool(use_pointer_mask)
        self.pointer_local_blocks = int(pointer_local_blocks)
        self.pointer_half_blocks = int(pointer_half_blocks)
        self.pointer_global_blocks = int(pointer_global_blocks)
        self.pointer_budget_blocks = int(pointer_budget_blocks)
        self.pointer_budget_is_total = bool(pointer_budget_is_total)
        self.pointer_budget_temp = float(pointer_budget_temp)
        self.pointer_radius_mode = str(pointer_radius_mode).strip().lower()
        if self.pointer_radius_mode not in {"fixed", "pi"}:
            raise ValueError("pointer_radius_mode must be one of: fixed|pi")
        self.pointer_qblock_rep = str(pointer_qblock_rep)
        if self.pointer_qblock_rep not in {"last", "mean"}:
            raise ValueError("pointer_qblock_rep must be one of: last|mean")
        self.pointer_doc_clamp = bool(pointer_doc_clamp)
        self.gumbel_topk = bool(gumbel_topk)
        self.gumbel_topk_k = int(gumbel_topk_k)
        self.gumbel_topk_tau = float(gumbel_topk_tau)
        self.pointer_reset_len = int(pointer_reset_len)
        self.eps = float(eps)
        self.debug_stats = bool(debug_stats)
        self.training = True
        # schedule state (host integers; the reference keeps them in device buffers)
        self._pointer_mask_active = 1 if self.use_pointer_mask else 0
        self._pointer_half_blocks_active = self.pointer_half_blocks if self.use_pointer_mask else 0
        self._pointer_global_blocks_active = self.pointer_global_blocks if self.use_pointer_mask else 0
        self._pointer_reset_active = 0
        self._pointer_reset_len_active = max(0, self.pointer_reset_len)
        self._gumbel_seed = int(gumbel_topk_seed)

    def train(self, mode: bool = True):
        self.training = bool(mode)
        return self

    def eval(self):
        return self.train(False)

    def set_pointer_mask_state(self, *, enabled: bool, half_blocks: int, global_blocks: int | None = None):
        half_blocks = int(half_blocks)
        if half_blocks < 0:
            raise ValueError("half_blocks must be >= 0")
        self._pointer_mask_active = 1 if enabled else 0
        self._pointer_half_blocks_active = min(half_blocks, self.pointer_half_blocks)
        if global_blocks is not None:
            gb = int(global_blocks)
            if gb < 0:
                raise ValueError("global_blocks must be >= 0")
            self._pointer_global_blocks_active = min(gb, self.pointer_global_blocks)

    def set_pointer_reset_state(self, *, enabled: bool, reset_len: int):
        reset_len = int(reset_len)
        if reset_len < 0:
            raise ValueError("reset_len must be >= 0")
        self._pointer_reset_active = 1 if enabled else 0
        self._pointer_reset_len_active = reset_len if enabled else 0

    def set_gumbel_seed(self, *, seed: int):
        self._gumbel_seed = int(seed)

    def _representatives(self, x: torch.Tensor, block_size: int) -> torch.Tensor:
        """[1,H,T,M] -> [H,QB,M] per model/attn_bias.py:714-719."""
        _, H, T, M = x.shape
        QB = T // block_size
        if self.pointer_qblock_rep == "last":
            return x[0, :, block_size - 1::block_size, :]
        return x[0].reshape(H, QB, block_size, M).mean(dim=2).contiguous()

    def _gumbel_noise(self, H, QB, device) -> torch.Tensor:
        """The reference's peak-masking noise: torch.rand from a generator
        seeded with the Gumbel seed on the mask's device, then
        g = -log(-log(u + eps) + eps) (model/attn_bias.py:768-771)."""
        gen = torch.Generator(device=device)
        gen.manual_seed(int(self._gumbel_seed))
        u = torch.rand((H, QB, self.M), device=device, generator=gen, dtype=torch.float32)
        return -torch.log(-torch.log(u + self.eps) + self.eps)

    def _common(self, *, T, block_size, local_blocks, ptr_half_blocks, pointer_budget_blocks, global_blocks):
        lb = self.pointer_local_blocks if local_blocks is None else int(local_blocks)
        ph = self.pointer_half_blocks if ptr_half_blocks is None else int(ptr_half_blocks)
        bb = self.pointer_budget_blocks if pointer_budget_blocks is None else int(pointer_budget_blocks)
        gact = self._pointer_global_blocks_active if global_blocks is None else int(global_blocks)
        return dict(T=T, block_size=block_size, M=self.M, local_blocks=lb, half_blocks=ph,
                    half_active=self._pointer_half_blocks_active, ptr_enabled=bool(self._pointer_mask_active),
                    global_blocks=self.pointer_global_blocks, global_active=gact,
                    radius_mode=self.pointer_radius_mode, budget_blocks=bb,
                    budget_is_total=self.pointer_budget_is_total, budget_temp=self.pointer_budget_temp,
                    doc_clamp=self.pointer_doc_clamp, reset_active=bool(self._pointer_reset_active),
                    reset_len=self._pointer_reset_len_active)

    @torch.no_grad()
    def build_pointer_blockmask(self, *, input_seq=None, docs=None, delta_star, pi, budget_logits,
                                block_size: int = 128, local_blocks=None, ptr_half_blocks=None,
                                pointer_budget_blocks=None, global_blocks=None, eod_token_id: int = EOD_TOKEN_ID,
                                layout: str = "compact") -> ScopeBlockMask:
        """Same arguments and meaning as SpectralBias.build_pointer_blockmask
        (model/attn_bias.py:623-649)."""
        if (input_seq is None) == (docs is None):
            raise ValueError("pass exactly one of: input_seq|docs")
        if docs is None:
            docs = (input_seq == eod_token_id).cumsum(0)
        B, H, T, M = delta_star.shape
        if B != 1 or H != self.num_heads or M != self.M or docs.numel() != T or T % block_size:
            raise ValueError("delta_star must be [1, num_heads, T, M] with T a multiple of block_size")
        if tuple(pi.shape) != (B, H, T, M) or tuple(budget_logits.shape) != (B, H, T, M):
            raise ValueError("pi and budget_logits must match delta_star")
        QB = T // block_size
        drep = self._representatives(delta_star.float(), block_size).contiguous()
        brep = self._representatives(budget_logits.float(), block_size).contiguous()
        kw = self._common(T=T, block_size=block_size, local_blocks=local_blocks, ptr_half_blocks=ptr_half_blocks,
                          pointer_budget_blocks=pointer_budget_blocks, global_blocks=global_blocks)
        pg = None
        k = 0
        if self.training and self.gumbel_topk and max(0, kw["half_blocks"]) > 0:
            k = self.gumbel_topk_k if 0 < self.gumbel_topk_k <= M else M
            if k < M:
                pg = self._gumbel_noise(H, QB, delta_star.device)
        return build_mask(H=H, device=delta_star.device, docs=docs, delta_rep=drep, budget_rep=brep,
                          peak_gumbel=pg, gumbel_k=k, gumbel_tau=self.gumbel_topk_tau, layout=layout,
                          stats=self.debug_stats, **kw)

    @torch.no_grad()
    def select_and_build(self, *, pointer_logits, gumbel, tau: float, docs=None, budget_rep=None,
                         block_size: int = 128, local_blocks=None, ptr_half_blocks=None,
                         pointer_budget_blocks=None, global_blocks=None, layout: str = "compact",
                         stats: bool | None = None, debug: bool = False) -> ScopeBlockMask:
        """Fused pointer selection + build: Gumbel top-M over the causal
        candidate blocks of ``pointer_logits`` [H,QB,QB] picks the M pointer
        centres per query block, then the reference's radius allocation,
        windows and packing follow."""
        H, QB, _ = pointer_logits.shape
        T = QB * block_size
        kw = self._common(T=T, block_size=block_size, local_blocks=local_blocks, ptr_half_blocks=ptr_half_blocks,
                          pointer_budget_blocks=pointer_budget_blocks, global_blocks=global_blocks)
        return build_mask(H=H, device=pointer_logits.device, docs=docs, sel_logits=pointer_logits,
                          sel_gumbel=gumbel, sel_tau=tau, budget_rep=budget_rep, layout=layout,
                          stats=self.debug_stats if stats is None else stats, debug=debug, **kw)
