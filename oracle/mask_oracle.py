"""Numpy restatement of the SCOPE pointer block-mask builder (TEST ORACLE ONLY).

Follows ``SpectralBias.build_pointer_blockmask`` in the reference
(model/attn_bias.py:623-874) step by step, with every float32 operation done
in float32 in the same order as the reference so that the integer outputs
(``kv_num_blocks``, ``kv_indices``, ``q_num_blocks``, ``q_indices``) are
bit-identical.  The one op whose last bit is platform dependent is the
sigmoid of the radius allocation (torch CPU, numpy and CUDA each round
``1/(1+exp(-x))`` slightly differently); ``radius_alloc`` therefore also
returns a per-row decision margin so that tests can tell an ulp tie from a
real mismatch.

It also restates the pointer *selection* stage used by the benchmark
configurations (Gumbel top-k over per-candidate pointer logits), which the
reference does not have as a separate function: its output (block centres)
enters the reference algorithm exactly as the pointer centres computed at
model/attn_bias.py:779-784 would.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# document / reset starts  (model/attn_bias.py:681-709)
# ---------------------------------------------------------------------------
def doc_start_blocks(docs, block_size: int, *, doc_clamp: bool = True,
                     reset_active: bool = False, reset_len: int = 0):
    """Per query block: (doc_start_blk_ptr, doc_start_blk_local) as int32 [QB].

    doc_start_token[t] is the most recent change point of ``docs`` at or
    before t (model/attn_bias.py:688-691); the pointer clamp uses the
    representative (last) token of the block, the local band the first token
    (model/attn_bias.py:693-697); reset segments (model/attn_bias.py:703-709).
    """
    docs = np.asarray(docs)
    T = docs.shape[0]
    assert T % block_size == 0
    QB = T // block_size
    change = np.ones(T, dtype=bool)
    change[1:] = docs[1:] != docs[:-1]
    tok = np.arange(T, dtype=np.int64)
    dst = np.maximum.accumulate(np.where(change, tok, 0))
    qb = np.arange(QB, dtype=np.int64)
    t_rep = (qb + 1) * block_size - 1
    start_tok = qb * block_size
    dsp = dst[t_rep] // block_size
    dsl = dst[start_tok] // block_size
    if not doc_clamp:
        dsp = np.zeros_like(dsp)
        dsl = np.zeros_like(dsl)
    if reset_active and reset_len > 0:
        seg_p = ((t_rep // reset_len) * reset_len) // block_size
        seg_l = ((start_tok // reset_len) * reset_len) // block_size
        dsp = np.maximum(dsp, seg_p)
        dsl = np.maximum(dsl, seg_l)
    return dsp.astype(np.int32), dsl.astype(np.int32)


def doc_block_ranges(docs, block_size: int):
    """Per block min/max document id (int32 [QB] each); used to classify
    attention tiles as fully visible or needing the element mask."""
    d = np.asarray(docs).reshape(-1, block_size)
    return d.min(axis=1).astype(np.int32), d.max(axis=1).astype(np.int32)


# ---------------------------------------------------------------------------
# radius allocation  (model/attn_bias.py:721-761)
# ---------------------------------------------------------------------------
def resolve_budget_rem(*, M: int, local_blocks: int, half_blocks: int,
                       budget_blocks: int, budget_is_total: bool) -> int:
    """Integer budget of extra pointer radius per (head, q-block)
    (model/attn_bias.py:724-734).  ``local_blocks`` is the resolved band."""
    budget_val = max(0, int(budget_blocks))
    if budget_is_total:
        cap = int(local_blocks + M + 2 * M * int(half_blocks))
        total = min(budget_val, cap)
        extra = max(total - int(local_blocks) - int(M), 0)
    else:
        extra = budget_val
    rem = extra // 2
    return min(rem, M * int(half_blocks))


def _sigmoid_f32(x):
    x = np.asarray(x, dtype=F32)
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def radius_alloc(budget_rep, *, mode: str, budget_rem: int, budget_temp: float,
                 half_blocks: int, half_active: int, ptr_enabled: bool):
    """Per-peak pointer radii r_m (int32 [H,QB,M]) and a decision margin [H,QB].

    "pi" mode: stick-breaking over sigmoid(budget/temp) of the integer budget,
    then largest-remainder rounding (model/attn_bias.py:735-758); "fixed"
    mode: every peak gets the scheduled radius (model/attn_bias.py:721-722).
    Then the schedule cap and the enable flag (model/attn_bias.py:760-761).

    The margin is the distance of the float32 decision quantities to the
    nearest flip (an alloc value to an integer, or the two fractional parts
    either side of the rounding cut-off); a row with margin below ~1e-5 can
    legitimately differ between devices by one ulp of the sigmoid.
    """
    b = np.asarray(budget_rep, dtype=F32)
    H, QB, M = b.shape
    margin = np.full((H, QB), np.inf, dtype=np.float64)
    if mode == "fixed":
        r = np.full((H, QB, M), int(half_active), dtype=np.int32)
    elif budget_rem <= 0:
        r = np.zeros((H, QB, M), dtype=np.int32)
    else:
        temp = F32(max(float(budget_temp), 1e-6))
        u = (b / temp).astype(F32)
        rem = np.full((H, QB), F32(budget_rem), dtype=F32)
        alloc = np.zeros((H, QB, M), dtype=F32)
        for m in range(M - 1):
            v = _sigmoid_f32(u[..., m])
            bb = (v * rem).astype(F32)
            alloc[..., m] = bb
            rem = (rem - bb).astype(F32)
        alloc[..., M - 1] = rem
        floor = np.floor(alloc).astype(F32)
        frac = (alloc - floor).astype(F32)
        floor_sum = floor.astype(np.float64).sum(-1).astype(np.int64)
        rem_int = np.clip(budget_rem - floor_sum, 0, M)
        # stable descending rank of the fractional parts (ties: lower index first)
        order = np.argsort(-frac, axis=-1, kind="stable")
        rank = np.argsort(order, axis=-1, kind="stable")
        add = (rank < rem_int[..., None]).astype(F32)
        extra = floor + add
        r = np.clip(extra.astype(np.int32), 0, int(half_blocks))
        # decision margin
        # (an alloc value is never negative, so only integers >= 1 can flip its floor)
        a64 = alloc.astype(np.float64)
        near = np.round(a64)
        m_int = np.where(near >= 1, np.abs(a64 - near) / np.maximum(a64, 1.0), np.inf).min(-1)
        fs = -np.sort(-frac.astype(np.float64), axis=-1)
        gaps = np.full((H, QB), np.inf)
        for h in range(H):
            for q in range(QB):
                k = int(rem_int[h, q])
                if 0 < k < M:
                    gaps[h, q] = fs[h, q, k - 1] - fs[h, q, k]
        margin = np.minimum(m_int, gaps)
    r = np.minimum(r, int(half_active)).astype(np.int32)
    if not ptr_enabled:
        r = np.zeros_like(r)
    return r, margin


def gumbel_peak_mask(r_m, budget_rep, g, *, k: int, tau: float):
    """Keep the radii of the top-k peaks of budget/tau + g, zero the rest
    (model/attn_bias.py:763-777).  ``g`` is the supplied Gumbel noise
    -log(-log(u+eps)+eps) [H,QB,M] float32.  Ties: lower index first."""
    M = r_m.shape[-1]
    if k <= 0 or k > M:
        k = M
    if k >= M:
        return r_m
    t = F32(max(float(tau), 1e-6))
    scores = ((np.asarray(budget_rep, F32) / t).astype(F32) + np.asarray(g, F32)).astype(F32)
    order = np.argsort(-scores, axis=-1, kind="stable")[..., :k]
    keep = np.zeros(r_m.shape, dtype=bool)
    np.put_along_axis(keep, order, True, axis=-1)
    return np.where(keep, r_m, 0).astype(np.int32)


def gumbel_from_uniform(u, eps: float = 1e-9):
    """g = -log(-log(u + eps) + eps) in float32 (model/attn_bias.py:771)."""
    u = np.asarray(u, F32)
    e = F32(eps)
    return (-np.log(-np.log(u + e) + e)).astype(F32)


# ---------------------------------------------------------------------------
# pointer centres  (model/attn_bias.py:779-784)
# ---------------------------------------------------------------------------
def centres_from_delta(delta_rep, block_size: int, dsp, *, ptr_enabled: bool):
    """Centre block of each peak from the representative Δ* (float32)."""
    d = np.asarray(delta_rep, F32)
    H, QB, M = d.shape
    qb = np.arange(QB, dtype=np.int64)
    t_rep = ((qb + 1) * block_size - 1).astype(F32)
    key = (t_rep[None, :, None] - d).astype(F32)
    key = np.maximum(key, F32(0.0))
    c = (key.astype(np.int64) // block_size)
    c = np.minimum(c, qb[None, :, None])
    if not ptr_enabled:
        c = np.broadcast_to(qb[None, :, None], c.shape).copy()
    c = np.maximum(c, np.asarray(dsp, np.int64)[None, :, None])
    return c.astype(np.int32)


def clamp_centres(centres, dsp, *, ptr_enabled: bool):
    """The same clamps as centres_from_delta for centres given as blocks
    (min with qb, disabled -> qb, max with the doc start)."""
    c = np.asarray(centres, np.int64)
    H, QB, M = c.shape
    qb = np.arange(QB, dtype=np.int64)
    c = np.minimum(c, qb[None, :, None])
    if not ptr_enabled:
        c = np.broadcast_to(qb[None, :, None], c.shape).copy()
    c = np.maximum(c, np.asarray(dsp, np.int64)[None, :, None])
    return c.astype(np.int32)


# ---------------------------------------------------------------------------
# pointer selection stage (benchmark configurations; not a reference function)
# ---------------------------------------------------------------------------
def select_pointer_blocks(logits, g, *, M: int, tau: float):
    """Gumbel top-M over causal candidate blocks.

    scores[h,qb,kb] = logits/tau + g for kb <= qb; the M best (descending
    score, ties to the lower block) become the pointer centres in that order.
    If fewer than M candidates exist (qb+1 < M) the remaining centres are qb.
    Returns int32 [H,QB,M].
    """
    lg = np.asarray(logits, F32)
    gg = np.asarray(g, F32)
    H, QB, C = lg.shape
    assert C == QB
    t = F32(max(float(tau), 1e-6))
    s = ((lg / t).astype(F32) + gg).astype(F32)
    kb = np.arange(QB)
    causal = kb[None, :] <= np.arange(QB)[:, None]       # [qb, kb]
    s = np.where(causal[None], s, -np.inf).astype(np.float64)
    # stable sort on (-score); -inf candidates sort last, then by index
    order = np.argsort(-s, axis=-1, kind="stable")[..., :M]
    if order.shape[-1] < M:          # fewer candidate blocks than peaks
        order = np.concatenate([order, np.zeros((H, QB, M - order.shape[-1]), order.dtype)], -1)
    out = order.astype(np.int32)
    nvalid = np.minimum(np.arange(QB) + 1, M)
    slot = np.arange(M)
    out = np.where(slot[None, None, :] < nvalid[None, :, None], out,
                   np.arange(QB, dtype=np.int32)[None, :, None])
    return out.astype(np.int32)


# ---------------------------------------------------------------------------
# window pieces, dedup and pack  (model/attn_bias.py:786-862)
# ---------------------------------------------------------------------------
def window_pieces(centres, r_m, dsp, dsl, *, QB: int, local_blocks: int, half_blocks: int,
                  global_max: int, global_active: int):
    """Concatenate local band, pointer windows and global anchors into
    kv_blocks [H,QB,MAX_KV] (model/attn_bias.py:786-825).

    ``local_blocks`` is the resolved band min(max(1,L),QB); ``global_max`` is
    min(pointer_global_blocks, QB); ``global_active`` the active count."""
    c = np.asarray(centres, np.int64)
    r = np.asarray(r_m, np.int64)
    H, _, M = c.shape
    qb = np.arange(QB, dtype=np.int64)
    dsp = np.asarray(dsp, np.int64)
    dsl = np.asarray(dsl, np.int64)
    pieces = []
    offs = np.arange(local_blocks, dtype=np.int64)
    local = np.maximum(qb[:, None] - offs[None, :], 0)
    local = np.maximum(local, dsl[:, None])
    pieces.append(np.broadcast_to(local[None], (H, QB, local_blocks)))
    p = int(half_blocks)
    if p > 0:
        o = np.arange(-p, p + 1, dtype=np.int64)
        active = np.abs(o)[None, None, None, :] <= r[..., None]
        ptr = c[..., None] + o[None, None, None, :]
        ptr = np.clip(ptr, 0, QB - 1)
        ptr = np.minimum(ptr, qb[None, :, None, None])
        ptr = np.maximum(ptr, dsp[None, :, None, None])
        ptr = np.where(active, ptr, c[..., None])
        pieces.append(ptr.reshape(H, QB, M * (2 * p + 1)))
    else:
        pieces.append(c)
    if global_max > 0:
        gi = np.arange(global_max, dtype=np.int64)
        g = np.minimum(dsp[:, None] + gi[None, :], qb[:, None])
        ga = min(max(int(global_active), 0), global_max)
        g = np.where(gi[None, :] < ga, g, qb[:, None])
        pieces.append(np.broadcast_to(g[None], (H, QB, global_max)))
    return np.concatenate(pieces, axis=-1).astype(np.int32)


def dedup_pack(kv_blocks, QB: int):
    """Sort, keep the first of each run, then order unique-ascending followed
    by the duplicates ascending (model/attn_bias.py:828-837).
    Returns (kv_num [H,QB] int32, kv_packed [H,QB,MAX_KV] int32)."""
    s = np.sort(np.asarray(kv_blocks, np.int64), axis=-1)
    keep = np.ones(s.shape, dtype=bool)
    keep[..., 1:] = s[..., 1:] != s[..., :-1]
    num = keep.sum(-1).astype(np.int32)
    big = QB + 1
    key = (~keep).astype(np.int64) * big + s
    order = np.argsort(key, axis=-1, kind="stable")
    packed = np.take_along_axis(s, order, axis=-1)
    return num, packed.astype(np.int32)


def flex_padded(kv_packed, QB: int):
    """Pad/truncate the packed list to QB columns as the reference does
    before BlockMask.from_kv_blocks (model/attn_bias.py:854-862)."""
    kp = np.asarray(kv_packed, np.int32)
    H, _, W = kp.shape
    if W >= QB:
        return np.ascontiguousarray(kp[..., :QB])
    out = np.empty((H, QB, QB), dtype=np.int32)
    out[..., :W] = kp
    out[..., W:] = kp[..., :1]
    return out


def transpose_ordered(kv_num, kv_idx):
    """torch BlockMask._transpose_ordered: dense [rows, cols] 0/1 from the
    valid prefixes, transposed, then (row count, stable descending argsort)
    -> q_num [H,KB], q_idx [H,KB,QB] (valid q-blocks ascending, then the
    rest ascending)."""
    kv_num = np.asarray(kv_num)
    kv_idx = np.asarray(kv_idx)
    H, QB, W = kv_idx.shape
    KB = W
    dense = np.zeros((H, QB, KB), dtype=np.int32)
    for h in range(H):
        for q in range(QB):
            n = int(kv_num[h, q])
            dense[h, q, kv_idx[h, q, :n]] = 1
    dt = np.swapaxes(dense, 1, 2)          # [H, KB, QB]
    q_num = dt.sum(-1).astype(np.int32)
    q_idx = np.argsort(-dt, axis=-1, kind="stable").astype(np.int32)
    return q_num, q_idx


# ---------------------------------------------------------------------------
# whole builder
# ---------------------------------------------------------------------------
def build_pointer_blockmask(*, docs, block_size: int, M: int,
                            budget_rep, delta_rep=None, centres=None,
                            local_blocks: int, half_blocks: int, half_active: int | None = None,
                            ptr_enabled: bool = True, global_blocks_max: int = 0,
                            global_active: int | None = None,
                            radius_mode: str = "pi", budget_blocks: int = 0,
                            budget_is_total: bool = True, budget_temp: float = 1.0,
                            gumbel_k: int = 0, gumbel_tau: float = 1.0, gumbel_g=None,
                            doc_clamp: bool = True, reset_active: bool = False, reset_len: int = 0,
                            with_transpose: bool = True):
    """Restatement of SpectralBias.build_pointer_blockmask with every knob explicit.

    Exactly one of ``delta_rep`` (representative Δ* [H,QB,M] float32) or
    ``centres`` (pointer centre blocks [H,QB,M], from select_pointer_blocks)
    is given.  ``gumbel_k > 0`` with ``gumbel_g`` applies the reference's
    Gumbel peak masking (training mode only in the reference).  Returns a dict
    with kv_num, kv_packed, kv_indices (flex-padded), r_m, margin and, if
    requested, q_num / q_indices.
    """
    docs = np.asarray(docs)
    T = docs.shape[0]
    QB = T // block_size
    lb = min(max(1, int(local_blocks)), QB)
    p = max(0, int(half_blocks))
    ha = p if half_active is None else int(half_active)
    dsp, dsl = doc_start_blocks(docs, block_size, doc_clamp=doc_clamp,
                                reset_active=reset_active, reset_len=reset_len)
    brem = resolve_budget_rem(M=M, local_blocks=lb, half_blocks=p,
                              budget_blocks=budget_blocks, budget_is_total=budget_is_total)
    r_m, margin = radius_alloc(budget_rep, mode=radius_mode, budget_rem=brem,
                               budget_temp=budget_temp, half_blocks=p, half_active=ha,
                               ptr_enabled=ptr_enabled)
    if gumbel_k and p > 0 and gumbel_g is not None:
        r_m = gumbel_peak_mask(r_m, budget_rep, gumbel_g, k=gumbel_k, tau=gumbel_tau)
    if delta_rep is not None:
        c = centres_from_delta(delta_rep, block_size, dsp, ptr_enabled=ptr_enabled)
    else:
        c = clamp_centres(centres, dsp, ptr_enabled=ptr_enabled)
    gmax = min(int(global_blocks_max), QB)
    ga = gmax if global_active is None else int(global_active)
    kvb = window_pieces(c, r_m, dsp, dsl, QB=QB, local_blocks=lb, half_blocks=p,
                        global_max=gmax, global_active=ga)
    num, packed = dedup_pack(kvb, QB)
    out = dict(kv_num=num, kv_packed=packed, kv_indices=flex_padded(packed, QB),
               r_m=r_m, margin=margin, centres=c, dsp=dsp, dsl=dsl, max_kv=kvb.shape[-1])
    if with_transpose:
        out["q_num"], out["q_indices"] = transpose_ordered(num, out["kv_indices"])
    return out


def pointer_stats(kv_num, r_m, *, max_kv: int, half_blocks: int, M: int):
    """Pointer statistics the reference keeps in its debug buffers
    (model/attn_bias.py:839-849): kv_unique_hist, ptr_radius_hist,
    ptr_extra_sum_hist and the count of zero radii."""
    kv_hist = np.bincount(np.asarray(kv_num).ravel(), minlength=max_kv + 1)[: max_kv + 1]
    # the reference's radius buffer has half_blocks+1 bins; radii above can only
    # come from a schedule cap above the call's half width and land in the top bin
    rad = np.clip(np.asarray(r_m).ravel(), 0, half_blocks)
    pr_hist = np.bincount(rad, minlength=half_blocks + 1)[: half_blocks + 1]
    max_extra = max(1, half_blocks * M)
    es = np.minimum(np.asarray(r_m).sum(-1), max_extra).ravel()
    ex_hist = np.bincount(es, minlength=max_extra + 1)[: max_extra + 1]
    zero = int((rad == 0).sum())
    return kv_hist.astype(np.int64), pr_hist.astype(np.int64), ex_hist.astype(np.int64), zero
