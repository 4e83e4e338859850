"""Generate golden fixtures by running the reference implementation on the CPU.

Usage (in a checkout that has the reference sources):

    CXX=/usr/bin/g++ python tests/golden/gen_golden.py --reference <path-to-onetensor-scope>

* Mask fixtures: ``SpectralBias.build_pointer_blockmask`` (model/attn_bias.py:623-874)
  run unmodified, with its Gumbel noise drawn from the same seeded generator
  the reference uses (model/attn_bias.py:768-771) and recorded as g.
* Attention fixtures: ``torch.compile(flex_attention)`` on the CPU (Inductor's
  C++ flex template), called the way scoped_medium.py:459-466 calls it with a
  scalar-form restatement of the score_mod closure of scoped_medium.py:425-457
  (the vectorised closure does not lower in Inductor; the scalar form is the
  same arithmetic), and the qk_aug augmentation of scoped_medium.py:380-423.
  Eager flex_attention is not used: it ignores the BlockMask's kv lists.
  The CPU flex path returns no lse (``return_lse`` is unsupported there), so
  only the outputs are pinned; lse is pinned through the float64 restatement.

* Coefficient fixtures: ``SpectralBias.forward`` (model/attn_bias.py:419-478)
  in eval mode and its ``_mlp_forward`` on seeded q and MLP weights.
* Teacher fixtures: the teacher's no-grad block (scoped_medium.py:1761-1819),
  its source lines executed unmodified on seeded inputs.

Outputs: tests/golden/mask_<case>.npz, attn_<case>.npz, coeff_<case>.npz and
teacher_<case>.npz.
The reference is read only at generation time; the tests never import it.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import cases as C  # noqa: E402
from oracle import mask_oracle as MO  # noqa: E402
from oracle import attn_oracle as AO  # noqa: E402

SMALL = 1 << 16


def make_sb(SpectralBias, case, H):
    sb = SpectralBias(
        head_dim=64, num_heads=H, L_train=max(case["T"], 256), K=2, M=case["M"],
        use_pointer_mask=True,
        pointer_local_blocks=case["local"], pointer_half_blocks=case["half"],
        pointer_global_blocks=case["glob"], pointer_budget_blocks=case["budget"],
        pointer_budget_is_total=case["total"], pointer_budget_temp=case["temp"],
        pointer_radius_mode=case["mode"], pointer_qblock_rep=case.get("rep", "last"),
        pointer_doc_clamp=case.get("doc_clamp", True),
        gumbel_topk=bool(case.get("gumbel_k", 0)), gumbel_topk_k=case.get("gumbel_k", 0),
        gumbel_topk_tau=case.get("gumbel_tau", 1.0), gumbel_topk_seed=case.get("gumbel_seed", 0),
        pointer_reset_len=case.get("reset_len", 0),
    )
    sb.set_pointer_mask_state(enabled=case.get("ptr_enabled", True),
                              half_blocks=case.get("half_active", case["half"]),
                              global_blocks=case.get("glob_active", case["glob"]))
    if case.get("reset_len", 0):
        sb.set_pointer_reset_state(enabled=True, reset_len=case["reset_len"])
    if case.get("gumbel_k", 0):
        sb.train()
    else:
        sb.eval()
    return sb


def run_mask_case(SpectralBias, name, case):
    H, T, bs, M = case["H"], case["T"], case["bs"], case["M"]
    QB = T // bs
    docs = C.mask_docs(case)
    t_rep = (np.arange(QB) + 1) * bs - 1
    if case["source"] == "select":
        logits, g = C.selection_inputs(case)
        centres = MO.select_pointer_blocks(logits, g, M=M, tau=case["sel_tau"])
        budget = C.budget_only(case)
        delta = np.zeros((1, H, T, M), dtype=np.float32)
        delta[0, :, t_rep, :] = (t_rep[None, :, None] - centres.astype(np.int64) * bs).astype(np.float32).transpose(1, 0, 2)
        in_hash = C.input_hash(logits, g, budget, docs)
    else:
        delta, budget = C.delta_budget_inputs(case)
        centres = None
        in_hash = C.input_hash(delta, budget, docs)
    pi = np.full((1, H, T, M), 1.0 / M, dtype=np.float32)
    sb = make_sb(SpectralBias, case, H)
    gumbel_g = None
    if case.get("gumbel_k", 0):
        gen = torch.Generator(device="cpu")
        gen.manual_seed(int(case.get("gumbel_seed", 0)))
        u = torch.rand((H, QB, M), generator=gen, dtype=torch.float32)
        gumbel_g = (-torch.log(-torch.log(u + 1e-9) + 1e-9)).numpy()
    bm = sb.build_pointer_blockmask(docs=torch.from_numpy(docs), delta_star=torch.from_numpy(delta),
                                    pi=torch.from_numpy(pi), budget_logits=torch.from_numpy(budget),
                                    block_size=bs)
    kv_num = bm.kv_num_blocks[0].numpy()
    kv_idx = bm.kv_indices[0].numpy()
    q_num = bm.q_num_blocks[0].numpy()
    q_idx = bm.q_indices[0].numpy()
    # representatives as the reference forms them (model/attn_bias.py:714-719)
    dt = torch.from_numpy(delta)[0]
    bt = torch.from_numpy(budget)[0]
    if case.get("rep", "last") == "last":
        delta_rep = dt[:, torch.from_numpy(t_rep)].numpy()
        budget_rep = bt[:, torch.from_numpy(t_rep)].numpy()
    else:
        delta_rep = dt.reshape(H, QB, bs, M).mean(dim=2).numpy()
        budget_rep = bt.reshape(H, QB, bs, M).mean(dim=2).numpy()
    out = dict(in_hash=np.array(in_hash), kv_num=kv_num, q_num=q_num,
               kv_indices_hash=np.array(C.arr_hash(kv_idx)), q_indices_hash=np.array(C.arr_hash(q_idx)))
    if gumbel_g is not None:
        out["gumbel_g"] = gumbel_g
    if not case.get("large"):
        out["delta_rep"] = delta_rep.astype(np.float32)
        out["budget_rep"] = budget_rep.astype(np.float32)
        if kv_idx.size <= SMALL:
            out["kv_indices"] = kv_idx
            out["q_indices"] = q_idx
        else:
            max_kv = case["local"] + (M * (2 * case["half"] + 1) if case["half"] > 0 else M) + min(case["glob"], QB)
            w = min(max_kv, QB)
            out["kv_indices_prefix"] = kv_idx[..., :w]
    np.savez_compressed(os.path.join(HERE, f"mask_{name}.npz"), **out)
    print(f"mask {name}: QB={QB} sum(kv_num)={int(kv_num.sum())}")


def scalar_score_mod(cc, cs, cos_wD, sin_wD, b0, slope, dm, wd, *, K, beta, gate, lam, tau):
    """Scalar-index form of the score_mod closure of scoped_medium.py:425-457
    (per-frequency accumulation in the same order)."""
    def score_mod(score, b, h, q_idx, kv_idx):
        delta = torch.clamp(q_idx - kv_idx, min=0)
        bias = torch.zeros_like(score)
        for kk in range(K):
            bias = bias + cc[b, h, q_idx, kk] * cos_wD[kk, delta] + cs[b, h, q_idx, kk] * sin_wD[kk, delta]
        df = delta.to(torch.float32)
        if b0 is not None:
            bias = bias - b0[b, h, q_idx]
        if slope is not None:
            bias = bias + slope[b, h, q_idx] * df
        if gate != "none" and lam > 0:
            x = ((df - dm[b, h, q_idx]).abs() - wd[b, h, q_idx]) / tau
            if gate == "relu":
                bias = bias - lam * torch.relu(x)
            else:
                bias = bias - lam * torch.nn.functional.softplus(x)
        return score + beta * bias
    return score_mod


def run_attn_case(SpectralBias, name, case):
    from torch.nn.attention.flex_attention import flex_attention
    H, T, bs, K = case["H"], case["T"], case["bs"], case["K"]
    QB = T // bs
    x = C.attn_inputs(case)
    docs = torch.from_numpy(C.attn_docs(case))
    kn = C.attn_mask_knobs(case)
    mcase = dict(H=H, T=T, bs=bs, M=kn["M"], local=kn["local"], half=kn["half"], glob=kn["glob"],
                 budget=kn["budget"], total=kn["total"], temp=kn["temp"], mode="pi", seed=case["seed"])
    sb = make_sb(SpectralBias, mcase, H)
    g = torch.Generator().manual_seed(case["seed"] + 5)
    delta = torch.rand(1, H, T, kn["M"], generator=g) * T * 0.8
    budget = torch.randn(1, H, T, kn["M"], generator=g)
    pi = torch.full((1, H, T, kn["M"]), 1.0 / kn["M"])
    bm = sb.build_pointer_blockmask(docs=docs, delta_star=delta, pi=pi, budget_logits=budget, block_size=bs)
    cos_wD, sin_wD = AO.trig_tables(x["omegas"], T)
    scale, beta, lam, tau = 0.12, 0.5, 0.2, 64.0
    fa = torch.compile(flex_attention, dynamic=False)
    q, k, v = (x[n][None] for n in ("q", "k", "v"))
    if case["impl"] == "score_mod":
        sm = scalar_score_mod(x["coeff_cos"][None], x["coeff_sin"][None], cos_wD, sin_wD,
                              x["b0"][None] if case["b0"] else None,
                              x["slope"][None] if case["slope"] else None,
                              x["delta_main"][None], x["width"][None], K=K, beta=beta,
                              gate=case["gate"], lam=lam, tau=tau)
        out = fa(q, k, v, block_mask=bm, score_mod=sm, scale=scale)
    else:
        qa, ka, va = AO.qk_aug_inputs(x["q"], x["k"], x["v"], x["coeff_cos"], x["coeff_sin"], cos_wD, sin_wD,
                                      beta=beta, scale=scale, slope=x["slope"] if case["slope"] else None)
        out = fa(qa[None], ka[None], va[None], block_mask=bm, scale=scale)
        out = out[..., :64]
    rows = np.linspace(0, T - 1, C.ATTN_ROWS).astype(np.int64)
    np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"),
                        out_rows=out[0][:, rows].float().numpy(), rows=rows,
                        kv_num=bm.kv_num_blocks[0].numpy(), kv_indices=bm.kv_indices[0].numpy(),
                        delta_rep=delta[0][:, (torch.arange(QB) + 1) * bs - 1].numpy(),
                        budget_rep=budget[0][:, (torch.arange(QB) + 1) * bs - 1].numpy(),
                        in_hash=np.array(C.input_hash(*(x[n].numpy() for n in sorted(x)))))
    print(f"attn {name}: done")


def reference_teacher_source(reference):
    """The body of the teacher's no-grad block (scoped_medium.py:1761-1819:
    the augmented dims, then the per-query-block dense softmax and its
    scatter into kv blocks), read from the reference file and dedented."""
    import textwrap
    with open(os.path.join(reference, "scoped_medium.py")) as f:
        src = f.read().splitlines()
    head = next(i for i, ln in enumerate(src) if "teacher dense attention" in ln)
    start = next(i for i in range(head, len(src)) if "q_bhtd = q.transpose(1, 2)" in src[i])
    end = next(i for i in range(start, len(src)) if "teacher_mass[:, qb, :] = mass" in src[i])
    return textwrap.dedent("\n".join(src[start:end + 1]))


def run_teacher_case(reference, name, case):
    """Runs the reference's teacher block unmodified in a namespace holding its
    free variables: q, k [1, T, H, 64], the coefficient block's outputs
    [1, H, T, K], the bf16 trig tables, docs, and stand-ins for ``sb``,
    ``args`` and ``attn`` carrying the knobs it reads."""
    import types
    H, T, K = case["H"], case["T"], case["K"]
    dt = getattr(torch, case["dtype"])
    x = C.attn_inputs(dict(H=H, T=T, K=K, seed=case["seed"]))
    docs = torch.from_numpy(C.attn_docs(dict(T=T, docs=case["docs"])))
    cos_wD, sin_wD = AO.trig_tables(x["omegas"], T)
    scale, beta = 0.12, 0.5
    ns = dict(torch=torch, math=math, device=torch.device("cpu"), teacher_len=T, docs=docs,
              q=x["q"].to(dt).transpose(0, 1)[None], k=x["k"].to(dt).transpose(0, 1)[None],
              coeff_cos=x["coeff_cos"][None], coeff_sin=x["coeff_sin"][None], slope=x["slope"][None],
              cos_wD=cos_wD, sin_wD=sin_wD,
              _select_teacher_heads=lambda nh, dev: torch.arange(nh, device=dev),
              sb=types.SimpleNamespace(use_slope=case["slope"], beta=beta, K=K),
              args=types.SimpleNamespace(spectral_bias=case["spectral"]),
              attn=types.SimpleNamespace(num_heads=H, attn_scale=scale))
    exec(compile(reference_teacher_source(reference), "scoped_medium.py:teacher", "exec"), ns)
    out = dict(q=x["q"].to(dt).float().numpy(), k=x["k"].to(dt).float().numpy(), docs=docs.numpy(),
               scale=np.array(scale, np.float32), mass=ns["teacher_mass"].numpy())
    if case["spectral"]:
        out["q_pos"] = ns["q_pos"].float().numpy()
        out["k_pos"] = ns["k_pos"].float().numpy()
    np.savez_compressed(os.path.join(HERE, f"teacher_{name}.npz"), **out)
    print(f"teacher {name}: done")


COEFF_OUTS = ("coeff_cos", "coeff_sin", "slope", "b0", "delta_star", "pi", "budget_logits", "delta_main", "width")


def run_coeff_case(SpectralBias, name, case):
    """SpectralBias.forward in eval mode (no regularisers) and its _mlp_forward,
    with the case's weights loaded into the module's float32 parameters
    (bf16-representable, so the module's cast to bf16 is exact)."""
    x = C.coeff_inputs(case)
    H, T, K, M = case["H"], case["T"], case["K"], case["M"]
    sb = SpectralBias(head_dim=64, num_heads=H, L_train=case["L_train"], K=K, M=M,
                      share_across_heads=case["share"], use_slope=case["use_slope"],
                      subtract_b0=case["subtract_b0"], delta_star_max=case["delta_star_max"])
    with torch.no_grad():
        if case["share"]:
            sb.mlp[0].weight.copy_(torch.from_numpy(x["w1"][0]))
            sb.mlp[0].bias.copy_(torch.from_numpy(x["b1"][0]))
            sb.mlp[2].weight.copy_(torch.from_numpy(x["w2"][0]))
            sb.mlp[2].bias.copy_(torch.from_numpy(x["b2"][0]))
        else:
            sb.w1.copy_(torch.from_numpy(x["w1"]))
            sb.b1.copy_(torch.from_numpy(x["b1"]))
            sb.w2.copy_(torch.from_numpy(x["w2"]))
            sb.b2.copy_(torch.from_numpy(x["b2"]))
    sb.eval()
    q = torch.from_numpy(x["q"]).to(torch.bfloat16).requires_grad_(True)
    outs = sb(q)
    with torch.no_grad():
        y = sb._mlp_forward(q).float()
    res = {n: outs[i].detach().float().numpy() for i, n in enumerate(COEFF_OUTS)}
    # the backward from seeded upstream gradients of all nine outputs
    ups = C.coeff_upstream(case)
    live = [i for i in range(len(COEFF_OUTS)) if outs[i].requires_grad]   # slope / b0 are constants when off
    torch.autograd.backward([outs[i] for i in live], [torch.from_numpy(ups[i]) for i in live])
    if case["share"]:
        wg = [sb.mlp[0].weight.grad[None], sb.mlp[0].bias.grad[None], sb.mlp[2].weight.grad[None],
              sb.mlp[2].bias.grad[None]]
    else:
        wg = [sb.w1.grad, sb.b1.grad, sb.w2.grad, sb.b2.grad]
    res.update(dq=q.grad.float().numpy(), **{n: t.numpy() for n, t in zip(("dw1", "db1", "dw2", "db2"), wg)})
    # training mode: the regularisers join reg_loss (model/attn_bias.py:480-506); backward
    # from the same upstream gradients plus 1 on reg_loss
    sb.zero_grad(set_to_none=True)
    sb.train()
    qt = torch.from_numpy(x["q"]).to(torch.bfloat16).requires_grad_(True)
    outs = sb(qt)
    live = [i for i in range(len(COEFF_OUTS)) if outs[i].requires_grad]
    torch.autograd.backward([outs[i] for i in live] + [outs[11]],
                            [torch.from_numpy(ups[i]) for i in live] + [torch.ones(())])
    if case["share"]:
        wg = [sb.mlp[0].weight.grad[None], sb.mlp[0].bias.grad[None], sb.mlp[2].weight.grad[None],
              sb.mlp[2].bias.grad[None]]
    else:
        wg = [sb.w1.grad, sb.b1.grad, sb.w2.grad, sb.b2.grad]
    res.update(t_reg=outs[11].detach().numpy(), t_dq=qt.grad.float().numpy(),
               **{"t_" + n: t.numpy() for n, t in zip(("dw1", "db1", "dw2", "db2"), wg)})
    # the gradients of reg_loss alone (the regularisers' share is far below the others')
    sb.zero_grad(set_to_none=True)
    qr = torch.from_numpy(x["q"]).to(torch.bfloat16).requires_grad_(True)
    outs = sb(qr)
    outs[11].backward()
    if case["share"]:
        wg = [sb.mlp[0].weight.grad[None], sb.mlp[0].bias.grad[None], sb.mlp[2].weight.grad[None],
              sb.mlp[2].bias.grad[None]]
    else:
        wg = [sb.w1.grad, sb.b1.grad, sb.w2.grad, sb.b2.grad]
    res.update(r_dq=qr.grad.float().numpy(), **{"r_" + n: t.numpy() for n, t in zip(("dw1", "db1", "dw2", "db2"), wg)})
    sb.eval()
    np.savez_compressed(os.path.join(HERE, f"coeff_{name}.npz"), **res, y=y.numpy(),
                        omegas=sb.omegas.numpy(), log_omegas=sb.log_omegas.numpy(),
                        logw_min=sb.logw_min.numpy(), logw_max=sb.logw_max.numpy(),
                        delta_star_max=np.array(int(sb._delta_star_max_active)),
                        c_scale=np.array(sb.c_scale, np.float32), width_min=np.array(sb.width_min, np.float32),
                        width_max=np.array(sb.width_max, np.float32), eps=np.array(sb.eps, np.float32),
                        in_hash=np.array(C.input_hash(*(x[n] for n in sorted(x)))))
    print(f"coeff {name}: done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the onetensor/scope checkout")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from model.attn_bias import SpectralBias
    torch.set_num_threads(os.cpu_count() or 1)
    for name, case in C.MASK_CASES.items():
        if a.only and a.only not in name:
            continue
        run_mask_case(SpectralBias, name, case)
    for name, case in C.ATTN_CASES.items():
        if a.only and a.only not in name:
            continue
        run_attn_case(SpectralBias, name, case)
    for name, case in C.COEFF_CASES.items():
        if a.only and a.only not in name:
            continue
        run_coeff_case(SpectralBias, name, case)
    for name, case in C.TEACHER_CASES.items():
        if a.only and a.only not in name:
            continue
        run_teacher_case(a.reference, name, case)


if __name__ == "__main__":
    main()
