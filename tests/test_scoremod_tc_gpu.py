"""The score_mod closure (scoped_medium.py:425-457) on the tensor cores: the
Fourier sum through augmented Q/K dims in the QK MMA; slope * Δ and the
softplus / relu gate per element in the softmax (forward) and elementwise
(backward) warps; dslope, dΔ_main and dwidth from per-query column sums of dS;
db0 = 0 (a per-row constant of the scores).  Checked against the float64
oracle of the closure and against the CUDA-core kernels on the same bf16
inputs.  Tolerance 2e-2 max-abs beyond the bf16 quantization of the output
(bias gradients: 2e-2 of their scale)."""
import math

import pytest
import torch

from oracle import attn_oracle as AO
from scope_b200 import SpectralScoreMod, device_errors, flex_attention, trig_tables
from test_attn_tc_gpu import _inputs, _maxabs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _extras(H, T, seed):
    g = torch.Generator().manual_seed(seed)
    return {"b0": 0.1 * torch.randn(H, T, generator=g),
            "slope": 0.01 * torch.tanh(torch.randn(H, T, generator=g)),
            "delta_main": torch.rand(H, T, generator=g) * 1500.0,
            "width": 32.0 + torch.rand(H, T, generator=g) * 224.0}


def _run(bm, x, ex, gate, do, *, cuda_cores=False, terms=("b0", "slope")):
    q, k, v = (x[n].transpose(0, 1).contiguous().to(DEV, torch.bfloat16).transpose(0, 1).requires_grad_(True)
               for n in ("q", "k", "v"))
    ct, st = trig_tables(x["omegas"].to(DEV), q.shape[1])
    leaf = lambda t: t.to(DEV).requires_grad_(True)  # noqa: E731
    lv = {"coeff_cos": leaf(x["coeff_cos"]), "coeff_sin": leaf(x["coeff_sin"])}
    for n in terms:
        lv[n] = leaf(ex[n])
    if gate != "none":
        lv["delta_main"], lv["width"] = leaf(ex["delta_main"]), leaf(ex["width"])
    sm = SpectralScoreMod(coeff_cos=lv["coeff_cos"], coeff_sin=lv["coeff_sin"], cos_tab=ct, sin_tab=st, beta=0.5,
                          b0=lv.get("b0"), slope=lv.get("slope"), delta_main=lv.get("delta_main"),
                          width=lv.get("width"), gate=gate, impl="score_mod")
    out, lse = flex_attention(q[None], k[None], v[None], bm, score_mod=sm, scale=0.12, return_lse=True,
                              cuda_cores=cuda_cores)
    out.backward(do.to(DEV, torch.bfloat16)[None])
    res = {"out": out[0], "lse": lse[0], "dq": q.grad, "dk": k.grad, "dv": v.grad}
    res.update({"d" + n: t.grad for n, t in lv.items()})
    return res


def _oracle(bm, x, ex, gate, do, docs, terms=("b0", "slope")):
    T = x["q"].shape[1]
    mask = AO.dense_mask(bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), T, 128,
                         docs=docs.numpy())
    rd = lambda t: t.to(torch.bfloat16).float()  # noqa: E731
    ct, st = AO.trig_tables(x["omegas"], T)
    g = AO.score_mod_grads(rd(x["q"]), rd(x["k"]), rd(x["v"]), rd(do), mask, scale=0.12, beta=0.5,
                           coeff_cos=x["coeff_cos"], coeff_sin=x["coeff_sin"], cos_tab=ct, sin_tab=st,
                           b0=ex["b0"] if "b0" in terms else None, slope=ex["slope"] if "slope" in terms else None,
                           delta_main=ex["delta_main"] if gate != "none" else None,
                           width=ex["width"] if gate != "none" else None, gate=gate)
    return g


def _half_ulp_bf16(x: float) -> float:
    """Half the bf16 spacing at magnitude x: what rounding the output alone costs."""
    return 0.0 if x <= 0 else 2.0 ** (math.floor(math.log2(x)) - 8)


def _check(res, ref, names):
    """out / lse / dq / dk / dv: 2e-2 max-abs beyond the bf16 quantization of
    the output (at |x| in [4, 8) rounding alone may cost 0.0156, which would
    leave 0.0044 of the bound); bias gradients (float32): 2e-2 of their scale."""
    for n in names:
        if n not in res or n not in ref:
            continue
        mx = ref[n].abs().max().item()
        if n in ("out", "dq", "dk", "dv"):
            bound = 2e-2 + _half_ulp_bf16(mx)
        elif n == "lse":
            bound = 2e-2
        else:
            bound = 2e-2 * max(1.0, mx)
        err = _maxabs(res[n], ref[n])
        assert err < bound, (n, err, bound)


@pytest.mark.parametrize("gate", ["none", "softplus", "relu"])
@pytest.mark.parametrize("K,docs_kind", [(8, "multi"), (16, "single")])
def test_scoremod_tc_matches_oracle(gate, K, docs_kind):
    T, H = 2048, 2
    bm, x, docs = _inputs(T, H, K, False, docs_kind, seed=21 + K)
    ex = _extras(H, T, seed=3)
    do = torch.randn(H, T, 64, generator=torch.Generator().manual_seed(8))
    device_errors(DEV)
    res = _run(bm, x, ex, gate, do)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    ref = _oracle(bm, x, ex, gate, do, docs)
    _check(res, ref, ("out", "lse", "dq", "dk", "dv", "dcoeff_cos", "dcoeff_sin", "dslope", "ddelta_main", "dwidth"))
    # b0 shifts every score of its row alike: its gradient vanishes
    assert res["db0"].abs().max().item() == 0.0
    assert ref["db0"].abs().max().item() < 1e-4


@pytest.mark.parametrize("gate", ["softplus", "relu"])
def test_scoremod_tc_long_lists_match_cuda_cores(gate):
    """Long kv lists and split dK/dV rows (T = 16384), against the CUDA-core
    score_mod kernels on the same inputs."""
    T, H = 16384, 2
    bm, x, docs = _inputs(T, H, 8, False, "multi", seed=4, M=8, half=3, local=8, glob=2)
    ex = _extras(H, T, seed=5)
    do = torch.randn(H, T, 64, generator=torch.Generator().manual_seed(9))
    a = _run(bm, x, ex, gate, do)
    b = _run(bm, x, ex, gate, do, cuda_cores=True)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    _check(a, b, [n for n in a if n != "db0"])


def test_scoremod_tc_without_slope_or_b0():
    """The closure with only the Fourier sum and the gate."""
    T, H = 2048, 2
    bm, x, docs = _inputs(T, H, 4, False, "single", seed=31)
    ex = _extras(H, T, seed=6)
    do = torch.randn(H, T, 64, generator=torch.Generator().manual_seed(10))
    res = _run(bm, x, ex, "softplus", do, terms=())
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    ref = _oracle(bm, x, ex, "softplus", do, docs, terms=())
    _check(res, ref, ("out", "lse", "dq", "dk", "dv", "dcoeff_cos", "dcoeff_sin", "ddelta_main", "dwidth"))
