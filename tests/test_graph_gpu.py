"""The layer step (fused pointer selection + mask build, attention forward
with the spectral bias, backward to q, k, v and the coefficients) captured
in a CUDA graph and replayed gives the eager step's results: the library
launches only on the caller's stream, allocates nothing itself and never
synchronises the host, so a whole step can be captured."""
import pytest
import torch

from scope_b200 import SpectralScoreMod, device_errors, flex_attention, trig_tables
from scope_b200.synth import BETA, CONFIGS, SCALE, build_config_mask, make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_graph_replay_of_a_layer_step_matches_eager():
    import dataclasses
    cfg = dataclasses.replace(CONFIGS["c3"], H=2, T=16384)
    x = make_inputs(cfg, device=DEV, seed=4)
    ct, st = trig_tables(x["omegas"], cfg.T)
    leaves = {n: x[n].detach().requires_grad_(True) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")}
    res = {}

    def step():
        for t in leaves.values():
            t.grad = None
        bm = build_config_mask(cfg, x)
        sm = SpectralScoreMod(coeff_cos=leaves["coeff_cos"], coeff_sin=leaves["coeff_sin"], cos_tab=ct, sin_tab=st,
                              beta=BETA, impl="qk_aug")
        out = flex_attention(leaves["q"][None], leaves["k"][None], leaves["v"][None], bm, score_mod=sm, scale=SCALE)
        out.backward(x["do"][None])
        res["out"] = out
        res["kv"] = bm.kv_indices
        return out

    device_errors(DEV)
    step()
    torch.cuda.synchronize()
    eager = {"out": res["out"].detach().clone(), "kv": res["kv"].clone()}
    eager.update({n: t.grad.clone() for n, t in leaves.items()})
    # no tensor may keep an eager step's autograd graph (and with it the leaves'
    # gradient-accumulation nodes, bound to the stream they ran on) alive into the capture
    res.clear()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
        res.clear()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    assert torch.equal(res["kv"], eager["kv"])
    assert torch.equal(res["out"].detach(), eager["out"])
    for n, t in leaves.items():
        tol = 1e-2 * max(1.0, eager[n].abs().max().item())
        assert (t.grad.float() - eager[n].float()).abs().max().item() <= tol, n
