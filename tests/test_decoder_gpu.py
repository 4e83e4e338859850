"""The C4 decoder (scope_b200.decoder) on a small shape: one layer's SCOPE
attention against the float64 oracle evaluated on the layer's own q, k, v,
coefficients and mask (the glue of scoped_medium.py:334-479: QK norm,
rotary, value mixing, qk_aug with slope), and a few AdamW steps of the whole
model on one batch (finite gradients everywhere, the loss goes down)."""
import pytest
import torch

from oracle import attn_oracle as AO

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _small():
    from scope_b200.decoder import ScopeDecoder
    torch.manual_seed(0)
    return ScopeDecoder(vocab_size=1024, num_layers=6, model_dim=256, num_heads=4, head_dim=64, max_seq_len=2048,
                        K=8, M=4, local_blocks=4).to(DEV)


def test_decoder_layer_attention_matches_oracle():
    from scope_b200 import device_errors
    from scope_b200.decoder import norm
    model = _small()
    T = 2048
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, T, 256, generator=g).to(DEV, torch.bfloat16)
    ve = torch.randn(1, T, 256, generator=g).to(DEV, torch.bfloat16)
    docs = torch.zeros(T, dtype=torch.int32, device=DEV)
    docs[1300:] = 1
    attn = model.blocks[0].attn
    keep = {}
    device_errors(DEV)
    with torch.no_grad():
        out = attn.attend(norm(x), ve, docs, keep)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    bm = keep["mask"]
    c = lambda t: t[0].float().cpu()                               # noqa: E731
    q, k, v = (keep[n][0].transpose(0, 1).float().cpu() for n in ("q", "k", "v"))   # [H, T, D]
    qa, ka, va = AO.qk_aug_inputs(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
                                  c(keep["coeff_cos"]), c(keep["coeff_sin"]), keep["cos_tab"].cpu(),
                                  keep["sin_tab"].cpu(), beta=0.5, scale=0.12, slope=c(keep["slope"]))
    mask = AO.dense_mask(bm.kv_num_blocks[0].cpu().numpy(), bm.kv_indices[0].cpu().numpy(), T, 128,
                         docs=docs.cpu().numpy())
    ref, _ = AO.attention(qa.float(), ka.float(), va.float(), mask, scale=0.12)
    got = out[0].view(T, 4, 64).transpose(0, 1).float().cpu()
    assert (got - ref[..., :64]).abs().max().item() < 2e-2


def test_decoder_trains_a_few_steps():
    from scope_b200.decoder import synthetic_tokens
    model = _small()
    inp, tgt = synthetic_tokens(2048, 1024, seed=1, device=DEV)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3, betas=(0.9, 0.95), fused=True)
    losses = []
    for _ in range(6):
        opt.zero_grad(set_to_none=True)
        loss = model(inp, tgt)
        loss.backward()
        for n, p in model.named_parameters():
            assert p.grad is not None and torch.isfinite(p.grad).all(), n
        opt.step()
        losses.append(loss.item())
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]
