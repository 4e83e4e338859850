"""Teacher block mass (scoped_medium.py:1793-1819) on the tensor cores against
the float64 oracle on the same bf16 inputs, and against the reference's own
teacher block run on bf16 inputs (the committed fixture).

Bounds: 4e-3 absolute per block against the oracle (mass values up to 128;
float32 scores and sums, MUFU / polynomial exp2); 0.05 against the reference
run, whose bf16 matmuls round every score to bf16 (the oracle itself is
0.011 from it on that fixture)."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import attn_oracle as AO
from scope_b200 import device_errors, teacher_block_mass

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bf(t):
    return t.to(torch.bfloat16)


def _aug(H, T, K, slope, seed, scale=0.12, beta=0.5):
    """The teacher's augmented dims (scoped_medium.py:1770-1787) for random
    coefficients and the reference's frequencies."""
    g = torch.Generator().manual_seed(seed)
    cc = 0.3 * torch.randn(H, T, K, generator=g)
    cs = 0.3 * torch.randn(H, T, K, generator=g)
    om = AO.reference_omegas(K, T, 1_000_000)
    ct, st = AO.trig_tables(om, T)
    ct, st = ct.T.float()[None].expand(H, T, K), st.T.float()[None].expand(H, T, K)
    qp = torch.cat([cc * ct + cs * st, cc * st - cs * ct], -1)
    kp = torch.cat([ct, st], -1)
    if slope:
        sl = 0.01 * torch.tanh(torch.randn(H, T, generator=g))
        pos = torch.arange(T, dtype=torch.float32)
        qp = torch.cat([qp, (-sl)[..., None]], -1)
        kp = torch.cat([kp, pos[None, :, None].expand(H, T, 1)], -1)
    s = math.sqrt(beta / scale)
    return _bf(qp * s), _bf(kp * s)


def _docs(T, cuts):
    d = np.zeros(T, np.int64)
    d[list(cuts)] = 1
    return torch.from_numpy(np.cumsum(d))


def _run(q, k, docs, qp, kp, scale):
    device_errors(DEV)
    m = teacher_block_mass(q.to(DEV), k.to(DEV), None if docs is None else docs.to(DEV), scale=scale,
                           q_pos=None if qp is None else qp.to(DEV), k_pos=None if kp is None else kp.to(DEV))
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    return m.cpu().double()


def _check_structure(m, docs, T):
    """Rows sum to 128; nothing above the diagonal; nothing before the
    document start block of the q block's first row."""
    QB = T // 128
    assert (m.sum(-1) - 128.0).abs().max().item() < 2e-3
    assert torch.triu(m, diagonal=1).abs().max().item() == 0.0
    if docs is not None:
        d = docs.numpy()
        for qb in range(QB):
            first = qb * 128
            start = first
            while start > 0 and d[start - 1] == d[first]:
                start -= 1
            if start >= 128:
                assert m[:, qb, : start // 128].abs().max().item() == 0.0


@pytest.mark.parametrize("K,slope,cuts", [(16, True, (700, 1024, 2500, 2900)), (8, False, ()), (4, True, (300,))])
def test_teacher_mass_matches_oracle(K, slope, cuts):
    T, H = 4096, 4
    g = torch.Generator().manual_seed(K + 7)
    q = _bf(torch.randn(H, T, 64, generator=g))
    k = _bf(torch.randn(H, T, 64, generator=g))
    qp, kp = _aug(H, T, K, slope, seed=K)
    docs = _docs(T, cuts) if cuts else None
    m = _run(q, k, docs, qp, kp, 0.12)
    ref = AO.teacher_block_mass(q.float(), k.float(), torch.zeros(T, dtype=torch.long) if docs is None else docs,
                                scale=0.12, q_pos=qp.float(), k_pos=kp.float())
    assert (m - ref).abs().max().item() < 4e-3
    _check_structure(m, docs, T)


def test_teacher_mass_without_bias_and_strided_heads():
    """No augmented dims; q and k as views of a [T, H, 64] tensor (the
    reference's q_bhtd[0, head_idx] layout)."""
    T, H = 2048, 3
    g = torch.Generator().manual_seed(5)
    qt = _bf(torch.randn(T, H, 64, generator=g)).to(DEV)
    kt = _bf(torch.randn(T, H, 64, generator=g)).to(DEV)
    docs = _docs(T, (129, 1000))
    device_errors(DEV)
    m = teacher_block_mass(qt.transpose(0, 1), kt.transpose(0, 1), docs.to(DEV), scale=0.125)
    torch.cuda.synchronize()
    assert device_errors(DEV) == 0
    ref = AO.teacher_block_mass(qt.transpose(0, 1).cpu().float(), kt.transpose(0, 1).cpu().float(), docs,
                                scale=0.125)
    assert (m.cpu().double() - ref).abs().max().item() < 4e-3
    _check_structure(m.cpu().double(), docs, T)


def test_teacher_mass_matches_reference_fixture():
    """The reference's teacher block on bf16 inputs (its training dtype)."""
    f = np.load(os.path.join(GOLD, "teacher_t_slope_multi_bf16.npz"))
    q, k = _bf(torch.from_numpy(f["q"])), _bf(torch.from_numpy(f["k"]))
    qp, kp = _bf(torch.from_numpy(f["q_pos"])), _bf(torch.from_numpy(f["k_pos"]))
    docs = torch.from_numpy(f["docs"])
    m = _run(q, k, docs, qp, kp, float(f["scale"]))
    ref = AO.teacher_block_mass(q.float(), k.float(), docs, scale=float(f["scale"]), q_pos=qp.float(),
                                k_pos=kp.float())
    assert (m - ref).abs().max().item() < 4e-3
    assert np.abs(m.numpy() - f["mass"]).max() < 0.05
