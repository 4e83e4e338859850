"""Host-side checks that need no GPU: the C-ABI library loads, exports every
symbol the header declares, its struct layouts match the ctypes mirror, and
argument validation rejects bad calls before touching the device."""
import ctypes
import os
import re

import pytest

import scope_b200
from scope_b200 import _lib
from scope_b200.attention import aug_dims

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "scope_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(scope_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = scope_b200.load_library()
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_struct_layouts_match():
    _lib.check_abi()


def test_error_strings():
    L = _lib.lib()
    assert L.scope_error_string(0) == b"ok"
    assert L.scope_error_string(-1) == b"invalid argument"
    assert L.scope_error_string(-6) == b"workspace missing or too small"
    assert L.scope_error_string(-99) == b"unknown status"


def test_validation_rejects_before_launch():
    L = _lib.lib()
    a = _lib.ScopeAttnArgs()
    assert L.scope_attn_fwd(ctypes.byref(a), None) == -1          # empty args
    a.H, a.T, a.D, a.block_size, a.dtype = 2, 256, 32, 128, 1
    assert L.scope_attn_fwd(ctypes.byref(a), None) == -1          # head_dim 32
    a.D, a.dtype = 64, 7
    assert L.scope_attn_fwd(ctypes.byref(a), None) == -2          # dtype
    m = _lib.ScopeMaskArgs()
    assert L.scope_mask_build(ctypes.byref(m), None) == -1
    m.H, m.QB, m.M, m.block_size = 1, 4, 17, 128
    assert L.scope_mask_build(ctypes.byref(m), None) == -1        # M > 16
    assert L.scope_block_info(None, 100, 128, 1, 0, 0, None, None) == -1
    b = _lib.ScopeAttnArgs()
    assert L.scope_block_mass(ctypes.byref(b), None, None) == -1  # no output
    assert L.scope_block_mass(ctypes.byref(b), 16, None) == -1    # empty args
    b.H, b.T, b.D, b.block_size, b.dtype, b.q, b.k = 2, 256, 64, 128, 0, 16, 16
    assert L.scope_block_mass(ctypes.byref(b), 16, None) == -2    # float32: bf16 only
    b.dtype, b.bias_mode, b.d_aug = 1, 2, 24
    assert L.scope_block_mass(ctypes.byref(b), 16, None) == -1    # d_aug not a multiple of 16
    b.bias_mode = 1
    assert L.scope_block_mass(ctypes.byref(b), 16, None) == -1    # score_mod closure: not the teacher's form
    assert L.scope_qk_aug_prepare(None, None, None, None, None, 0, 1, 1, 1, 16, 0.5, 0.12, 1, None, None, None) == -1
    # the backward's workspace: delta and lse2 [H, T], the fp32 dQ accumulator
    # [H, T, 64 + d_aug] and slope sums [H, T], the work plan
    a2 = _lib.ScopeAttnArgs()
    a2.H, a2.T, a2.block_size = 16, 131072, 128
    a2.bias_mode, a2.d_aug = 2, 32
    ws = L.scope_workspace_bytes(ctypes.byref(a2))
    assert 16 * 131072 * (2 * 4 + 96 * 4 + 4) <= ws < 16 * 131072 * (2 * 4 + 96 * 4 + 4) + (16 << 20)
    assert ws > L.scope_static_scratch_bytes()           # config 3 is beyond the static scratch
    a2.H, a2.T = 2, 2048
    assert L.scope_workspace_bytes(ctypes.byref(a2)) < L.scope_static_scratch_bytes()


def test_mask_max_kv():
    L = _lib.lib()
    assert L.scope_mask_max_kv(8, 8, 4, 1) == 8 + 8 * 9 + 1
    assert L.scope_mask_max_kv(8, 4, 0, 1) == 13


def test_aug_dims():
    assert aug_dims(8, False) == 16 and aug_dims(8, True) == 32
    assert aug_dims(16, False) == 32 and aug_dims(16, True) == 48


def test_ops_registered():
    import torch
    assert hasattr(torch.ops.scope, "sparse_attn")
    assert hasattr(torch.ops.scope, "sparse_attn_bwd")


def test_coefficient_entry_points_reject_bad_arguments():
    """Validation happens before any launch, so it runs without a GPU."""
    import ctypes
    import torch
    from scope_b200 import _lib, spectral_coefficients
    L = _lib.lib()
    a = _lib.ScopeCoeffArgs()                      # all zero: no shape, no pointers
    assert L.scope_spectral_coeffs(ctypes.byref(a), None) == -1
    a.H, a.T, a.D, a.hidden, a.K, a.M = 2, 100, 64, 128, 16, 8   # T not a multiple of 128
    assert L.scope_spectral_coeffs(ctypes.byref(a), None) == -1
    b = _lib.ScopeCoeffBwdArgs()
    assert L.scope_spectral_coeffs_bwd(ctypes.byref(b), None) == -1
    assert L.scope_spectral_coeffs(None, None) == -1 and L.scope_spectral_coeffs_bwd(None, None) == -1
    with pytest.raises(TypeError):                 # a CPU q is refused on the host side
        spectral_coefficients(torch.zeros(1, 2, 128, 64, dtype=torch.bfloat16), torch.zeros(128, 64),
                              torch.zeros(128), torch.zeros(41, 128), torch.zeros(41), omegas=torch.ones(16), M=8,
                              delta_cap=127.0, logw_min=-5.0, logw_max=-1.0)


@pytest.mark.parametrize("cuts", [(), (100, 300, 301, 560)])
def test_bench_torch_builder_ops_match_oracle(cuts):
    """The flex arm of the bench times the reference builder's steps as eager
    torch ops; they give the oracle's lists, with and without documents."""
    import numpy as np
    import torch

    import bench
    from oracle import mask_oracle as MO
    H, QB, M, L, p, G, bud, bs = 2, 48, 6, 4, 3, 2, 40, 16
    g = torch.Generator().manual_seed(1)
    lg, gu = torch.randn(H, QB, QB, generator=g), torch.randn(H, QB, QB, generator=g)
    br = torch.randn(H, QB, M, generator=g)
    d = np.zeros(QB * bs, np.int64)
    d[list(cuts)] = 1
    docs = np.cumsum(d)
    brem = MO.resolve_budget_rem(M=M, local_blocks=L, half_blocks=p, budget_blocks=bud, budget_is_total=True)
    num, packed = bench.torch_builder_ops(lg, gu, br, tau=0.5, M=M, L=L, p=p, G=G, budget_rem=brem, temp=0.7,
                                          docs=torch.from_numpy(docs), block_size=bs)
    cen = MO.select_pointer_blocks(lg.numpy(), gu.numpy(), M=M, tau=0.5)
    o = MO.build_pointer_blockmask(docs=docs, block_size=bs, M=M, budget_rep=br.numpy(),
                                   centres=cen, local_blocks=L, half_blocks=p, global_blocks_max=G,
                                   budget_blocks=bud, budget_is_total=True, budget_temp=0.7, with_transpose=False)
    assert np.array_equal(o["kv_num"], num.numpy())
    for h in range(H):
        for q in range(QB):
            n = int(num[h, q])
            assert np.array_equal(o["kv_packed"][h, q, :n], packed[h, q, :n].numpy())


def test_teacher_block_mass_rejects_bad_inputs():
    """Argument checks of teacher_block_mass, before any device work."""
    import torch

    from scope_b200 import teacher_block_mass
    q = torch.zeros(2, 256, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        teacher_block_mass(q, q, scale=0.12)                              # CPU tensors
    with pytest.raises(TypeError):
        teacher_block_mass(q.float(), q.float(), scale=0.12)              # bf16 only
    with pytest.raises(ValueError):
        teacher_block_mass(q, q[:1], scale=0.12)                          # q and k differ
    with pytest.raises(ValueError):
        teacher_block_mass(q[:, :200], q[:, :200], scale=0.12)            # T not a multiple of 128
