"""scope_b200: the SCOPE sparse-attention hot path, B200-native (sm_100a).

Replaces, behind the reference's own interfaces:
  * SpectralBias.build_pointer_blockmask  -> PointerBlockMaskBuilder / build_mask
  * the spectral score_mod / qk_aug bias   -> SpectralScoreMod (evaluated in-kernel)
  * SpectralBias.forward's coefficient block -> SpectralCoefficients / spectral_coefficients
  * flex_attention(q, k, v, block_mask, score_mod, scale) -> flex_attention
  * the spectral teacher's dense block-mass loop        -> teacher_block_mass
Every op runs hand-written CUDA through the C ABI of libscope_b200.so
(include/scope_b200.h); there is no CPU fallback.
"""
from . import _lib
from .attention import SpectralScoreMod, aug_dims, flex_attention, trig_tables
from .coeff import CoeffOutputs, SpectralCoefficients, spectral_coefficients
from .mask import PointerBlockMaskBuilder, ScopeBlockMask, block_info, build_mask
from .teacher import teacher_block_mass
from ._lib import device_errors

__all__ = [
    "PointerBlockMaskBuilder", "ScopeBlockMask", "SpectralScoreMod", "aug_dims", "block_info", "build_mask",
    "flex_attention", "trig_tables", "load_library", "device_errors", "CoeffOutputs", "SpectralCoefficients",
    "spectral_coefficients", "teacher_block_mass",
]


def load_library():
    """Load libscope_b200.so and check the C struct layouts against ctypes."""
    _lib.lib()
    _lib.check_abi()
    return _lib.lib()
