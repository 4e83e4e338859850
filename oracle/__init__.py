"""CPU oracle for the SCOPE sparse-attention hot path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the algorithm of
the reference implementation (onetensor/scope) so that the CUDA kernels in
``scope_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and only as the checker.  The product path never routes through
this package and has no CPU fallback.

Modules:
  mask_oracle  -- numpy restatement of ``SpectralBias.build_pointer_blockmask``
                  (model/attn_bias.py:623-874) plus the Gumbel top-k pointer
                  selection stage used by the benchmark configurations, and
                  torch's ``BlockMask`` q-side transpose.
  attn_oracle  -- dense float64 torch restatement of the block-sparse,
                  document-causal flex_attention call with the spectral
                  score_mod (scoped_medium.py:425-466) and the qk_aug mode
                  (scoped_medium.py:380-423), forward and autograd backward.

Parity pinning: the restatements are checked against golden fixtures produced
by running the reference code itself (``tests/golden/gen_golden.py``).
"""
