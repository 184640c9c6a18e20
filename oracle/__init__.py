"""CPU oracle for the ats-v2 hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of the reference's PyTorch
path for RMSNorm, rotary embedding and the MoE layer (router, permutation,
SwiGLU experts, combine, auxiliary loss), forward and backward.  Each function
cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA library in ``ats_v2_b200`` never calls into this package and fails
loudly when its shared library is missing.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by running the reference's own modules
(``tests/golden/make_golden.py``).

Numerics: values are carried as float32 numpy arrays.  Where the reference
computes in bfloat16, the oracle rounds to bfloat16 (round-to-nearest-even)
at the same points the reference's torch ops round, so a bf16 tensor is a
float32 array whose values are all bf16-representable.
"""

from oracle.bf16 import round_bf16, bf16_bits_to_f32, f32_to_bf16_bits, round_to  # noqa: F401
