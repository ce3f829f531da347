"""MSDA CPU oracle -- TEST INFRASTRUCTURE ONLY.

Nothing in ``muspace_b200`` imports this package. It is the checker that the
parity tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` compare the CUDA path against:

* :mod:`oracle.msda_oracle` -- ctypes binding of ``msda_oracle.c``, a scalar C
  restatement of the reference kernel arithmetic (fp32 geometry, double sums).
* :mod:`oracle.msda_torch` -- the reference's PyTorch ``grid_sample``
  formulation restated on CPU tensors; it is the timed CPU baseline.
* :mod:`oracle.sca_scatter` -- the fused spatial-cross-attention scatter
  (MSDA forward + rebatch scatter + count normalisation) on top of the C oracle.

Both are pinned by the golden vectors in ``tests/golden/``, which were produced
by importing the muSPACE reference itself (``tests/golden/gen_golden.py``).
"""

from .msda_oracle import build, oracle_backward, oracle_forward  # noqa: F401
from .sca_scatter import oracle_scatter_div  # noqa: F401
