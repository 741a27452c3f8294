"""CPU oracle for the spiking hot path (test infrastructure only).

This package is a CPU restatement, in plain PyTorch fp32, of the reference
implementation of the spiking layers (flofiz/SpikingTransformer,
``Triton_Layers/*.py``).  It exists to check the CUDA path: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product package
(``spikingtransformer_b200``) never imports it and has no CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own modules
(its Triton LIF kernels executed by the Triton interpreter) on seeded inputs
and stores inputs, state dicts and outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against those fixtures.
"""

from .lif import lif_forward, lif_backward, superspike_grad, arctan_grad  # noqa: F401
from . import modules  # noqa: F401
