"""B200 (sm_100a) implementation of the spiking hot path of
flofiz/SpikingTransformer behind its ``Triton_Layers`` module surface.

Modules mirror the reference files: ``Lif``, ``SSA``, ``SpikingMLP``,
``Encoder``, ``Decoder``, ``ImageEncoder``, ``Seq2Seq``.  The compute runs in
``libspk.so`` (built by ``python -m spikingtransformer_b200.build``); there is
no CPU fallback.

``install_as_triton_layers()`` registers these modules under the reference
package name so ``from Triton_Layers.Seq2Seq import Seq2Seq`` resolves here.
"""

import importlib
import sys

__version__ = "0.1.0"

_MODULES = ("Lif", "SSA", "SpikingMLP", "Encoder", "Decoder", "ImageEncoder", "Seq2Seq")


def install_as_triton_layers():
    """Make ``import Triton_Layers.<module>`` load this package's modules."""
    pkg = sys.modules[__name__]
    sys.modules.setdefault("Triton_Layers", pkg)
    for name in _MODULES:
        mod = importlib.import_module("%s.%s" % (__name__, name))
        sys.modules["Triton_Layers.%s" % name] = mod
    return pkg
